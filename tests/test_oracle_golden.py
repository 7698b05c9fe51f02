"""The CPU oracle (oracle/mlp_oracle.py) against golden outputs of the reference's own PyTorch
models (tests/golden/*.npz, produced by tests/golden/make_golden.py)."""
import torch

from tests._util import load_golden, u16_to
from oracle import mlp_oracle as O
from tests.golden.make_golden import checksum, layer_params

TOL = dict(atol=2e-5, rtol=1e-5)


def _layers(g, dims, dtype=torch.float16, init="kaiming"):
    layers = layer_params(int(g["seed"]), list(dims), dtype=dtype, init=init)
    assert abs(checksum(layers) - float(g["wsum"])) < 1e-6, "weight generator drifted"
    return layers


def test_mgn_fullmlp_matches_reference_model():
    for name in ("mgn_fullmlp_k384", "mgn_fullmlp_k256"):
        g = load_golden(name)
        layers = _layers(g, g["dims"])
        x = u16_to(g["x"], torch.float16)
        ln = (u16_to(g["gamma"], torch.float16), u16_to(g["beta"], torch.float16))
        y = O.chain_forward(x, layers, [O.ACT_RELU, O.ACT_RELU, O.ACT_NONE], O.TAIL_LAYERNORM, ln, 1e-5)
        torch.testing.assert_close(y, torch.from_numpy(g["y"]), **TOL)
        torch.testing.assert_close(O.mgn_mlp(x, layers, ln), torch.from_numpy(g["y"]), **TOL)


def test_mgn_linears_and_testmlp_match_reference_model():
    for name in ("mgn_linears_k384", "testmlp_k128"):
        g = load_golden(name)
        layers = _layers(g, g["dims"])
        x = u16_to(g["x"], torch.float16)
        y = O.chain_forward(x, layers, [O.ACT_RELU, O.ACT_RELU, O.ACT_NONE])
        torch.testing.assert_close(y, torch.from_numpy(g["y"]), **TOL)


def test_dlrm_matches_reference_model():
    for name in ("dlrm_bot", "dlrm_top"):
        g = load_golden(name)
        layers = _layers(g, g["dims"], init="xavier")
        x = u16_to(g["x"], torch.float16)
        sig = int(g["sigmoid_i"])
        y = O.dlrm_mlp(x, layers, None if sig < 0 else sig)
        torch.testing.assert_close(y, torch.from_numpy(g["y"]), **TOL)
        acts = [O.ACT_SIGMOID if i == sig else O.ACT_RELU for i in range(len(layers))]
        torch.testing.assert_close(O.chain_forward(x, layers, acts), torch.from_numpy(g["y"]), **TOL)


def test_bert_ffn_matches_reference_model():
    g = load_golden("bert_ffn_128")
    layers = _layers(g, g["dims"], dtype=torch.bfloat16, init="normal002")
    x = u16_to(g["x"], torch.bfloat16)
    ln = (torch.ones(128), torch.zeros(128))
    y = O.bert_ffn(x, layers, ln, act_id=O.ACT_RELU, ln_eps=1e-5)
    torch.testing.assert_close(y, torch.from_numpy(g["y"]), **TOL)
    y2 = O.chain_forward(x, layers, [O.ACT_RELU, O.ACT_NONE], O.TAIL_RESIDUAL_LN, ln, 1e-5)
    torch.testing.assert_close(y2, torch.from_numpy(g["y"]), **TOL)


def test_gc_edges_matches_reference_model():
    g = load_golden("gc_edges_relu")
    layers = _layers(g, g["dims"], dtype=torch.bfloat16)
    x = u16_to(g["x"], torch.bfloat16)
    ln = (torch.ones(512), torch.zeros(512))
    y = O.gc_edges(x, layers, ln, act_id=O.ACT_RELU)
    torch.testing.assert_close(y, torch.from_numpy(g["y"]), **TOL)


def test_nerf_matches_reference_model():
    g = load_golden("nerf_63")
    gen = torch.Generator().manual_seed(int(g["seed"]))
    layers = []
    for k, n in zip(g["dims_in"], g["dims_out"]):
        s = int(torch.randint(0, 2**31 - 1, (1,), generator=gen))
        layers.append(layer_params(s, [int(k), int(n)])[0])
    assert abs(checksum(layers) - float(g["wsum"])) < 1e-6
    x = u16_to(g["x"], torch.float16)
    y = O.nerf(x, layers, skip=4)
    torch.testing.assert_close(y, torch.from_numpy(g["y"]), **TOL)


def _nerf_full_layers(g):
    gen = torch.Generator().manual_seed(int(g["seed"]))
    layers = []
    for k, n in zip(g["dims_in"], g["dims_out"]):
        s = int(torch.randint(0, 2**31 - 1, (1,), generator=gen))
        layers.append(layer_params(s, [int(k), int(n)])[0])
    return layers


def test_nerf_full_matches_reference_model():
    """Nerf(64, 32, radiance_dim=64, rgb_dim=64) with view directions, as
    apps/nerf_full/pipelined/val.py:10 builds it."""
    g = load_golden("nerf_full_viewdirs")
    layers = _nerf_full_layers(g)
    assert [tuple(w.shape) for w, _ in layers] == [
        (64, 256), (256, 256), (256, 256), (256, 256), (256, 256), (320, 256), (256, 256),
        (256, 256), (256, 64), (256, 256), (288, 128), (128, 64)]
    assert abs(checksum(layers) - float(g["wsum"])) < 1e-6
    alpha, rgb = O.nerf_full(u16_to(g["x"], torch.float16), u16_to(g["d"], torch.float16), layers)
    torch.testing.assert_close(alpha, torch.from_numpy(g["alpha"]), **TOL)
    torch.testing.assert_close(rgb, torch.from_numpy(g["rgb"]), **TOL)


def test_mgn_graph_step_matches_reference_model():
    """Edge update, segment sum and node update (graphmodel/mgn_dp.py:28-54) with the reference's
    MgnMlp."""
    g = load_golden("mgn_graph_step")
    seed = int(g["seed"])
    le = layer_params(seed + 1, [384, 128, 128, 128])
    ln_ = layer_params(seed + 2, [256, 128, 128, 128])
    assert abs(checksum(le) - float(g["edge_wsum"])) < 1e-6
    assert abs(checksum(ln_) - float(g["node_wsum"])) < 1e-6
    nf, ef = u16_to(g["nf"], torch.float16), u16_to(g["ef"], torch.float16)
    srcs, dsts = torch.from_numpy(g["srcs"]), torch.from_numpy(g["dsts"])
    lne = (u16_to(g["edge_gamma"], torch.float16), u16_to(g["edge_beta"], torch.float16))
    lnn = (u16_to(g["node_gamma"], torch.float16), u16_to(g["node_beta"], torch.float16))
    y_edge = O.mgn_edge_update(nf, ef, srcs, dsts, le, lne)
    torch.testing.assert_close(y_edge, torch.from_numpy(g["y_edge"]), **TOL)
    # one fp16 ulp where the two fp32 edge outputs round to different halves
    agg = O.mgn_aggregate(y_edge.half(), dsts, nf.shape[0])
    torch.testing.assert_close(agg, torch.from_numpy(g["agg"]), atol=2e-3, rtol=1e-3)
    y_node = O.mgn_node_update(nf, [torch.from_numpy(g["agg"])], ln_, lnn)
    torch.testing.assert_close(y_node, torch.from_numpy(g["y_node"]), **TOL)


def test_layernorm_known_row():
    """misc_tests/layer_norm/torch_val.py:87-116: one 128-value row, gamma=1, beta=0."""
    g = load_golden("ln_known_row")
    x = u16_to(g["x"], torch.float16).float()[None]
    y = O.layernorm(x, None, None, 1e-5)[0]
    torch.testing.assert_close(y, torch.from_numpy(g["y"]), **TOL)


def test_compare_thresholds():
    e = torch.randn(1000, 64)
    assert O.compare(e + 1e-4, e)["ok"]
    bad = e.clone()
    bad[3, 7] += 0.5
    assert not O.compare(bad, e)["ok"]
    nan = e.clone()
    nan[0, 0] = float("nan")
    assert not O.compare(nan, e)["ok"]


def test_bert_addln_ffn_matches_reference_model():
    g = load_golden("bert_addln_ffn_128")
    seed = int(g["seed"])
    layers = layer_params(seed, [128, 128]) + layer_params(seed + 1, [128, 512, 128])
    assert abs(checksum(layers) - float(g["wsum"])) < 1e-6, "weight generator drifted"
    attn = u16_to(g["attn"], torch.float16)
    x = u16_to(g["x"], torch.float16)
    ln0 = (u16_to(g["ln0_gamma"], torch.float16), u16_to(g["ln0_beta"], torch.float16))
    ln2 = (u16_to(g["ln2_gamma"], torch.float16), u16_to(g["ln2_beta"], torch.float16))
    y = O.bert_addln_ffn(attn, x, layers, ln0, ln2)
    torch.testing.assert_close(y, torch.from_numpy(g["y"]), **TOL)
