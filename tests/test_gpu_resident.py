"""GPU parity of the weight-resident fused chain (MeshGraphNet family) against the CPU oracle.

Every call goes through the C ABI (libgpipes.so). Tolerances are the north-star ones:
max |err| <= 2e-2 and relative L2 <= 5e-3 against the fp32 oracle; known-answer cases are exact.
"""
import pytest
import torch

from gpu_pipes_b200 import _lib as L
from gpu_pipes_b200 import cuda_ext
from gpu_pipes_b200 import workloads as W
from oracle import mlp_oracle as O
from tests._util import load_golden, u16_to
from tests.golden.make_golden import layer_params

pytestmark = pytest.mark.gpu

NONE, RELU = L.ACT_NONE, L.ACT_RELU


@pytest.fixture(params=[0, 1], ids=["default", "other"])
def variant(request):
    """Run a test with the default kernels and with the other form (single-CTA / CTA-pair)."""
    L.set_kernel_variant(request.param)
    yield request.param
    L.set_kernel_variant(0)


def _dev(ts, dev):
    return [t.to(dev) if t is not None else None for t in ts]


def _assert_close(out, ref, what):
    r = O.compare(out.float().cpu(), ref)
    assert r["ok"], f"{what}: {r}"
    return r


# ------------------------------------------------------------------ known answers (exact)
def test_single_gemm_all_ones(cuda_dev, variant):
    """misc_tests/gemm-val/blockgemm-val.cu:198-219 pattern: I = W = 1 -> every output = K."""
    x = torch.ones(256, 128, dtype=torch.float16, device=cuda_dev)
    w = torch.ones(128, 128, dtype=torch.float16, device=cuda_dev)
    out = torch.zeros(256, 128, dtype=torch.float16, device=cuda_dev)
    cuda_ext.fused_mlp_out(x, [w], [None], out, acts=[NONE])
    torch.cuda.synchronize()
    assert torch.equal(out, torch.full_like(out, 128.0))


def test_single_gemm_permutation(cuda_dev, variant):
    """x @ P for a permutation P is an exact column shuffle: checks the B-operand layout."""
    g = torch.Generator().manual_seed(5)
    x = torch.randn(384, 128, generator=g).half()
    perm = torch.randperm(128, generator=g)
    P = torch.zeros(128, 128)
    P[torch.arange(128), perm] = 1.0  # row i -> column perm[i]
    out = torch.zeros(384, 128, dtype=torch.float16, device=cuda_dev)
    cuda_ext.fused_mlp_out(x.to(cuda_dev), [P.half().to(cuda_dev)], [None], out, acts=[NONE])
    torch.cuda.synchronize()
    expect = torch.zeros(384, 128, dtype=torch.float16)
    expect[:, perm] = x
    assert torch.equal(out.cpu(), expect)


def test_two_layer_tmem_handoff_exact(cuda_dev, variant):
    """Layer 2 reads layer 1's output from TMEM (A operand in tensor memory). With W1 a
    permutation and W2 = 2*I the result is exact, so any packing error shows up."""
    g = torch.Generator().manual_seed(6)
    x = (torch.randn(1000, 128, generator=g) * 4).half()
    perm = torch.randperm(128, generator=g)
    P = torch.zeros(128, 128)
    P[torch.arange(128), perm] = 1.0
    W2 = 2 * torch.eye(128)
    out = torch.zeros(1000, 128, dtype=torch.float16, device=cuda_dev)
    cuda_ext.fused_mlp_out(x.to(cuda_dev), [P.half().to(cuda_dev), W2.half().to(cuda_dev)],
                           [None, None], out, acts=[NONE, NONE])
    torch.cuda.synchronize()
    expect = torch.zeros(1000, 128, dtype=torch.float16)
    expect[:, perm] = x * 2
    assert torch.equal(out.cpu(), expect)


def test_layernorm_known_row(cuda_dev):
    """The reference's known LayerNorm row (misc_tests/layer_norm/torch_val.py:87-116) repeated
    over 128 rows, carried through identity layers (x+1, relu, relu, -1) into the LN epilogue."""
    g = load_golden("ln_known_row")
    row = u16_to(g["x"], torch.float16)
    x = row.repeat(128, 1).to(cuda_dev)
    eye = torch.eye(128, dtype=torch.float16, device=cuda_dev)
    one = torch.ones(128, dtype=torch.float16, device=cuda_dev)
    zero = torch.zeros_like(one)
    out = cuda_ext.mgn_fullmlp(x, eye, one, eye, zero, eye, -one, one, zero)
    torch.cuda.synchronize()
    ref = torch.from_numpy(g["y"]).repeat(128, 1)
    _assert_close(out, ref, "ln known row")


# ------------------------------------------------------------------ golden fixtures (reference models)
@pytest.mark.parametrize("name", ["mgn_fullmlp_k384", "mgn_fullmlp_k256"])
def test_golden_mgn_fullmlp(cuda_dev, name):
    g = load_golden(name)
    layers = layer_params(int(g["seed"]), list(g["dims"]))
    x = u16_to(g["x"], torch.float16)
    gamma, beta = u16_to(g["gamma"], torch.float16), u16_to(g["beta"], torch.float16)
    d = _dev([x] + [t for p in layers for t in p] + [gamma, beta], cuda_dev)
    out = cuda_ext.mgn_fullmlp(*d)
    torch.cuda.synchronize()
    _assert_close(out, torch.from_numpy(g["y"]), name)


def test_golden_mgn_linears(cuda_dev):
    g = load_golden("mgn_linears_k384")
    layers = layer_params(int(g["seed"]), list(g["dims"]))
    x = u16_to(g["x"], torch.float16)
    out = cuda_ext.mgn_linears(*_dev([x] + [t for p in layers for t in p], cuda_dev))
    torch.cuda.synchronize()
    _assert_close(out, torch.from_numpy(g["y"]), "mgn_linears")


def test_golden_testmlp(cuda_dev):
    g = load_golden("testmlp_k128")
    layers = layer_params(int(g["seed"]), list(g["dims"]))
    x = u16_to(g["x"], torch.float16)
    out = cuda_ext.testmlp(*_dev([x] + [t for p in layers for t in p], cuda_dev))
    torch.cuda.synchronize()
    _assert_close(out, torch.from_numpy(g["y"]), "testmlp")


# ------------------------------------------------------------------ benchmark configs, full size
def _run_workload(w, dev, x=None):
    x = W.make_input(w) if x is None else x
    layers, ln = W.make_weights(w)
    out = torch.empty(w.m, w.n_out, dtype=w.dtype, device=dev)
    cuda_ext.run_workload_out(w, x.to(dev), [(a.to(dev), b.to(dev)) for a, b in layers],
                              None if ln is None else tuple(t.to(dev) for t in ln), out)
    torch.cuda.synchronize()
    return x, layers, ln, out


@pytest.mark.parametrize("wname", ["mgn_edge", "mgn_node"])
def test_config_full_size(cuda_dev, wname, variant):
    w = W.WORKLOADS[wname]
    x, layers, ln, out = _run_workload(w, cuda_dev)
    ref = O.workload_forward(w, x, layers, ln)
    r = _assert_close(out, ref, wname)
    print(wname, r)


@pytest.mark.parametrize("m", [1, 2, 127, 128, 129, 255, 300, 1000, 65537])
def test_ragged_rows(cuda_dev, m, variant):
    w = W.MGN_EDGE.with_m(m)
    x, layers, ln, out = _run_workload(w, cuda_dev)
    _assert_close(out, O.workload_forward(w, x, layers, ln), f"m={m}")


def test_no_write_past_last_row(cuda_dev):
    w = W.MGN_EDGE.with_m(300)
    x = W.make_input(w)
    layers, ln = W.make_weights(w)
    buf = torch.full((300 + 128, 128), 7.0, dtype=torch.float16, device=cuda_dev)
    out = buf[:300]
    cuda_ext.run_workload_out(w, x.to(cuda_dev), [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers],
                              tuple(t.to(cuda_dev) for t in ln), out)
    torch.cuda.synchronize()
    assert torch.all(buf[300:] == 7.0)
    _assert_close(out, O.workload_forward(w, x, layers, ln), "guarded")


@pytest.mark.parametrize("k0", [128, 256, 384])
def test_bf16_mgn(cuda_dev, k0):
    w = W.Workload(**{**W.MGN_EDGE.with_m(4096).__dict__, "dtype": torch.bfloat16,
                      "layers": W._mgn("t", 1, k0, 0).layers, "input_logical": k0})
    x, layers, ln, out = _run_workload(w, cuda_dev)
    _assert_close(out, O.workload_forward(w, x, layers, ln), f"bf16 k0={k0}")


@pytest.mark.parametrize("k0", [128, 256, 384])
def test_no_layernorm_variants(cuda_dev, k0):
    w = W.Workload(**{**W.MGN_LINEARS.with_m(5000).__dict__, "layers": W._mgn("t", 1, k0, 0).layers,
                      "input_logical": k0})
    x, layers, ln, out = _run_workload(w, cuda_dev)
    _assert_close(out, O.workload_forward(w, x, layers, ln), f"no-LN k0={k0}")


def test_deterministic_and_counts_launches(cuda_dev):
    w = W.MGN_NODE.with_m(70000)
    x = W.make_input(w).to(cuda_dev)
    layers, ln = W.make_weights(w)
    wd = [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers]
    lnd = tuple(t.to(cuda_dev) for t in ln)
    outs = []
    before = L.launch_count()
    for _ in range(3):
        o = torch.empty(w.m, 128, dtype=torch.float16, device=cuda_dev)
        cuda_ext.run_workload_out(w, x, wd, lnd, o)
        outs.append(o)
    torch.cuda.synchronize()
    assert L.launch_count() == before + 3
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])


def test_honours_caller_stream(cuda_dev):
    w = W.MGN_EDGE.with_m(20000)
    x = W.make_input(w)
    layers, ln = W.make_weights(w)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        xd = x.to(cuda_dev, non_blocking=False)
        wd = [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers]
        lnd = tuple(t.to(cuda_dev) for t in ln)
        out = torch.empty(w.m, 128, dtype=torch.float16, device=cuda_dev)
        cuda_ext.run_workload_out(w, xd, wd, lnd, out)
    s.synchronize()
    _assert_close(out, O.workload_forward(w, x, layers, ln), "side stream")


# ------------------------------------------------------------------ errors
def test_misaligned_device_pointer_rejected(cuda_dev):
    w = W.MGN_EDGE.with_m(64)
    layers, ln = W.make_weights(w)
    big = torch.zeros(64 * 384 + 1, dtype=torch.float16, device=cuda_dev)
    x = big[1:].view(64, 384)  # 2-byte offset
    out = torch.empty(64, 128, dtype=torch.float16, device=cuda_dev)
    with pytest.raises(L.GpError) as e:
        cuda_ext.run_workload_out(w, x, [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers],
                                  tuple(t.to(cuda_dev) for t in ln), out)
    assert e.value.code == L.GP_ERR_ALIGN


def test_wrong_width_raises(cuda_dev):
    x = torch.zeros(64, 384, dtype=torch.float16, device=cuda_dev)
    w1 = torch.zeros(384, 64, dtype=torch.float16, device=cuda_dev)
    w = torch.zeros(128, 128, dtype=torch.float16, device=cuda_dev)
    b = torch.zeros(128, dtype=torch.float16, device=cuda_dev)
    with pytest.raises(RuntimeError):
        cuda_ext.mgn_fullmlp(x, w1, b, w, b, w, b, b, b)


def test_timeout_is_reported_and_context_survives(cuda_dev, variant):
    """Fault injection on the host side: the producer never issues its loads, so every consumer
    wait runs out after 5 ms; the kernel exits cleanly, the status word says which role gave up,
    and the next launch on the same context is correct."""
    w = W.MGN_EDGE.with_m(4096)
    x = W.make_input(w)
    layers, ln = W.make_weights(w)
    xd = x.to(cuda_dev)
    wd = [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers]
    lnd = tuple(t.to(cuda_dev) for t in ln)
    out = torch.empty(w.m, 128, dtype=torch.float16, device=cuda_dev)
    assert L.device_status(0, clear=True) == 0
    try:
        L.set_timeout_ns(5_000_000)
        L.set_fault_injection(1)
        cuda_ext.run_workload_out(w, xd, wd, lnd, out)
        torch.cuda.synchronize()
    finally:
        L.set_fault_injection(0)
        L.set_timeout_ns(0)
    st = L.device_status(0, clear=True)
    assert st in (0x100, 0x200, 0x300), hex(st)
    assert L.device_status(0) == 0
    cuda_ext.run_workload_out(w, xd, wd, lnd, out)
    torch.cuda.synchronize()
    _assert_close(out, O.workload_forward(w, x, layers, ln), "after timeout")
