"""Generate the golden fixtures in this directory from the REFERENCE's own PyTorch models.

Run where the reference source tree is available ($GP_REFERENCE, default: a directory named
`reference` beside this repository):
    python tests/golden/make_golden.py
It imports the reference's model classes straight from its sources
(common/mlps.py MgnMlp/DlrmMlp, apps/bert_ffn/torch/model.py BertFfn,
apps/gc_edges/torch/model.py GraphCastEdges, apps/nerf_full/torch/model.py Nerf), loads seeded
weights into them, runs them in fp32 on the CPU and stores inputs and outputs as .npz. It also
stores the reference's known-answer LayerNorm row (misc_tests/layer_norm/torch_val.py:87-116),
parsed from that file as text.

Weights are not stored: `layer_params()` below regenerates them bit-exactly from the seed (the
tests import it), and each fixture keeps a float64 checksum of them to detect drift.
"""
from __future__ import annotations

import importlib.util
import math
import os
import re
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def layer_params(seed: int, dims: list[int], dtype=torch.float16, init="kaiming"):
    """Seeded [K, N] weights and [N] biases for Linear(dims[i] -> dims[i+1]), rounded to dtype."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for k, n in zip(dims[:-1], dims[1:]):
        if init == "kaiming":
            bound = 1.0 / math.sqrt(k)
            w = (torch.rand(n, k, generator=g) * 2 - 1) * bound
        elif init == "normal002":
            w = torch.randn(n, k, generator=g) * 0.02
        else:
            bound = math.sqrt(6.0 / (k + n))
            w = (torch.rand(n, k, generator=g) * 2 - 1) * bound
        b = (torch.rand(n, generator=g) * 2 - 1) / math.sqrt(k)
        out.append((w.t().contiguous().to(dtype), b.to(dtype)))
    return out


def checksum(layers) -> float:
    return float(sum(w.double().sum() + b.double().sum() for w, b in layers))


def _load(ref: Path, rel: str, name: str):
    spec = importlib.util.spec_from_file_location(name, ref / rel)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _set_linear(lin, w_kn, b):
    with torch.no_grad():
        lin.weight.copy_(w_kn.float().t())
        lin.bias.copy_(b.float())


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _save(name: str, **arrays):
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print("wrote", name, {k: v.shape for k, v in arrays.items()})


def main() -> None:
    ref = Path(os.environ.get("GP_REFERENCE", ROOT.parent / "reference"))
    mlps = _load(ref, "common/mlps.py", "ref_mlps")
    torch.manual_seed(0)
    rows = 48

    # ---- MgnMlp (common/mlps.py:3-20) in the four shapes the resident kernel serves
    for name, k0, ln, seed in (("mgn_fullmlp_k384", 384, True, 11), ("mgn_fullmlp_k256", 256, True, 12),
                               ("mgn_linears_k384", 384, False, 13), ("testmlp_k128", 128, False, 14)):
        layers = layer_params(seed, [k0, 128, 128, 128])
        net = mlps.MgnMlp(k0, [128, 128, 128], layernorm=ln).eval()
        for i, (w, b) in enumerate(layers):
            _set_linear(net.model[i][0], w, b)
        g = torch.Generator().manual_seed(seed + 100)
        x = torch.randn(rows, k0, generator=g).half()
        gamma = beta = None
        if ln:
            gamma = (1 + 0.1 * torch.randn(128, generator=g)).half()
            beta = (0.1 * torch.randn(128, generator=g)).half()
            with torch.no_grad():
                net.model[3].weight.copy_(gamma.float())
                net.model[3].bias.copy_(beta.float())
        with torch.no_grad():
            y = net(x.float())
        extra = {} if not ln else {"gamma": _u16(gamma), "beta": _u16(beta)}
        _save(name, seed=np.int64(seed), dims=np.array([k0, 128, 128, 128]), x=_u16(x),
              y=y.numpy().astype(np.float32), wsum=np.float64(checksum(layers)), **extra)

    # ---- DlrmMlp (common/mlps.py:23-35): bottom (ReLU everywhere) and top (sigmoid last)
    for name, dims, sig, seed in (("dlrm_bot", [16, 512, 256, 128], None, 21),
                                  ("dlrm_top", [480, 1024, 1024, 512, 256, 1], 4, 22)):
        layers = layer_params(seed, dims, init="xavier")
        net = mlps.DlrmMlp(dims, sigmoid_i=sig).eval()
        lins = [m for m in net.model if isinstance(m, torch.nn.Linear)]
        for lin, (w, b) in zip(lins, layers):
            _set_linear(lin, w, b)
        g = torch.Generator().manual_seed(seed + 100)
        x = torch.randn(rows, dims[0], generator=g).half()
        with torch.no_grad():
            y = net(x.float())
        _save(name, seed=np.int64(seed), dims=np.array(dims), x=_u16(x),
              y=y.numpy().astype(np.float32), wsum=np.float64(checksum(layers)),
              sigmoid_i=np.int64(-1 if sig is None else sig))

    # ---- BertFfn (apps/bert_ffn/torch/model.py:4-15), the reference's own 128/512 ReLU shape
    bert = _load(ref, "apps/bert_ffn/torch/model.py", "ref_bert")
    seed = 31
    layers = layer_params(seed, [128, 512, 128], dtype=torch.bfloat16, init="normal002")
    net = bert.BertFfn(128, 512).eval()
    _set_linear(net.ffn[0], *layers[0])
    _set_linear(net.ffn[2], *layers[1])
    g = torch.Generator().manual_seed(seed + 100)
    x = torch.randn(rows, 128, generator=g).bfloat16()
    with torch.no_grad():
        y = net(x.float())
    _save("bert_ffn_128", seed=np.int64(seed), dims=np.array([128, 512, 128]), x=_u16(x),
          y=y.numpy().astype(np.float32), wsum=np.float64(checksum(layers)))

    # ---- GraphCastEdges (apps/gc_edges/torch/model.py:4-14), ReLU as in the reference
    gc = _load(ref, "apps/gc_edges/torch/model.py", "ref_gc")
    seed = 41
    layers = layer_params(seed, [1536, 512, 512], dtype=torch.bfloat16)
    net = gc.GraphCastEdges().eval()
    _set_linear(net.mlp[0], *layers[0])
    _set_linear(net.mlp[2], *layers[1])
    g = torch.Generator().manual_seed(seed + 100)
    x = torch.randn(16, 1536, generator=g).bfloat16()
    with torch.no_grad():
        y = net(x.float())
    _save("gc_edges_relu", seed=np.int64(seed), dims=np.array([1536, 512, 512]), x=_u16(x),
          y=y.numpy().astype(np.float32), wsum=np.float64(checksum(layers)))

    # ---- Nerf (apps/nerf_full/torch/model.py:5-66) without view directions, out_ch=4
    nf = _load(ref, "apps/nerf_full/torch/model.py", "ref_nerf")
    seed = 51
    net = nf.Nerf(in_x_ch=63, use_viewdirs=False, out_ch=4).eval()
    lins = [m for m in list(net.preskip) + list(net.postskip) if isinstance(m, torch.nn.Linear)]
    lins.append(net.decode)
    dims_in = [lin.in_features for lin in lins]
    dims_out = [lin.out_features for lin in lins]
    g = torch.Generator().manual_seed(seed)
    layers = []
    for lin, k, n in zip(lins, dims_in, dims_out):
        p = layer_params(int(torch.randint(0, 2**31 - 1, (1,), generator=g)), [k, n])[0]
        layers.append(p)
        _set_linear(lin, *p)
    gx = torch.Generator().manual_seed(seed + 100)
    x = (torch.rand(rows, 63, generator=gx) * 2 - 1).half()
    with torch.no_grad():
        y = net(x.float())
    _save("nerf_63", seed=np.int64(seed), dims_in=np.array(dims_in), dims_out=np.array(dims_out),
          x=_u16(x), y=y.numpy().astype(np.float32), wsum=np.float64(checksum(layers)))

    gen_bert_addln(ref, rows)
    gen_nerf_full(ref, rows)
    gen_mgn_graph(ref)
    gen_val_replay(ref)

    # ---- known-answer LayerNorm row from misc_tests/layer_norm/torch_val.py:87-116
    src = (ref / "misc_tests/layer_norm/torch_val.py").read_text()
    body = src[src.index("def manual_test"):]
    lit = body[body.index("torch.tensor([") + len("torch.tensor(["):body.index("]", body.index("torch.tensor(["))]
    vals = [float(v) for v in re.findall(r"-?\d+\.\d+", lit)]
    assert len(vals) == 128, len(vals)
    row = torch.tensor(vals, dtype=torch.float16)
    y = torch.nn.functional.layer_norm(row.float()[None], [128])[0]
    _save("ln_known_row", x=_u16(row), y=y.numpy().astype(np.float32))


def gen_bert_addln(ref: Path, rows: int = 48) -> None:
    """BertFfn of apps/bert_addln_ffn/torch/model.py:4-19 (attention-output Linear + x + LN0, then
    the 128 -> 512 ReLU -> 128 FFN + residual + LN2), fp16 inputs, perturbed LayerNorm params."""
    mod = _load(ref, "apps/bert_addln_ffn/torch/model.py", "ref_bert_addln")
    seed = 61
    layers = layer_params(seed, [128, 128]) + layer_params(seed + 1, [128, 512, 128])
    net = mod.BertFfn(128, 512).eval()
    _set_linear(net.y0w0, *layers[0])
    _set_linear(net.ffn[0], *layers[1])
    _set_linear(net.ffn[2], *layers[2])
    g = torch.Generator().manual_seed(seed + 100)
    attn = torch.randn(rows, 128, generator=g).half()
    x = torch.randn(rows, 128, generator=g).half()
    lnp = {}
    for name, lnm in (("ln0", net.ln0), ("ln2", net.ln2)):
        ga = (1 + 0.1 * torch.randn(128, generator=g)).half()
        be = (0.1 * torch.randn(128, generator=g)).half()
        with torch.no_grad():
            lnm.weight.copy_(ga.float())
            lnm.bias.copy_(be.float())
        lnp[name + "_gamma"], lnp[name + "_beta"] = _u16(ga), _u16(be)
    with torch.no_grad():
        y = net(attn.float(), x.float())
    _save("bert_addln_ffn_128", seed=np.int64(seed), attn=_u16(attn), x=_u16(x),
          y=y.numpy().astype(np.float32), wsum=np.float64(checksum(layers)), **lnp)


def gen_nerf_full(ref: Path, rows: int = 48) -> None:
    """Nerf of apps/nerf_full/torch/model.py:5-66 with view directions, built the way the
    reference's own check builds it (apps/nerf_full/pipelined/val.py:10: Nerf(64, 32,
    radiance_dim=64, rgb_dim=64)); x and d from randn, as there."""
    nf = _load(ref, "apps/nerf_full/torch/model.py", "ref_nerf_full")
    seed = 71
    net = nf.Nerf(64, 32, radiance_dim=64, rgb_dim=64).eval()
    lins = [m for m in list(net.preskip) + list(net.postskip) if isinstance(m, torch.nn.Linear)]
    lins += [net.alpha, net.bottleneck, net.rgb[0], net.rgb[2]]
    dims_in = [lin.in_features for lin in lins]
    dims_out = [lin.out_features for lin in lins]
    g = torch.Generator().manual_seed(seed)
    layers = []
    for lin, k, n in zip(lins, dims_in, dims_out):
        p = layer_params(int(torch.randint(0, 2**31 - 1, (1,), generator=g)), [k, n])[0]
        layers.append(p)
        _set_linear(lin, *p)
    gx = torch.Generator().manual_seed(seed + 100)
    x = torch.randn(rows, 64, generator=gx).half()
    d = torch.randn(rows, 32, generator=gx).half()
    with torch.no_grad():
        rgb, alpha = net(x.float(), d.float())
    _save("nerf_full_viewdirs", seed=np.int64(seed), dims_in=np.array(dims_in),
          dims_out=np.array(dims_out), x=_u16(x), d=_u16(d), rgb=rgb.numpy().astype(np.float32),
          alpha=alpha.numpy().astype(np.float32), wsum=np.float64(checksum(layers)))


def gen_mgn_graph(ref: Path, n_nodes: int = 40, n_edges: int = 96) -> None:
    """One MeshGraphNet message-passing step on a random graph (graphmodel/mgn_dp.py:28-54), with
    the reference's MgnMlp (common/mlps.py:3-20) for the edge (384 -> 128 x 3 + LN) and node
    (256 -> 128 x 3 + LN) MLPs. The aggregate is the segment sum by destination of the edge
    outputs rounded to fp16, and enters the node MLP rounded to fp16."""
    mlps = _load(ref, "common/mlps.py", "ref_mlps_graph")
    seed = 81
    g = torch.Generator().manual_seed(seed)
    nf = torch.randn(n_nodes, 128, generator=g).half()
    ef = torch.randn(n_edges, 128, generator=g).half()
    srcs = torch.randint(0, n_nodes, (n_edges,), generator=g)
    dsts = torch.randint(0, n_nodes, (n_edges,), generator=g)
    out = {}
    nets = {}
    for name, k0, s in (("edge", 384, seed + 1), ("node", 256, seed + 2)):
        layers = layer_params(s, [k0, 128, 128, 128])
        net = mlps.MgnMlp(k0, [128, 128, 128], layernorm=True).eval()
        for i, (w, b) in enumerate(layers):
            _set_linear(net.model[i][0], w, b)
        gamma = (1 + 0.1 * torch.randn(128, generator=g)).half()
        beta = (0.1 * torch.randn(128, generator=g)).half()
        with torch.no_grad():
            net.model[3].weight.copy_(gamma.float())
            net.model[3].bias.copy_(beta.float())
        nets[name] = net
        out[f"{name}_gamma"], out[f"{name}_beta"] = _u16(gamma), _u16(beta)
        out[f"{name}_wsum"] = np.float64(checksum(layers))
    with torch.no_grad():
        y_edge = nets["edge"](torch.cat([nf[srcs], ef, nf[dsts]], dim=-1).float())
        agg = torch.zeros(n_nodes, 128).index_add_(0, dsts, y_edge.half().float())
        y_node = nets["node"](torch.cat([nf, agg.half()], dim=-1).float())
    _save("mgn_graph_step", seed=np.int64(seed), nf=_u16(nf), ef=_u16(ef), srcs=srcs.numpy(),
          dsts=dsts.numpy(), y_edge=y_edge.numpy().astype(np.float32), agg=agg.numpy(),
          y_node=y_node.numpy().astype(np.float32), **out)


def gen_val_replay(ref: Path, rows: int = 16) -> None:
    """The eleven apps' models built exactly as their apps/<app>/pipelined/val.py builds them
    (torch.manual_seed(0), the reference's model class, .eval().half()). Stores, per app, the
    parameter checksum (which pins tests/_val_apps.build() to the reference's construction order)
    and the reference model's fp32 output on `rows` input rows."""
    from tests import _val_apps as V

    mlps = _load(ref, "common/mlps.py", "ref_mlps_val")
    mods = {a: _load(ref, f"apps/{a}/torch/model.py", f"ref_val_{a}")
            for a in ("bert_ffn", "bert_addln_ffn", "gc_edges", "gc_nodes", "nerf_a", "nerf_full")}
    ctor = {
        "mgn_fullmlp": lambda: mlps.MgnMlp(384, [128, 128, 128], layernorm=True),
        "mgn_linears": lambda: mlps.MgnMlp(384, [128, 128, 128], layernorm=False),
        "test_mlp": lambda: mlps.MgnMlp(128, [128, 128, 128], layernorm=False),
        "dlrm_botmlp": lambda: mlps.DlrmMlp([13 + 19, 512, 256, 128]),
        "dlrm_topmlp": lambda: mlps.DlrmMlp([479 + 33, 1024, 1024, 512, 256, 64]),
        "bert_ffn": lambda: mods["bert_ffn"].BertFfn(),
        "bert_addln_ffn": lambda: mods["bert_addln_ffn"].BertFfn(),
        "gc_edges": lambda: mods["gc_edges"].GraphCastEdges(),
        "gc_nodes": lambda: mods["gc_nodes"].GraphCastNodes(),
        "nerf_a": lambda: mods["nerf_a"].NerfA(64),
        "nerf_full": lambda: mods["nerf_full"].Nerf(64, 32, radiance_dim=64, rgb_dim=64),
    }
    out = {}
    for app, make in ctor.items():
        torch.manual_seed(0)
        net = make().eval().half()
        lins = [m for m in net.modules() if isinstance(m, torch.nn.Linear)]
        ref_sum = float(sum(m.weight.detach().double().sum() + m.bias.detach().double().sum() for m in lins))
        ws, bs, _ = V.build(app)
        assert abs(ref_sum - V.checksum(ws, bs)) < 1e-9, (app, ref_sum, V.checksum(ws, bs))
        xs = V.inputs(app, rows)
        with torch.no_grad():
            y = net.float()(*[x.float() for x in xs])
        out[f"{app}_wsum"] = np.float64(ref_sum)
        for i, x in enumerate(xs):
            out[f"{app}_x{i}"] = _u16(x)
        if isinstance(y, tuple):   # Nerf with view directions returns (rgb, alpha)
            out[f"{app}_rgb"] = y[0].numpy().astype(np.float32)
            out[f"{app}_alpha"] = y[1].numpy().astype(np.float32)
        else:
            out[f"{app}_y"] = y.numpy().astype(np.float32)
    _save("val_replay", **out)


if __name__ == "__main__":
    sys.path.insert(0, str(ROOT))
    main()
