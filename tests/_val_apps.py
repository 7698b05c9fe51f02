"""The reference's eleven app checks (apps/<app>/pipelined/val.py), restated so they can run
where the reference tree is absent.

Each val.py does `torch.manual_seed(0)`, builds the app's PyTorch model with default
(Kaiming-uniform) nn.Linear init, casts it to fp16, and calls `ext.cuda_ext.<app>(...)` with
`linear.weight.t().contiguous()` and `linear.bias` (and LayerNorm weight / bias) in a fixed
argument order. `build(app)` reproduces the model's parameters bit for bit by constructing the
same nn.Linear modules in the same order under the same seed (LayerNorm and activation modules
draw no random numbers); tests/golden/make_golden.py pins that against the reference's own model
classes (a checksum of every parameter, and the reference model's fp32 output on the first rows).

The inputs differ from val.py's only in where they are drawn: val.py draws them on the GPU
(`torch.randn(..., device='cuda')`); here a CPU generator seeded from the app name draws them.
"""
from __future__ import annotations

import torch

# app -> (rows M as in val.py, nn.Linear (in, out) in construction order, input widths,
#         LayerNorm widths in argument order)
APPS = {
    "mgn_fullmlp": (1280 * 1024, [(384, 128), (128, 128), (128, 128)], [384], [128]),
    "mgn_linears": (1280 * 1024, [(384, 128), (128, 128), (128, 128)], [384], []),
    "test_mlp": (1280 * 1024, [(128, 128), (128, 128), (128, 128)], [128], []),
    "dlrm_botmlp": (2048, [(32, 512), (512, 256), (256, 128)], [32], []),
    "dlrm_topmlp": (2048, [(512, 1024), (1024, 1024), (1024, 512), (512, 256), (256, 64)], [512], []),
    "bert_ffn": (64 * 512, [(128, 512), (512, 128)], [128], [128]),
    # BertFfn of bert_addln_ffn builds y0w0, ln0, ffn[0], ffn[2], ln2 in that order
    "bert_addln_ffn": (64 * 512, [(128, 128), (128, 512), (512, 128)], [128, 128], [128, 128]),
    "gc_edges": (64 * 512, [(1536, 512), (512, 512)], [1536], [512]),
    "gc_nodes": (64 * 512, [(1024, 512), (512, 512)], [1024], [512]),
    # NerfA(64): preskip 64 -> 256, 4 x 256 -> 256; postskip 320 -> 256, 2 x 256 -> 256
    "nerf_a": (65536, [(64, 256)] + [(256, 256)] * 4 + [(320, 256), (256, 256), (256, 256)], [64], []),
    # Nerf(64, 32, radiance_dim=64, rgb_dim=64): trunk as NerfA, then alpha 256 -> 64,
    # bottleneck 256 -> 256, rgb 288 -> 128 -> 64
    "nerf_full": (2048, [(64, 256)] + [(256, 256)] * 4 + [(320, 256), (256, 256), (256, 256),
                                                         (256, 64), (256, 256), (288, 128), (128, 64)],
                  [64, 32], []),
}


def build(app: str):
    """(weights [K, N] fp16, biases [N] fp16, LayerNorm (weight, bias) pairs) exactly as val.py's
    model holds them after `.eval().half()`."""
    _, lins, _, lns = APPS[app]
    torch.manual_seed(0)
    mods = [torch.nn.Linear(k, n) for k, n in lins]
    ws = [m.weight.detach().half().t().contiguous() for m in mods]
    bs = [m.bias.detach().half().contiguous() for m in mods]
    ln = [(torch.ones(n, dtype=torch.float16), torch.zeros(n, dtype=torch.float16)) for n in lns]
    return ws, bs, ln


def checksum(ws, bs) -> float:
    return float(sum(w.double().sum() + b.double().sum() for w, b in zip(ws, bs)))


def inputs(app: str, rows: int | None = None):
    m, _, widths, _ = APPS[app]
    g = torch.Generator().manual_seed(sum(map(ord, app)))
    return [torch.randn(rows or m, k, generator=g).half() for k in widths]


def call(cuda_ext, app: str, xs, ws, bs, ln):
    """The ext.cuda_ext call of the app's val.py, argument for argument."""
    wb = [t for p in zip(ws, bs) for t in p]
    lnf = [t for p in ln for t in p]
    if app == "bert_addln_ffn":
        return cuda_ext.bert_addln_ffn(xs[0], xs[1], *wb, *lnf)
    if app == "nerf_full":
        return cuda_ext.nerf_full(xs[0], xs[1], *wb)
    fn = {"test_mlp": cuda_ext.testmlp}.get(app) or getattr(cuda_ext, app)
    return fn(xs[0], *wb, *lnf)


def oracle(O, app: str, xs, ws, bs, ln):
    """fp32 result of the app's model (oracle restatement); a tuple for nerf_full."""
    layers = list(zip(ws, bs))
    x = xs[0]
    if app == "mgn_fullmlp":
        return O.mgn_mlp(x, layers, ln[0], 1e-5)
    if app in ("mgn_linears", "test_mlp"):
        return O.mgn_mlp(x, layers)
    if app in ("dlrm_botmlp", "dlrm_topmlp"):
        return O.dlrm_mlp(x, layers)
    if app == "bert_ffn":
        return O.bert_ffn(x, layers, ln[0], O.ACT_RELU, 1e-5)
    if app == "bert_addln_ffn":
        return O.bert_addln_ffn(xs[0], xs[1], layers, ln[0], ln[1])
    if app in ("gc_edges", "gc_nodes"):
        return O.gc_edges(x, layers, ln[0], O.ACT_RELU, 1e-5)
    if app == "nerf_a":
        return O.chain_forward(x, layers, [O.ACT_RELU] * 8, skip_layer=5)
    if app == "nerf_full":
        return O.nerf_full(xs[0], xs[1], layers)
    raise KeyError(app)
