"""Reference-compatible entry points: `cuda_ext.<app>(...)` and `cuda_ext.<app>_out(...)`.

The reference exposes each app as a pybind11 extension, e.g.
apps/mgn_fullmlp/pipelined/mgn_fullmlp_pl_ext.cu:24-93:
    mgn_fullmlp_out(x, w1, b1, w2, b2, w3, b3, gamma, beta, out) -> None
    mgn_fullmlp(x, w1, b1, w2, b2, w3, b3, gamma, beta) -> out
with weights in [K, N] layout (`linear.weight.t().contiguous()`, apps/mgn_fullmlp/pipelined/val.py:17-19).
The same names and argument meanings are kept here, so the reference's val.py / perf.py call
pattern (`ext.cuda_ext.mgn_fullmlp(...)`) works unchanged. Differences, all deliberate:
  * checks raise RuntimeError (the reference's TORCH_CHECK does too; its width `assert`s abort
    the process instead),
  * the launch goes to torch's current stream (the reference uses the legacy default stream),
  * M need not be a multiple of the reference's `n_rows * mblk`.
Each call goes through the C ABI (libgpipes.so) with raw device pointers.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib as L
from . import workloads as W

_DT = {torch.float16: L.GP_F16, torch.bfloat16: L.GP_BF16}


def _check_input(name: str, t: torch.Tensor | None, dtype: torch.dtype | None = None) -> None:
    if t is None:
        return
    if (type(t) is torch.Tensor and t.is_cuda and t.is_contiguous()
            and (dtype is None or t.dtype == dtype)):
        return  # the common case, in one test
    if not isinstance(t, torch.Tensor):
        raise RuntimeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")
    if dtype is not None and t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    """torch's current stream on t's device (the raw handle straight from torch's C layer where
    available: the Stream object costs a couple of microseconds per call)."""
    if _raw_stream is not None and t.device.index is not None:
        return ctypes.c_void_p(_raw_stream(t.device.index))
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


class _on_device:
    """`with torch.cuda.device(dev)`, skipped when `dev` is already current (the common case;
    switching costs microseconds of host time per call)."""

    __slots__ = ("idx", "prev")

    def __init__(self, dev: torch.device):
        self.idx = dev.index if dev.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False


_SPECS: dict = {}


def _spec(widths, acts, tail, dt, ln_eps, skip_layer):
    """The chain description, built once per distinct chain (the struct is read-only to C)."""
    key = (tuple(widths), tuple(acts), tail, dt, ln_eps, skip_layer)
    s = _SPECS.get(key)
    if s is None:
        s = _SPECS[key] = L.make_spec(widths, acts, tail, dt, ln_eps, skip_layer)
    return s


def fused_mlp_out(x, weights, biases, out, *, acts, tail=L.TAIL_NONE, gamma=None, beta=None,
                  ln_eps=1e-5, skip_layer=0) -> None:
    """Generic chain: out = tail(act_L(... act_1(x W_1 + b_1) ...)). Weights are [K, N].

    skip_layer = s > 0: layer s reads [output of layer s-1 || x] and its weight is
    [N_{s-1} + K0, N_s] (the NeRF skip connection)."""
    _check_input("x", x)
    dt = _DT.get(x.dtype)
    if dt is None:
        raise RuntimeError(f"x must be float16 or bfloat16, got {x.dtype}")
    for i, (w, b) in enumerate(zip(weights, biases)):
        _check_input(f"w{i + 1}", w, x.dtype)
        _check_input(f"b{i + 1}", b, x.dtype)
    _check_input("gamma", gamma, x.dtype)
    _check_input("beta", beta, x.dtype)
    _check_input("out", out, x.dtype)
    if x.dim() != 2 or out.dim() != 2:
        raise RuntimeError("x and out must be 2-D")
    widths = [x.shape[1]] + [w.shape[1] for w in weights]
    for i, w in enumerate(weights):
        k = widths[i] + (widths[0] if skip_layer and i == skip_layer else 0)
        if w.dim() != 2 or w.shape[0] != k:
            raise RuntimeError(f"w{i + 1} has shape {tuple(w.shape)}, expected [{k}, N]")
    if out.shape[0] != x.shape[0] or out.shape[1] != widths[-1]:
        raise RuntimeError(f"out has shape {tuple(out.shape)}, expected [{x.shape[0]}, {widths[-1]}]")
    spec = _spec(widths, acts, tail, dt, ln_eps, skip_layer)
    n = len(weights)
    wp = (ctypes.c_void_p * n)(*[w.data_ptr() for w in weights])
    bp = (ctypes.c_void_p * n)(*[(b.data_ptr() if b is not None else None) for b in biases])
    with _on_device(x.device):
        L.check(L.lib().gp_fused_mlp_out(ctypes.byref(spec), x.shape[0], _ptr(x), wp, bp,
                                         _ptr(gamma), _ptr(beta), _ptr(out), _stream(x)))


def fused_mlp_host_out(x_host, weights, biases, out_host, *, acts, tail=L.TAIL_NONE, gamma=None,
                       beta=None, ln_eps=1e-5, skip_layer=0, chunk_rows=0, device=None) -> None:
    """fused_mlp_out with x and out in HOST memory (pinned for overlap): the rows are streamed in
    chunks, H2D copies, kernels and D2H copies of neighbouring chunks overlapping. Weights and
    LayerNorm parameters are device tensors. Enqueued on the current stream of their device;
    synchronise it before reading out_host."""
    if x_host.is_cuda or out_host.is_cuda:
        raise RuntimeError("x_host and out_host must be host tensors")
    if not x_host.is_contiguous() or not out_host.is_contiguous():
        raise RuntimeError("x_host and out_host must be contiguous")
    dt = _DT.get(x_host.dtype)
    if dt is None or out_host.dtype != x_host.dtype:
        raise RuntimeError(f"x_host and out_host must both be float16 or bfloat16")
    dev = device if device is not None else weights[0].device
    for i, (w, b) in enumerate(zip(weights, biases)):
        _check_input(f"w{i + 1}", w, x_host.dtype)
        _check_input(f"b{i + 1}", b, x_host.dtype)
    _check_input("gamma", gamma, x_host.dtype)
    _check_input("beta", beta, x_host.dtype)
    widths = [x_host.shape[1]] + [w.shape[1] for w in weights]
    if out_host.dim() != 2 or out_host.shape[0] != x_host.shape[0] or out_host.shape[1] != widths[-1]:
        raise RuntimeError(f"out_host has shape {tuple(out_host.shape)}, expected [{x_host.shape[0]}, {widths[-1]}]")
    spec = L.make_spec(widths, acts, tail, dt, ln_eps, skip_layer)
    n = len(weights)
    wp = (ctypes.c_void_p * n)(*[w.data_ptr() for w in weights])
    bp = (ctypes.c_void_p * n)(*[(b.data_ptr() if b is not None else None) for b in biases])
    with torch.cuda.device(dev):
        L.check(L.lib().gp_fused_mlp_host(ctypes.byref(spec), x_host.shape[0],
                                          ctypes.c_void_p(x_host.data_ptr()), wp, bp, _ptr(gamma),
                                          _ptr(beta), ctypes.c_void_p(out_host.data_ptr()),
                                          int(chunk_rows),
                                          ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)))


# ------------------------------------------------------------------------------------------------
# MeshGraphNet family (apps/mgn_fullmlp, apps/mgn_linears, apps/test_mlp)
# ------------------------------------------------------------------------------------------------
def _mgn_checks(x, ws, bs, out, extra=()):
    _check_input("x", x, torch.float16)
    for i, (w, b) in enumerate(zip(ws, bs)):
        _check_input(f"w{i + 1}", w, torch.float16)
        _check_input(f"b{i + 1}", b, torch.float16)
    for name, t in extra:
        _check_input(name, t, torch.float16)
    _check_input("out", out, torch.float16)
    k0 = x.shape[1]
    shapes = [(k0, 128), (128, 128), (128, 128)]
    for i, (w, shp) in enumerate(zip(ws, shapes)):
        if tuple(w.shape) != shp:
            raise RuntimeError(f"w{i + 1} has shape {tuple(w.shape)}, expected {shp}")
    for i, b in enumerate(bs):
        if b is not None and tuple(b.shape) != (128,):
            raise RuntimeError(f"b{i + 1} has shape {tuple(b.shape)}, expected (128,)")
    if tuple(out.shape) != (x.shape[0], 128):
        raise RuntimeError(f"out has shape {tuple(out.shape)}, expected ({x.shape[0]}, 128)")


def mgn_fullmlp_out(x, w1, b1, w2, b2, w3, b3, gamma, beta, out) -> None:
    """x [M, K0] (K0 in 128/256/384) -> out [M, 128]; 3 Linear (ReLU, ReLU, none) + LayerNorm."""
    _mgn_checks(x, (w1, w2, w3), (b1, b2, b3), out, (("gamma", gamma), ("beta", beta)))
    with torch.cuda.device(x.device):
        L.check(L.lib().gp_mgn_fullmlp_out(x.shape[0], x.shape[1], _ptr(x), _ptr(w1), _ptr(b1),
                                           _ptr(w2), _ptr(b2), _ptr(w3), _ptr(b3), _ptr(gamma),
                                           _ptr(beta), _ptr(out), _stream(x)))


def mgn_fullmlp(x, w1, b1, w2, b2, w3, b3, gamma, beta) -> torch.Tensor:
    out = torch.zeros(x.shape[0], 128, dtype=x.dtype, device=x.device)
    mgn_fullmlp_out(x, w1, b1, w2, b2, w3, b3, gamma, beta, out)
    return out


def mgn_linears_out(x, w1, b1, w2, b2, w3, b3, out) -> None:
    _mgn_checks(x, (w1, w2, w3), (b1, b2, b3), out)
    with torch.cuda.device(x.device):
        L.check(L.lib().gp_mgn_linears_out(x.shape[0], x.shape[1], _ptr(x), _ptr(w1), _ptr(b1),
                                           _ptr(w2), _ptr(b2), _ptr(w3), _ptr(b3), _ptr(out),
                                           _stream(x)))


def mgn_linears(x, w1, b1, w2, b2, w3, b3) -> torch.Tensor:
    out = torch.zeros(x.shape[0], 128, dtype=x.dtype, device=x.device)
    mgn_linears_out(x, w1, b1, w2, b2, w3, b3, out)
    return out


def testmlp_out(x, w1, b1, w2, b2, w3, b3, out) -> None:
    if x.shape[1] != 128:
        raise RuntimeError(f"x has {x.shape[1]} columns, expected 128")
    _mgn_checks(x, (w1, w2, w3), (b1, b2, b3), out)
    with torch.cuda.device(x.device):
        L.check(L.lib().gp_testmlp_out(x.shape[0], _ptr(x), _ptr(w1), _ptr(b1), _ptr(w2),
                                       _ptr(b2), _ptr(w3), _ptr(b3), _ptr(out), _stream(x)))


def testmlp(x, w1, b1, w2, b2, w3, b3) -> torch.Tensor:
    out = torch.zeros(x.shape[0], 128, dtype=x.dtype, device=x.device)
    testmlp_out(x, w1, b1, w2, b2, w3, b3, out)
    return out


# ------------------------------------------------------------------------------------------------
# DLRM bottom MLP (apps/dlrm_botmlp), GraphCast MLPs (apps/gc_edges, apps/gc_nodes), NeRF
# ------------------------------------------------------------------------------------------------
def _out_like(x, n):
    return torch.zeros(x.shape[0], n, dtype=x.dtype, device=x.device)


def _check_chain(x, ws, bs, out, widths, dtype=torch.float16):
    """Shapes of a plain chain call: x [M, widths[0]], w_i [widths[i], widths[i+1]], b_i
    [widths[i+1]] (or None), out [M, widths[-1]]."""
    _check_input("x", x, dtype)
    _check_input("out", out, dtype)
    if x.dim() != 2 or x.shape[1] != widths[0]:
        raise RuntimeError(f"x has shape {tuple(x.shape)}, expected [M, {widths[0]}]")
    for i, (w, b) in enumerate(zip(ws, bs)):
        _check_input(f"w{i + 1}", w, dtype)
        _check_input(f"b{i + 1}", b, dtype)
        if w is None or tuple(w.shape) != (widths[i], widths[i + 1]):
            raise RuntimeError(f"w{i + 1} has shape {None if w is None else tuple(w.shape)}, "
                               f"expected {(widths[i], widths[i + 1])}")
        if b is not None and tuple(b.shape) != (widths[i + 1],):
            raise RuntimeError(f"b{i + 1} has shape {tuple(b.shape)}, expected ({widths[i + 1]},)")
    if out.dim() != 2 or tuple(out.shape) != (x.shape[0], widths[-1]):
        raise RuntimeError(f"out has shape {tuple(out.shape)}, expected [{x.shape[0]}, {widths[-1]}]")


def dlrm_botmlp_out(x, w1, b1, w2, b2, w3, b3, out) -> None:
    """x [M, K0] -> 512 -> 256 -> 128, ReLU after every layer. K0 = 32 is the reference app's own
    input (apps/dlrm_botmlp/pipelined/val.py:11-12, DlrmMlp([13 + 19, 512, 256, 128])); K0 = 16 is
    13 dense features zero padded (the benchmark config). Calls gp_dlrm_botmlp_out."""
    _check_input("x", x, torch.float16)
    k0 = x.shape[1] if x.dim() == 2 else -1
    _check_chain(x, [w1, w2, w3], [b1, b2, b3], out, [k0, 512, 256, 128])
    with torch.cuda.device(x.device):
        L.check(L.lib().gp_dlrm_botmlp_out(x.shape[0], k0, _ptr(x), _ptr(w1), _ptr(b1), _ptr(w2),
                                           _ptr(b2), _ptr(w3), _ptr(b3), _ptr(out), _stream(x)))


def dlrm_botmlp(x, w1, b1, w2, b2, w3, b3) -> torch.Tensor:
    out = _out_like(x, 128)
    dlrm_botmlp_out(x, w1, b1, w2, b2, w3, b3, out)
    return out


def gc_edges_out(x, w0, b0, w1, b1, ga, be, out, act=L.ACT_RELU) -> None:
    """x [M, 1536] -> 512 (act; ReLU as in the reference, SiLU for GraphCast) -> 512, LayerNorm."""
    fused_mlp_out(x, [w0, w1], [b0, b1], out, acts=[act, L.ACT_NONE], tail=L.TAIL_LAYERNORM,
                  gamma=ga, beta=be, ln_eps=1e-5)


def gc_edges(x, w0, b0, w1, b1, ga, be, act=L.ACT_RELU) -> torch.Tensor:
    out = _out_like(x, 512)
    gc_edges_out(x, w0, b0, w1, b1, ga, be, out, act=act)
    return out


gc_nodes_out = gc_edges_out  # x [M, 1024]; same chain shape after the first layer


def gc_nodes(x, w0, b0, w1, b1, ga, be, act=L.ACT_RELU) -> torch.Tensor:
    out = _out_like(x, 512)
    gc_nodes_out(x, w0, b0, w1, b1, ga, be, out, act=act)
    return out


def nerf_a_out(x, w1, b1, w2, b2, w3, b3, w4, b4, w5, b5, w6, b6, w7, b7, w8, b8, out) -> None:
    """NeRF trunk: x [M, 64] -> 256 (x5, ReLU), [h || x] -> 256 (w6 is [320, 256]), 256 x2."""
    fused_mlp_out(x, [w1, w2, w3, w4, w5, w6, w7, w8], [b1, b2, b3, b4, b5, b6, b7, b8], out,
                  acts=[L.ACT_RELU] * 8, skip_layer=5)


def nerf_a(x, *wb) -> torch.Tensor:
    out = _out_like(x, 256)
    nerf_a_out(x, *wb, out)
    return out


def nerf_out(x, weights, biases, out) -> None:
    """NeRF trunk + decode head 256 -> 4 (9 weights; the last one is [256, 4])."""
    fused_mlp_out(x, list(weights), list(biases), out, acts=[L.ACT_RELU] * 8 + [L.ACT_NONE],
                  skip_layer=5)


def _check_mgn_weights(k0, w1, b1, w2, b2, w3, b3, gamma, beta):
    for name, t, shape in (("w1", w1, (k0, 128)), ("w2", w2, (128, 128)), ("w3", w3, (128, 128)),
                           ("b1", b1, (128,)), ("b2", b2, (128,)), ("b3", b3, (128,)),
                           ("gamma", gamma, (128,)), ("beta", beta, (128,))):
        _check_input(name, t, torch.float16)
        if t is not None and tuple(t.shape) != shape:
            raise RuntimeError(f"{name} has shape {tuple(t.shape)}, expected {shape}")


def mgn_edge_update_out(nf, ef, srcs, dsts, w1, b1, w2, b2, w3, b3, gamma, beta, out,
                        agg=None) -> None:
    """MeshGraphNet edge update (graphmodel/mgn_dp.py:28-32) with the gather fused:
    out[e] = LN(MgnMlp([nf[srcs[e]] | ef[e] | nf[dsts[e]]])). nf [N, 128], ef [M, 128], srcs and
    dsts int64 [M], fp16. With agg (fp32 [N, 128]) the output rows are also summed into
    agg[dsts[e]] (accumulated onto agg's contents)."""
    _check_input("nf", nf, torch.float16)
    _check_input("ef", ef, torch.float16)
    _check_input("srcs", srcs, torch.int64)
    _check_input("dsts", dsts, torch.int64)
    _check_input("out", out, torch.float16)
    _check_input("agg", agg, torch.float32)
    m, n = ef.shape[0], nf.shape[0]
    if nf.dim() != 2 or nf.shape[1] != 128 or ef.dim() != 2 or ef.shape[1] != 128:
        raise RuntimeError(f"nf {tuple(nf.shape)} and ef {tuple(ef.shape)} must be [*, 128]")
    if tuple(srcs.shape) != (m,) or tuple(dsts.shape) != (m,):
        raise RuntimeError(f"srcs {tuple(srcs.shape)} and dsts {tuple(dsts.shape)} must be [{m}]")
    if tuple(out.shape) != (m, 128):
        raise RuntimeError(f"out has shape {tuple(out.shape)}, expected [{m}, 128]")
    if agg is not None and tuple(agg.shape) != (n, 128):
        raise RuntimeError(f"agg has shape {tuple(agg.shape)}, expected [{n}, 128]")
    _check_mgn_weights(384, w1, b1, w2, b2, w3, b3, gamma, beta)
    wp = (ctypes.c_void_p * 3)(w1.data_ptr(), w2.data_ptr(), w3.data_ptr())
    bp = (ctypes.c_void_p * 3)(*[None if t is None else t.data_ptr() for t in (b1, b2, b3)])
    with torch.cuda.device(ef.device):
        L.check(L.lib().gp_mgn_edge_update_out(m, n, _ptr(nf), _ptr(ef), _ptr(srcs), _ptr(dsts), wp,
                                               bp, _ptr(gamma), _ptr(beta), _ptr(out), _ptr(agg),
                                               _stream(ef)))


def mgn_edge_update(nf, ef, srcs, dsts, w1, b1, w2, b2, w3, b3, gamma, beta, agg=None):
    out = torch.empty(ef.shape[0], 128, dtype=ef.dtype, device=ef.device)
    mgn_edge_update_out(nf, ef, srcs, dsts, w1, b1, w2, b2, w3, b3, gamma, beta, out, agg=agg)
    return out


def mgn_node_update_out(nf, aggs, w1, b1, w2, b2, w3, b3, gamma, beta, out) -> None:
    """MeshGraphNet node update (graphmodel/mgn_dp.py:46-54): out = LN(MgnMlp([nf | aggs[0] |
    ...])), nf [N, 128] fp16, aggs: one or two fp32 [N, 128] edge-set aggregates (rounded to
    fp16 as the MLP input), w1 [128 (1 + len(aggs)), 128]."""
    aggs = list(aggs)
    _check_input("nf", nf, torch.float16)
    _check_input("out", out, torch.float16)
    n = nf.shape[0]
    if len(aggs) not in (1, 2):
        raise RuntimeError("one or two edge-set aggregates")
    for i, a in enumerate(aggs):
        _check_input(f"aggs[{i}]", a, torch.float32)
        if tuple(a.shape) != (n, 128):
            raise RuntimeError(f"aggs[{i}] has shape {tuple(a.shape)}, expected [{n}, 128]")
    if nf.dim() != 2 or nf.shape[1] != 128 or tuple(out.shape) != (n, 128):
        raise RuntimeError(f"nf {tuple(nf.shape)} and out {tuple(out.shape)} must be [{n}, 128]")
    _check_mgn_weights(128 * (1 + len(aggs)), w1, b1, w2, b2, w3, b3, gamma, beta)
    ap = (ctypes.c_void_p * 2)(*([a.data_ptr() for a in aggs] + [None] * (2 - len(aggs))))
    wp = (ctypes.c_void_p * 3)(w1.data_ptr(), w2.data_ptr(), w3.data_ptr())
    bp = (ctypes.c_void_p * 3)(*[None if t is None else t.data_ptr() for t in (b1, b2, b3)])
    with torch.cuda.device(nf.device):
        L.check(L.lib().gp_mgn_node_update_out(n, len(aggs), _ptr(nf), ap, wp, bp, _ptr(gamma),
                                               _ptr(beta), _ptr(out), _stream(nf)))


def mgn_node_update(nf, aggs, w1, b1, w2, b2, w3, b3, gamma, beta):
    out = torch.empty_like(nf)
    mgn_node_update_out(nf, aggs, w1, b1, w2, b2, w3, b3, gamma, beta, out)
    return out


_NERF_FULL_W = [(64, 256)] + [(256, 256)] * 4 + [(320, 256), (256, 256), (256, 256),
                (256, 64), (256, 256), (288, 128), (128, 64)]


def nerf_full_out(x, d, weights, biases, out_r, out_rgb) -> None:
    """NeRF with view directions (apps/nerf_full/pipelined/nerf_full_pl_ext.cu:22-95): x [M, 64],
    d [M, 32], weights w1..w12 ([K, N], shapes as the reference asserts), biases b1..b12 (entries
    may be None) -> out_r [M, 64] (alpha head), out_rgb [M, 64]. fp16."""
    _check_input("x", x, torch.float16)
    _check_input("d", d, torch.float16)
    _check_input("out_r", out_r, torch.float16)
    _check_input("out_rgb", out_rgb, torch.float16)
    m = x.shape[0]
    if x.dim() != 2 or x.shape[1] != 64:
        raise RuntimeError(f"x has shape {tuple(x.shape)}, expected [M, 64]")
    if tuple(d.shape) != (m, 32):
        raise RuntimeError(f"d has shape {tuple(d.shape)}, expected [{m}, 32]")
    for name, o in (("out_r", out_r), ("out_rgb", out_rgb)):
        if tuple(o.shape) != (m, 64):
            raise RuntimeError(f"{name} has shape {tuple(o.shape)}, expected [{m}, 64]")
    weights, biases = list(weights), list(biases) if biases is not None else [None] * 12
    if len(weights) != 12 or len(biases) != 12:
        raise RuntimeError("nerf_full takes 12 weights and 12 biases")
    for i, (wt, bt) in enumerate(zip(weights, biases)):
        _check_input(f"w{i + 1}", wt, torch.float16)
        _check_input(f"b{i + 1}", bt, torch.float16)
        if tuple(wt.shape) != _NERF_FULL_W[i]:
            raise RuntimeError(f"w{i + 1} has shape {tuple(wt.shape)}, expected {_NERF_FULL_W[i]}")
        if bt is not None and tuple(bt.shape) != (_NERF_FULL_W[i][1],):
            raise RuntimeError(f"b{i + 1} has shape {tuple(bt.shape)}, expected ({_NERF_FULL_W[i][1]},)")
    wp = (ctypes.c_void_p * 12)(*[wt.data_ptr() for wt in weights])
    bp = (ctypes.c_void_p * 12)(*[None if bt is None else bt.data_ptr() for bt in biases])
    with torch.cuda.device(x.device):
        L.check(L.lib().gp_nerf_full_out(m, _ptr(x), _ptr(d), wp, bp, _ptr(out_r), _ptr(out_rgb),
                                         _stream(x)))


def nerf_full(x, d, *wb):
    """nerf_full(x, d, w1, b1, ..., w12, b12) -> (out_r, out_rgb), like the reference's binding."""
    if len(wb) != 24:
        raise RuntimeError("nerf_full takes x, d and 12 (weight, bias) pairs")
    out_r = torch.zeros(x.shape[0], 64, dtype=x.dtype, device=x.device)
    out_rgb = torch.zeros_like(out_r)
    nerf_full_out(x, d, wb[0::2], wb[1::2], out_r, out_rgb)
    return out_r, out_rgb


def bert_ffn_out(x, w1, b1, w2, b2, ga, be, out, eps=None) -> None:
    """out = LN(x + W2 act(W1 x + b1) + b2).

    x [M, 128]: the reference's own BERT FFN (apps/bert_ffn: 128 -> 512 ReLU -> 128, LayerNorm eps
    1e-5), fp16 or bf16. x [M, 1024]: BERT-large (1024 -> 4096 GELU(tanh) -> 1024, eps 1e-12),
    bf16."""
    if x.dim() == 2 and x.shape[1] == 128:
        act0, eps = L.ACT_RELU, 1e-5 if eps is None else eps
    else:
        act0, eps = L.ACT_GELU_TANH, 1e-12 if eps is None else eps
    fused_mlp_out(x, [w1, w2], [b1, b2], out, acts=[act0, L.ACT_NONE],
                  tail=L.TAIL_RESIDUAL_LN, gamma=ga, beta=be, ln_eps=eps)


def bert_ffn(x, w1, b1, w2, b2, ga, be, eps=None) -> torch.Tensor:
    out = _out_like(x, x.shape[1])
    bert_ffn_out(x, w1, b1, w2, b2, ga, be, out, eps=eps)
    return out


def bert_addln_ffn_out(attn_out, x, w0, b0, w1, b1, w2, b2, ga0, be0, ga2, be2, out) -> None:
    """apps/bert_addln_ffn (H = 128, ff = 512, fp16): h = LN0(attn_out W0 + b0 + x),
    out = LN2(ReLU(h W1 + b1) W2 + b2 + h). Same argument order as the reference's
    bert_addln_ffn_out (bert_addln_ffn_pl_ext.cu:15-58)."""
    for name, t in (("attn_out", attn_out), ("x", x), ("out", out)):
        _check_input(name, t, torch.float16)
        if t.dim() != 2 or t.shape[1] != 128 or t.shape[0] != x.shape[0]:
            raise RuntimeError(f"{name} has shape {tuple(t.shape)}, expected [{x.shape[0]}, 128]")
    for name, w, shp in (("w0", w0, (128, 128)), ("w1", w1, (128, 512)), ("w2", w2, (512, 128))):
        _check_input(name, w, torch.float16)
        if tuple(w.shape) != shp:
            raise RuntimeError(f"{name} has shape {tuple(w.shape)}, expected {shp}")
    for name, t, n in (("b0", b0, 128), ("b1", b1, 512), ("b2", b2, 128), ("ga0", ga0, 128),
                       ("be0", be0, 128), ("ga2", ga2, 128), ("be2", be2, 128)):
        _check_input(name, t, torch.float16)
        if t is not None and tuple(t.shape) != (n,):
            raise RuntimeError(f"{name} has shape {tuple(t.shape)}, expected ({n},)")
    with torch.cuda.device(x.device):
        L.check(L.lib().gp_bert_addln_ffn_out(
            x.shape[0], _ptr(attn_out), _ptr(x), _ptr(w0), _ptr(b0), _ptr(w1), _ptr(b1), _ptr(w2),
            _ptr(b2), _ptr(ga0), _ptr(be0), _ptr(ga2), _ptr(be2), _ptr(out), _stream(x)))


def bert_addln_ffn(attn_out, x, w0, b0, w1, b1, w2, b2, ga0, be0, ga2, be2) -> torch.Tensor:
    """Allocating form. (The reference's passes be0 where be2 belongs,
    bert_addln_ffn_pl_ext.cu:74; this one passes be2.)"""
    out = _out_like(x, 128)
    bert_addln_ffn_out(attn_out, x, w0, b0, w1, b1, w2, b2, ga0, be0, ga2, be2, out)
    return out


def dlrm_interaction_out(bot, sparse, out) -> None:
    """DLRM feature interaction (graphmodel/dlrm.py:28-42): bot [M, 128] (bottom MLP output),
    sparse [M, 26, 128] (embedding vectors) -> out [M, 480] = [bot | 351 pairwise dot products
    below the diagonal, row-major | 0], the top MLP's input. fp16."""
    _check_input("bot", bot, torch.float16)
    _check_input("sparse", sparse, torch.float16)
    _check_input("out", out, torch.float16)
    m = bot.shape[0]
    if bot.dim() != 2 or bot.shape[1] != 128:
        raise RuntimeError(f"bot has shape {tuple(bot.shape)}, expected [M, 128]")
    if tuple(sparse.shape) != (m, 26, 128):
        raise RuntimeError(f"sparse has shape {tuple(sparse.shape)}, expected [{m}, 26, 128]")
    if tuple(out.shape) != (m, 480):
        raise RuntimeError(f"out has shape {tuple(out.shape)}, expected [{m}, 480]")
    with torch.cuda.device(bot.device):
        L.check(L.lib().gp_dlrm_interaction_out(m, _ptr(bot), _ptr(sparse), _ptr(out), _stream(bot)))


def dlrm_interaction(bot, sparse) -> torch.Tensor:
    out = torch.empty(bot.shape[0], 480, dtype=bot.dtype, device=bot.device)
    dlrm_interaction_out(bot, sparse, out)
    return out


def dlrm_topmlp_out(x, w1, b1, w2, b2, w3, b3, w4, b4, w5, b5, out) -> None:
    """Two width sets (gp_dlrm_topmlp_out):
      * x [M, 512] -> 1024 -> 1024 -> 512 -> 256 -> 64, ReLU after every layer: the reference
        app's own DlrmMlp([479 + 33, 1024, 1024, 512, 256, 64]) (apps/dlrm_topmlp/pipelined/val.py:11-12);
      * x [M, 480] -> 1024 -> 1024 -> 512 -> 256 (ReLU) -> 1 (sigmoid): DlrmMlp(..., sigmoid_i=4),
        the benchmark config."""
    _check_input("x", x, torch.float16)
    _check_input("w5", w5, torch.float16)
    k0 = x.shape[1] if x.dim() == 2 else -1
    n_out = w5.shape[1] if w5.dim() == 2 else -1
    ws, bs = [w1, w2, w3, w4, w5], [b1, b2, b3, b4, b5]
    _check_chain(x, ws, bs, out, [k0, 1024, 1024, 512, 256, n_out])
    wp = (ctypes.c_void_p * 5)(*[w.data_ptr() for w in ws])
    bp = (ctypes.c_void_p * 5)(*[(b.data_ptr() if b is not None else None) for b in bs])
    with torch.cuda.device(x.device):
        L.check(L.lib().gp_dlrm_topmlp_out(x.shape[0], k0, n_out, _ptr(x), wp, bp, _ptr(out),
                                           _stream(x)))


def dlrm_topmlp(x, *wb) -> torch.Tensor:
    out = _out_like(x, wb[8].shape[1])
    dlrm_topmlp_out(x, *wb, out)
    return out


def run_workload_host(w, x_host, weights, ln, out_host) -> None:
    """A plain-chain workloads.Workload end to end on host buffers (gp_fused_mlp_host)."""
    if w.block:
        raise RuntimeError(f"{w.name}: host pipeline covers plain chains only")
    gamma, beta = ln if ln is not None else (None, None)
    fused_mlp_host_out(x_host, [p[0] for p in weights], [p[1] for p in weights], out_host,
                       acts=w.acts, tail=w.tail, gamma=gamma, beta=beta, ln_eps=w.ln_eps,
                       skip_layer=w.skip_layer)


_SCRATCH = {}


def _scratch_f32(device, n):
    """A cached fp32 device buffer of at least n elements per device (grown, never shrunk)."""
    key = (device.type, device.index)
    buf = _SCRATCH.get(key)
    if buf is None or buf.numel() < n:
        buf = torch.empty(n, dtype=torch.float32, device=device)
        _SCRATCH[key] = buf
    return buf[:n]


def run_workload_out(w, x, weights, ln, out) -> None:
    """Run a workloads.Workload chain through the generic C entry point."""
    if w.block == "dlrm_interaction":
        m = x.shape[0] // 27
        dlrm_interaction_out(x[:m], x[m:].view(m, 26, x.shape[1]), out)
        return
    if w.block == "mgn_mp":
        ef, nf, srcs, dsts = W.split_mgn_input(x)
        m, n = ef.shape[0], nf.shape[0]
        o = out.view(-1)
        agg = _scratch_f32(x.device, n * 128).view(n, 128)
        agg.zero_()
        (e1, e2, e3, n1, n2, n3) = weights
        ge, be, gn, bn = ln
        mgn_edge_update_out(nf, ef, srcs, dsts, e1[0], e1[1], e2[0], e2[1], e3[0], e3[1], ge, be,
                            o[:m * 128].view(m, 128), agg=agg)
        mgn_node_update_out(nf, [agg], n1[0], n1[1], n2[0], n2[1], n3[0], n3[1], gn, bn,
                            o[m * 128:].view(n, 128))
        return
    if w.block == "nerf_full":
        m = x.numel() // 96
        o = out.view(-1)
        nerf_full_out(x[:m * 64].view(m, 64), x[m * 64:].view(m, 32), [p[0] for p in weights],
                      [p[1] for p in weights], o[:m * 64].view(m, 64), o[m * 64:].view(m, 64))
        return
    if w.block == "bert_addln":
        m = x.shape[0] // 2
        (w0, b0), (w1, b1), (w2, b2) = weights
        ga0, be0, ga2, be2 = ln
        bert_addln_ffn_out(x[:m], x[m:], w0, b0, w1, b1, w2, b2, ga0, be0, ga2, be2, out)
        return
    gamma, beta = ln if ln is not None else (None, None)
    fused_mlp_out(x, [p[0] for p in weights], [p[1] for p in weights], out, acts=w.acts,
                  tail=w.tail, gamma=gamma, beta=beta, ln_eps=w.ln_eps, skip_layer=w.skip_layer)
