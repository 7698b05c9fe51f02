"""The allocation-free GraphCast entry point (gp_gc_edges_bf16_noalloc_out).

It exists for callers that may not allocate GPU memory while running -- frameworks that own every
device allocation, or serving loops that must never enter an allocator -- and keeps its scratch
(the fp16 copy of the second layer's weights) in a fixed buffer compiled into the library. These
tests call it through the C ABI, two calls in a row, for both compiled activations, and check each
result against the regular entry point (gp_gc_edges_out, whose scratch comes from the library's
workspace) and against the fp32 oracle, with the tolerance of the other parity tests. A host-side
fault injection makes its device waits run out; the status word reports it through
gp_device_status and the next call is correct. This file sorts last so that a run stopping at the
first failure has already run every other test; it also passes when run on its own.
"""
import ctypes

import pytest
import torch

from gpu_pipes_b200 import _lib as L
from gpu_pipes_b200 import workloads as W
from oracle import mlp_oracle as O

pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _case(dev, m=5000):
    w = W.GC_EDGE.with_m(m)
    x = W.make_input(w)
    layers, ln = W.make_weights(w)
    d = dict(x=x.to(dev), layers=[(a.to(dev), b.to(dev)) for a, b in layers],
             ln=tuple(t.to(dev) for t in ln))
    return w, x, layers, ln, d


def _noalloc(lib, act, d, out, stream):
    (w0, b0), (w1, b1) = d["layers"]
    ga, be = d["ln"]
    return lib.gp_gc_edges_bf16_noalloc_out(out.shape[0], act, _p(d["x"]), _p(w0), _p(b0), _p(w1),
                                            _p(b1), _p(ga), _p(be), _p(out), stream)


@pytest.mark.parametrize("act", [L.ACT_SILU, L.ACT_RELU], ids=["silu", "relu"])
def test_noalloc_matches_regular_entry_point(cuda_dev, act):
    lib = L.lib()
    w, x, layers, ln, d = _case(cuda_dev)
    (w0, b0), (w1, b1) = d["layers"]
    ga, be = d["ln"]
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)

    ref = torch.empty(w.m, 512, dtype=torch.bfloat16, device=cuda_dev)
    L.check(lib.gp_gc_edges_out(w.m, L.GP_BF16, act, _p(d["x"]), _p(w0), _p(b0), _p(w1), _p(b1),
                                _p(ga), _p(be), _p(ref), stream))
    torch.cuda.synchronize()
    oracle = O.gc_edges(x, layers, ln, act, 1e-5)
    for call in range(2):
        out = torch.full((w.m, 512), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
        n0 = L.launch_count()
        L.check(_noalloc(lib, act, d, out, stream))
        assert L.launch_count() == n0 + 2
        torch.cuda.synchronize()
        r = O.compare(out.float().cpu(), ref.float().cpu())
        assert r["ok"], f"call {call} vs regular entry point: {r}"
        r = O.compare(out.float().cpu(), oracle)
        assert r["ok"], f"call {call} vs oracle: {r}"
    assert L.device_status(0) == 0


def test_noalloc_timeout_is_reported(cuda_dev):
    """The producer skips its loads (host-side injection), every consumer wait runs out after 5 ms,
    the status word says so, and the next call on the same context is correct."""
    lib = L.lib()
    w, x, layers, ln, d = _case(cuda_dev, m=2048)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)
    out = torch.empty(w.m, 512, dtype=torch.bfloat16, device=cuda_dev)
    assert L.device_status(0, clear=True) == 0
    try:
        L.set_timeout_ns(5_000_000)
        L.set_fault_injection(1)
        L.check(_noalloc(lib, L.ACT_SILU, d, out, stream))
        torch.cuda.synchronize()
    finally:
        L.set_fault_injection(0)
        L.set_timeout_ns(0)
    st = L.device_status(0, clear=True)
    assert st in (0x100, 0x200, 0x300), hex(st)
    assert L.device_status(0) == 0
    L.check(_noalloc(lib, L.ACT_SILU, d, out, stream))
    torch.cuda.synchronize()
    r = O.compare(out.float().cpu(), O.gc_edges(x, layers, ln, L.ACT_SILU, 1e-5))
    assert r["ok"], f"after timeout: {r}"
