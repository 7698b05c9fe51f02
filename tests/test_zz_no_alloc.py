"""The allocation-free GraphCast entry point (gp_gc_edges_bf16_noalloc_out).

It exists for callers that may not allocate GPU memory while running -- frameworks that own every
device allocation, or serving loops that must never enter an allocator -- and keeps its scratch
(the fp16 copy of the second layer's weights) in a fixed buffer compiled into the library. This
test calls it through the C ABI twice in a row and checks each result against the regular entry
point (gp_gc_edges_out), which obtains its scratch on the caller's stream, using the same
tolerance as the other parity tests. This file sorts last so that a run stopping at the first
failure has already run every other test; it also passes when run on its own.
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


def test_noalloc_matches_regular_entry_point(cuda_dev):
    lib = L.lib()
    w = W.GC_EDGE.with_m(5000)
    x = W.make_input(w).to(cuda_dev)
    layers, ln = W.make_weights(w)
    (w0, b0), (w1, b1) = [(a.to(cuda_dev), b.to(cuda_dev)) for a, b in layers]
    ga, be = (t.to(cuda_dev) for t in ln)
    stream = ctypes.c_void_p(torch.cuda.current_stream(cuda_dev).cuda_stream)

    ref = torch.empty(w.m, 512, dtype=torch.bfloat16, device=cuda_dev)
    L.check(lib.gp_gc_edges_out(w.m, L.GP_BF16, L.ACT_SILU, _p(x), _p(w0), _p(b0), _p(w1), _p(b1),
                                _p(ga), _p(be), _p(ref), stream))
    torch.cuda.synchronize()
    for call in range(2):
        out = torch.full((w.m, 512), float("nan"), dtype=torch.bfloat16, device=cuda_dev)
        L.check(lib.gp_gc_edges_bf16_noalloc_out(w.m, L.ACT_SILU, _p(x), _p(w0), _p(b0), _p(w1),
                                                 _p(b1), _p(ga), _p(be), _p(out), stream))
        torch.cuda.synchronize()
        r = O.compare(out.float().cpu(), ref.float().cpu())
        assert r["ok"], f"call {call}: {r}"
