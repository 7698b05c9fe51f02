"""C ABI checks that need no GPU: the library loads, exports every declared symbol, and rejects
bad arguments before touching CUDA."""
import ctypes
import re
from pathlib import Path

import pytest

from gpu_pipes_b200 import _lib as L

HEADER = Path(__file__).resolve().parent.parent / "include" / "gpipes.h"


def test_header_symbols_exported():
    declared = set(re.findall(r"GP_API\s+[\w\s\*]+?\b(gp_\w+)\s*\(", HEADER.read_text()))
    assert declared, "no declarations parsed"
    assert declared == set(L.EXPORTED_SYMBOLS)
    lib = L.lib()
    for name in declared:
        assert hasattr(lib, name), name


def _fake(addr):
    return ctypes.c_void_p(addr)


def _call(spec, m=256, x=0x10000, w=None, b=None, out=0x20000):
    n = spec.n_layers if spec is not None else 1
    w = w or [0x30000 + 0x1000 * i for i in range(max(n, 1))]
    wp = (ctypes.c_void_p * len(w))(*w)
    bp = None if b is None else (ctypes.c_void_p * len(b))(*b)
    return L.lib().gp_fused_mlp_out(None if spec is None else ctypes.byref(spec), m, _fake(x), wp,
                                    bp, None, None, _fake(out), None)


def mgn(k0=384, tail=L.TAIL_LAYERNORM, dtype=L.GP_F16):
    return L.make_spec([k0, 128, 128, 128], [L.ACT_RELU, L.ACT_RELU, L.ACT_NONE], tail, dtype)


def test_rejects_null_spec():
    assert _call(None) == L.GP_ERR_ARG
    assert "spec" in L.last_error()


def test_rejects_bad_shapes():
    s = mgn()
    s.n_layers = 0
    assert _call(s) == L.GP_ERR_SHAPE
    s = mgn()
    s.widths[2] = 0
    assert _call(s) == L.GP_ERR_SHAPE
    s = mgn()
    s.widths[0] = 100  # input rows must be a multiple of 16 bytes
    assert _call(s) == L.GP_ERR_SHAPE
    s = mgn()
    s.skip_layer = 3  # past the last layer
    assert _call(s) == L.GP_ERR_SHAPE
    assert _call(mgn(), m=-1) == L.GP_ERR_ARG
    assert _call(mgn(), m=2**31) == L.GP_ERR_SHAPE


def test_rejects_null_and_misaligned_pointers():
    assert _call(mgn(), x=0) == L.GP_ERR_ARG
    assert _call(mgn(), out=0) == L.GP_ERR_ARG
    assert _call(mgn(), x=0x10008) == L.GP_ERR_ALIGN
    assert _call(mgn(), w=[0x30000, 0x31002, 0x32000]) == L.GP_ERR_ALIGN
    assert _call(mgn(), b=[0x40000, 0x40002, 0x40004]) == L.GP_ERR_ALIGN


def test_unsupported_chain():
    s = L.make_spec([384, 136, 128], [L.ACT_RELU, L.ACT_NONE])
    assert _call(s) == L.GP_ERR_UNSUPPORTED
    assert "no compiled kernel" in L.last_error()


def test_empty_input_is_noop():
    # m == 0 returns before any CUDA call (no device needed)
    assert _call(mgn(), m=0) == L.GP_OK
    assert _call(mgn(256), m=0) == L.GP_OK


def test_residual_tail_shape_rule():
    s = L.make_spec([1024, 4096, 512], [L.ACT_GELU_TANH, L.ACT_NONE], L.TAIL_RESIDUAL_LN, L.GP_BF16)
    assert _call(s) == L.GP_ERR_SHAPE


def test_knobs():
    L.set_timeout_ns(10**6)
    L.set_timeout_ns(0)
    L.set_fault_injection(0)
    with pytest.raises(L.GpError):
        L.set_fault_injection(7)
    assert L.launch_count() >= 0


P = ctypes.c_void_p


def _arr(vals):
    return (ctypes.c_void_p * len(vals))(*vals)


def _edge(m=256, n=100, nf=0x10000, ef=0x20000, src=0x30000, dst=0x38000, w=(0x40000, 0x50000, 0x60000),
          b=None, agg=None, out=0x70000):
    return L.lib().gp_mgn_edge_update_out(m, n, P(nf), P(ef), P(src), P(dst), _arr(list(w)),
                                          None if b is None else _arr(list(b)), None, None, P(out),
                                          None if agg is None else P(agg), None)


def test_mgn_edge_update_argument_checks():
    assert _edge(m=0) == L.GP_OK  # nothing to do, no device touched
    assert _edge(m=-1) == L.GP_ERR_ARG
    assert _edge(m=2**31) == L.GP_ERR_SHAPE
    assert _edge(n=0) == L.GP_ERR_ARG
    assert _edge(n=2**25 + 1) == L.GP_ERR_SHAPE  # 32-bit node row offsets in the kernel
    assert _edge(nf=0) == L.GP_ERR_ARG
    assert _edge(dst=0) == L.GP_ERR_ARG
    assert _edge(ef=0x20008) == L.GP_ERR_ALIGN
    assert _edge(src=0x30004) == L.GP_ERR_ALIGN
    assert _edge(agg=0x80004) == L.GP_ERR_ALIGN
    assert _edge(w=(0x40000, 0x50002, 0x60000)) == L.GP_ERR_ALIGN
    assert _edge(b=(0x90000, 0x90002, None)) == L.GP_ERR_ALIGN


def _node(n=256, n_sets=1, nf=0x10000, aggs=(0x20000, 0x28000), w=(0x40000, 0x50000, 0x60000),
          out=0x70000):
    return L.lib().gp_mgn_node_update_out(n, n_sets, P(nf), _arr(list(aggs)), _arr(list(w)), None,
                                          None, None, P(out), None)


def test_mgn_node_update_argument_checks():
    assert _node(n=0) == L.GP_OK
    assert _node(n=-5) == L.GP_ERR_ARG
    assert _node(n_sets=3) == L.GP_ERR_UNSUPPORTED
    assert _node(n_sets=0) == L.GP_ERR_UNSUPPORTED
    assert _node(nf=0) == L.GP_ERR_ARG
    assert _node(n_sets=2, aggs=(0x20000, 0x28004)) == L.GP_ERR_ALIGN
    assert _node(out=0x70002) == L.GP_ERR_ALIGN


def _nerf_full(m=256, x=0x10000, d=0x18000, w=None, out_r=0x70000, out_rgb=0x78000):
    w = list(w) if w is not None else [0x100000 + 0x10000 * i for i in range(12)]
    return L.lib().gp_nerf_full_out(m, P(x), P(d), _arr(w), None, P(out_r), P(out_rgb), None)


def test_nerf_full_argument_checks():
    assert _nerf_full(m=0) == L.GP_OK
    assert _nerf_full(m=-1) == L.GP_ERR_ARG
    assert _nerf_full(d=0) == L.GP_ERR_ARG
    assert _nerf_full(out_rgb=0) == L.GP_ERR_ARG
    w = [0x100000 + 0x10000 * i for i in range(12)]
    w[9] = 0
    assert _nerf_full(w=w) == L.GP_ERR_ARG and "w[9]" in L.last_error()
    w[9] = 0x190008
    assert _nerf_full(w=w) == L.GP_ERR_ALIGN
    assert _nerf_full(x=0x10002) == L.GP_ERR_ALIGN


def test_dlrm_interaction_argument_checks():
    f = L.lib().gp_dlrm_interaction_out
    assert f(0, P(0x10000), P(0x20000), P(0x30000), None) == L.GP_OK
    assert f(-1, P(0x10000), P(0x20000), P(0x30000), None) == L.GP_ERR_ARG
    assert f(64, None, P(0x20000), P(0x30000), None) == L.GP_ERR_ARG
    assert f(64, P(0x10000), P(0x20008), P(0x30000), None) == L.GP_ERR_ALIGN


def test_fused_mlp_host_argument_checks():
    f = L.lib().gp_fused_mlp_host
    s = mgn(256)
    w = _arr([0x30000, 0x31000, 0x32000])
    assert f(None, 16, P(0x1000), w, None, None, None, P(0x2000), 0, None) == L.GP_ERR_ARG
    assert f(ctypes.byref(s), -1, P(0x1000), w, None, None, None, P(0x2000), 0, None) == L.GP_ERR_ARG
    assert f(ctypes.byref(s), 0, P(0x1000), w, None, None, None, P(0x2000), 0, None) == L.GP_OK
    assert f(ctypes.byref(s), 16, None, w, None, None, None, P(0x2000), 0, None) == L.GP_ERR_ARG


def _noalloc(m=256, act=L.ACT_SILU, x=0x10000, w0=0x30000, w1=0x40000, out=0x20000):
    return L.lib().gp_gc_edges_bf16_noalloc_out(m, act, _fake(x), _fake(w0), None, _fake(w1), None,
                                                None, None, _fake(out), None)


def test_noalloc_rejects_bad_arguments():
    """The allocation-free entry point checks its arguments before any CUDA call."""
    assert _noalloc(act=L.ACT_GELU_TANH) == L.GP_ERR_UNSUPPORTED
    assert "act" in L.last_error()
    assert _noalloc(act=L.ACT_NONE) == L.GP_ERR_UNSUPPORTED
    assert _noalloc(x=0x10008) == L.GP_ERR_ALIGN
    assert _noalloc(out=0x20002) == L.GP_ERR_ALIGN
    assert _noalloc(w1=0x40004) == L.GP_ERR_ALIGN
    assert _noalloc(x=0) == L.GP_ERR_ARG
    assert _noalloc(m=-1) == L.GP_ERR_ARG
    assert _noalloc(m=2**31) == L.GP_ERR_SHAPE
    assert _noalloc(m=0) == L.GP_OK
    assert L.last_error() == ""  # a successful call clears the previous message


def test_dlrm_entry_points_reject_uncompiled_widths():
    """Only the compiled width sets are accepted: bottom k0 16 / 32, top (480, 1) / (512, 64)."""
    lib = L.lib()
    w = (ctypes.c_void_p * 5)(*[0x30000 + 0x1000 * i for i in range(5)])
    assert lib.gp_dlrm_botmlp_out(256, 48, _fake(0x10000), _fake(0x30000), None, _fake(0x31000),
                                  None, _fake(0x32000), None, _fake(0x20000), None) == L.GP_ERR_UNSUPPORTED
    assert lib.gp_dlrm_topmlp_out(256, 512, 1, _fake(0x10000), w, None, _fake(0x20000), None) == L.GP_ERR_UNSUPPORTED
    assert lib.gp_dlrm_topmlp_out(256, 480, 64, _fake(0x10000), w, None, _fake(0x20000), None) == L.GP_ERR_UNSUPPORTED


def test_kernel_variant_range():
    """Forms 0-2 are selectable (a chain without the requested form runs its default); others are
    rejected."""
    lib = L.lib()
    try:
        for v in (0, 1, 2):
            assert lib.gp_set_kernel_variant(v) == L.GP_OK
        assert lib.gp_set_kernel_variant(3) == L.GP_ERR_ARG
        assert lib.gp_set_kernel_variant(-1) == L.GP_ERR_ARG
    finally:
        lib.gp_set_kernel_variant(0)
