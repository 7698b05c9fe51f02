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
