"""ctypes binding of the C ABI in include/gpipes.h (libgpipes.so).

This is the same binding a reference-side maintainer would add in place of the pybind11 module
(`ext.cuda_ext`): it passes raw device pointers, sizes and the caller's stream, nothing else.
The library must exist: there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libgpipes.so"

GP_MAX_LAYERS = 10

GP_OK = 0
GP_ERR_ARG = -1
GP_ERR_SHAPE = -2
GP_ERR_ALIGN = -3
GP_ERR_UNSUPPORTED = -4
GP_ERR_CUDA = -5
GP_ERR_TIMEOUT = -6
GP_ERR_DRIVER = -7

STATUS_NAMES = {
    GP_OK: "GP_OK",
    GP_ERR_ARG: "GP_ERR_ARG",
    GP_ERR_SHAPE: "GP_ERR_SHAPE",
    GP_ERR_ALIGN: "GP_ERR_ALIGN",
    GP_ERR_UNSUPPORTED: "GP_ERR_UNSUPPORTED",
    GP_ERR_CUDA: "GP_ERR_CUDA",
    GP_ERR_TIMEOUT: "GP_ERR_TIMEOUT",
    GP_ERR_DRIVER: "GP_ERR_DRIVER",
}

GP_F16 = 0
GP_BF16 = 1

ACT_NONE, ACT_RELU, ACT_GELU_TANH, ACT_SILU, ACT_SIGMOID = 0, 1, 2, 3, 4
TAIL_NONE, TAIL_LAYERNORM, TAIL_RESIDUAL_LN = 0, 1, 2

# every symbol include/gpipes.h declares
EXPORTED_SYMBOLS = (
    "gp_fused_mlp_out",
    "gp_mgn_fullmlp_out",
    "gp_mgn_linears_out",
    "gp_testmlp_out",
    "gp_dlrm_botmlp_out",
    "gp_gc_edges_out",
    "gp_gc_nodes_out",
    "gp_bert_ffn_out",
    "gp_bert_addln_ffn_out",
    "gp_dlrm_interaction_out",
    "gp_dlrm_topmlp_out",
    "gp_nerf_a_out",
    "gp_nerf_out",
    "gp_nerf_full_out",
    "gp_fused_mlp_host",
    "gp_mgn_edge_update_out",
    "gp_mgn_node_update_out",
    "gp_gc_edges_bf16_noalloc_out",
    "gp_last_error",
    "gp_device_status",
    "gp_set_timeout_ns",
    "gp_set_fault_injection",
    "gp_launch_count",
    "gp_debug_pdl_flags",
    "gp_set_kernel_variant",
)


class GpError(RuntimeError):
    """Raised when a gp_* call returns a non-zero status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {message}")
        self.code = code


class GpSpec(ctypes.Structure):
    _fields_ = [
        ("n_layers", ctypes.c_int),
        ("widths", ctypes.c_int * (GP_MAX_LAYERS + 1)),
        ("act", ctypes.c_int * GP_MAX_LAYERS),
        ("tail", ctypes.c_int),
        ("dtype", ctypes.c_int),
        ("ln_eps", ctypes.c_float),
        ("skip_layer", ctypes.c_int),
    ]


_lib = None

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_INT = ctypes.c_int


def _declare(lib: ctypes.CDLL) -> None:
    lib.gp_fused_mlp_out.argtypes = [ctypes.POINTER(GpSpec), _I64, _P, ctypes.POINTER(_P),
                                     ctypes.POINTER(_P), _P, _P, _P, _P]
    lib.gp_fused_mlp_out.restype = _INT
    lib.gp_mgn_fullmlp_out.argtypes = [_I64, _INT] + [_P] * 11
    lib.gp_mgn_fullmlp_out.restype = _INT
    lib.gp_mgn_linears_out.argtypes = [_I64, _INT] + [_P] * 9
    lib.gp_mgn_linears_out.restype = _INT
    lib.gp_testmlp_out.argtypes = [_I64] + [_P] * 9
    lib.gp_testmlp_out.restype = _INT
    lib.gp_dlrm_botmlp_out.argtypes = [_I64, _INT] + [_P] * 9
    lib.gp_dlrm_botmlp_out.restype = _INT
    for name in ("gp_gc_edges_out", "gp_gc_nodes_out"):
        getattr(lib, name).argtypes = [_I64, _INT, _INT] + [_P] * 9
        getattr(lib, name).restype = _INT
    for name in ("gp_nerf_a_out", "gp_nerf_out"):
        getattr(lib, name).argtypes = [_I64, _P, ctypes.POINTER(_P), ctypes.POINTER(_P), _P, _P]
        getattr(lib, name).restype = _INT
    lib.gp_bert_ffn_out.argtypes = [_I64] + [_P] * 7 + [ctypes.c_float, _P, _P]
    lib.gp_bert_ffn_out.restype = _INT
    lib.gp_bert_addln_ffn_out.argtypes = [_I64] + [_P] * 14
    lib.gp_bert_addln_ffn_out.restype = _INT
    lib.gp_fused_mlp_host.argtypes = [ctypes.POINTER(GpSpec), _I64, _P, ctypes.POINTER(_P),
                                      ctypes.POINTER(_P), _P, _P, _P, _I64, _P]
    lib.gp_fused_mlp_host.restype = _INT
    lib.gp_mgn_edge_update_out.argtypes = [_I64, _I64, _P, _P, _P, _P, ctypes.POINTER(_P),
                                           ctypes.POINTER(_P), _P, _P, _P, _P, _P]
    lib.gp_mgn_edge_update_out.restype = _INT
    lib.gp_mgn_node_update_out.argtypes = [_I64, _INT, _P, ctypes.POINTER(_P), ctypes.POINTER(_P),
                                           ctypes.POINTER(_P), _P, _P, _P, _P]
    lib.gp_mgn_node_update_out.restype = _INT
    lib.gp_nerf_full_out.argtypes = [_I64, _P, _P, ctypes.POINTER(_P), ctypes.POINTER(_P), _P, _P, _P]
    lib.gp_nerf_full_out.restype = _INT
    lib.gp_dlrm_interaction_out.argtypes = [_I64, _P, _P, _P, _P]
    lib.gp_dlrm_interaction_out.restype = _INT
    lib.gp_dlrm_topmlp_out.argtypes = [_I64, _INT, _INT, _P, ctypes.POINTER(_P), ctypes.POINTER(_P), _P, _P]
    lib.gp_dlrm_topmlp_out.restype = _INT
    lib.gp_gc_edges_bf16_noalloc_out.argtypes = [_I64, _INT] + [_P] * 9
    lib.gp_gc_edges_bf16_noalloc_out.restype = _INT
    lib.gp_last_error.argtypes = []
    lib.gp_last_error.restype = ctypes.c_char_p
    lib.gp_device_status.argtypes = [_INT, _INT, ctypes.POINTER(_INT)]
    lib.gp_device_status.restype = _INT
    lib.gp_set_timeout_ns.argtypes = [ctypes.c_uint64]
    lib.gp_set_timeout_ns.restype = _INT
    lib.gp_set_fault_injection.argtypes = [_INT]
    lib.gp_set_fault_injection.restype = _INT
    lib.gp_set_kernel_variant.argtypes = [_INT]
    lib.gp_set_kernel_variant.restype = _INT
    lib.gp_launch_count.argtypes = []
    lib.gp_launch_count.restype = ctypes.c_uint64
    lib.gp_debug_pdl_flags.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                       ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_int),
                                       ctypes.c_int]
    lib.gp_debug_pdl_flags.restype = ctypes.c_int


def lib() -> ctypes.CDLL:
    """Load libgpipes.so (once). Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with __graft_entry__.build() "
                "(there is no non-CUDA fallback)")
        h = ctypes.CDLL(str(LIB_PATH), mode=os.RTLD_NOW | getattr(os, "RTLD_LOCAL", 0))
        _declare(h)
        _lib = h
    return _lib


def last_error() -> str:
    return lib().gp_last_error().decode(errors="replace")


def check(code: int) -> None:
    if code != GP_OK:
        raise GpError(code, last_error())


def make_spec(widths, acts, tail=TAIL_NONE, dtype=GP_F16, ln_eps=1e-5, skip_layer=0) -> GpSpec:
    s = GpSpec()
    n = len(widths) - 1
    if n < 1 or n > GP_MAX_LAYERS:
        raise ValueError(f"layer count {n} out of range")
    s.n_layers = n
    for i, w in enumerate(widths):
        s.widths[i] = int(w)
    for i, a in enumerate(acts):
        s.act[i] = int(a)
    s.tail = int(tail)
    s.dtype = int(dtype)
    s.ln_eps = float(ln_eps)
    s.skip_layer = int(skip_layer)
    return s


def device_status(device: int, clear: bool = False) -> int:
    st = ctypes.c_int(0)
    check(lib().gp_device_status(int(device), 1 if clear else 0, ctypes.byref(st)))
    return st.value


def set_timeout_ns(ns: int) -> None:
    check(lib().gp_set_timeout_ns(int(ns)))


def set_fault_injection(mode: int) -> None:
    check(lib().gp_set_fault_injection(int(mode)))


def set_kernel_variant(v: int) -> None:
    check(lib().gp_set_kernel_variant(int(v)))


def launch_count() -> int:
    return int(lib().gp_launch_count())


def pdl_flags(stream: int, ranges, record: bool = True) -> int:
    """gp_debug_pdl_flags: ranges are (address, bytes, kind) with kind 0 parameter, 1 input rows,
    2 written, 3 writes not listed. Returns the early-read bits (negative on error)."""
    n = len(ranges)
    ptrs = (ctypes.c_void_p * max(n, 1))(*[r[0] for r in ranges])
    sizes = (ctypes.c_uint64 * max(n, 1))(*[r[1] for r in ranges])
    kinds = (ctypes.c_int * max(n, 1))(*[r[2] for r in ranges])
    return int(lib().gp_debug_pdl_flags(ctypes.c_void_p(stream), n, ptrs, sizes, kinds, int(record)))
