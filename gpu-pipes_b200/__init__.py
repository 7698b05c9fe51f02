"""B200-native fused multi-layer MLP (the hot path of medav/gpu-pipes), sm_100a only.

Import name: ``gpu_pipes_b200`` (the directory is ``gpu-pipes_b200``; ``__graft_entry__`` and the
tests register it under that name). Submodules:
  _lib       ctypes binding of the C ABI (include/gpipes.h, libgpipes.so)
  cuda_ext   the reference's per-app entry points (mgn_fullmlp, mgn_fullmlp_out, ...)
  workloads  layer chains, FLOP/byte counts, seeded data
  build      nvcc build of libgpipes.so
"""
import importlib

from . import _lib, workloads  # noqa: F401

__all__ = ["_lib", "workloads", "cuda_ext", "build"]


def __getattr__(name):
    if name in ("cuda_ext", "build"):
        return importlib.import_module(f"{__name__}.{name}")
    raise AttributeError(name)
