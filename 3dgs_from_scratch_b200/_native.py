"""ctypes binding of lib3dgs_b200.so (the C ABI declared in include/gs_b200.h).

The library is the only compute path: if it cannot be loaded this module
raises, there is no fallback. Pointers are passed as integers (tensor
data_ptr()), streams as the raw cudaStream_t of torch's current stream.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib3dgs_b200.so")

GS_OK = 0
GS_ERR_INVALID_ARGUMENT = 1
GS_ERR_CUDA = 2
GS_ERR_DEVICE_TIMEOUT = 3
GS_ERR_CAPACITY = 4
GS_ERR_PEER = 5
_MESSAGES = {
    GS_ERR_INVALID_ARGUMENT: "invalid argument (size, pointer or alignment)",
    GS_ERR_CUDA: "CUDA error",
    GS_ERR_DEVICE_TIMEOUT: "a bounded device-side wait timed out",
    GS_ERR_CAPACITY: "capacity exceeded (scratch too small or count >= 2^30)",
    GS_ERR_PEER: "another rank reported an error in this step (update skipped on every rank)",
}

P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
F = ctypes.c_float
SZ = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/gs_b200.h
SIGNATURES = {
    "gs_version": (I, []),
    "gs_last_cuda_error": (I, []),
    "gs_launch_count": (ctypes.c_uint64, []),
    "gs_note_launches": (None, [I64]),
    "gs_check_status": (I, [P]),
    "gs_sync": (I, [P]),
    "gs_selftest_bounded_wait": (I, [P, P]),
    "gs_selftest_set_timeout": (I, [P, P]),
    "gs_status_export": (I, [P, P]),
    "gs_status_merge": (I, [P, P]),
    "gs_project_points": (I, [I, P, P, P, P, P, P, F, F, F, F, F, I, I, P, P, P, P, P, P, P]),
    "gs_project_points_backward": (I, [I, P, P, P, P, P, P, P, P, P, I, I, P, P, P, P]),
    "gs_evaluate_sh": (I, [I, P, P, P, P, P, I, P, P]),
    "gs_evaluate_sh_backward": (I, [I, P, P, P, P, P, P, I, P, P, P, P]),
    "gs_count_tiles": (I, [I, P, P, P, I, I, P, P]),
    "gs_scan_scratch_bytes": (SZ, [I]),
    "gs_exclusive_scan": (I, [I, P, P, P, P, SZ, P]),
    "gs_exclusive_scan_noalloc": (I, [I, P, P, P, P]),
    "gs_read_total": (I, [P, P, P]),
    "gs_tile_layout_scratch_bytes": (SZ, [I, I64, I, I]),
    "gs_tile_layout": (I, [I, P, P, P, P, I64, I, I, P, P, P, P, SZ, P]),
    "gs_tile_layout_capped": (I, [I, P, P, P, P, I64, I, I, P, P, P, P, SZ, P]),
    "gs_tile_bins_scratch_bytes": (SZ, [I, I64, I, I]),
    "gs_tile_bins": (I, [I, P, P, P, P, I64, I, I, P, P, P, P, SZ, P, P]),
    "gs_tile_layout_views_scratch_bytes": (SZ, [I, I, P, I, I]),
    "gs_tile_layout_views": (I, [I, I, P, P, P, P, P, I, I, P, P, P, SZ, P]),
    "gs_sort_scratch_bytes": (SZ, [I64]),
    "gs_sort_pairs": (I, [I64, P, P, P, P, I, P, SZ, P]),
    "gs_rasterize": (I, [I, P, I64, P, I, P, P, P, P, I, I, F, F, F, P, P, P, P]),
    "gs_rasterize_backward": (I, [I, P, I64, P, I, P, P, P, P, P, I, I, F, F, F, P, P, P, P, P,
                                  P, P]),
    "gs_preprocess_forward": (I, [I, P, P, P, P, P, P, P, P, P, F, F, F, F, F, I, I, I, I, P, P,
                                  P, P, P, P, P, P]),
    "gs_blend_forward": (I, [I, P, I64, P, I, P, P, I, I, F, F, F, P, P, P, P, P, P]),
    "gs_blend_backward": (I, [I, P, I64, P, I, P, P, P, P, P, I, I, F, F, F, P, P, P, P, P]),
    "gs_tile_order": (I, [I, P, I64, P, P]),
    "gs_l1_loss_grad": (I, [I64, P, P, I, P, P, P]),
    "gs_adam_table_bytes": (SZ, []),
    "gs_adam_table": (I, [I64, I, P, P, P, F, F, I64, P, SZ]),
    "gs_adam_step_table": (I, [I64, P, P, P, P, P, F, F, P]),
    "gs_adam_step_ranges": (I, [P, P, P, P, I, P, P, P, F, F, P]),
    "gs_adam_step": (I, [I64, P, P, P, P, I, P, P, P, F, F, I64, P]),
    "gs_ssim_scratch_bytes": (SZ, [I, I, I]),
    "gs_densify_accumulate": (I, [I, P, P, I, I, P, P, P]),
    "gs_densify_plan": (I, [I, P, P, P, P, F, I, F, F, F, P, P, P, P, P]),
    "gs_densify_apply": (I, [I, P, P, P, P, I64, I64, I64, P, P, P, P, P, P, P, P, P,
                             ctypes.c_uint64, F, P]),
    "gs_reset_opacities": (I, [I, P, P, P, F, P]),
    "gs_dp_flag_words": (SZ, [I]),
    "gs_dp_max_blocks": (I, []),
    "gs_dp_adam_step": (I, [I, I, P, P, P, P, P, I64, P, P, I, P, P, P, F, F, I64, ctypes.c_uint32,
                            I, P, P]),
    "gs_ssim_forward": (I, [I, I, I, P, P, I, P, SZ, P, P]),
    "gs_ssim_backward": (I, [I, I, I, P, P, P, P, P, P]),
    "gs_l1_ssim_loss_grad": (I, [I, I, P, P, I, F, P, P, P, SZ, P]),
    "gs_preprocess_backward": (I, [I, P, P, P, P, P, P, P, P, P, I, I, I, I, I, P, P, I, P, I, P,
                                   P, P, P, P, P, P]),
    "gs_preprocess_forward_views": (I, [I, I, P, P, P, P, P, P, P, P, P, F, F, F, F, F, I, I, I,
                                        I, P, P, P, P, P, P, P, P]),
    "gs_preprocess_backward_views_range": (I, [I, I, I, I, P, P, P, P, P, P, P, P, P, I, I, I,
                                                I, I, P, P, I, P, I, P, P, P, P, P, P, P]),
    "gs_preprocess_backward_views": (I, [I, I, P, P, P, P, P, P, P, P, P, I, I, I, I, I, P, P, I,
                                         P, I, P, P, P, P, P, P, P]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """Load lib3dgs_b200.so (building it first when nvcc is available)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            from . import build as _build  # noqa: WPS433

            _build.build()
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"native library missing: {LIB_PATH}")
        handle = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class NativeError(RuntimeError):
    """A nonzero status returned through the C ABI."""

    def __init__(self, fn: str, code: int, cuda_code: int = 0):
        msg = _MESSAGES.get(code, f"status {code}")
        if code == GS_ERR_CUDA:
            msg += f" (cudaError {cuda_code})"
        super().__init__(f"{fn}: {msg}")
        self.code = code


def call(name: str, *args):
    """Call a status-returning entry point; raise NativeError on failure."""
    rc = getattr(lib(), name)(*args)
    if rc != GS_OK:
        raise NativeError(name, rc, lib().gs_last_cuda_error())
    return rc


def query(name: str, *args):
    return getattr(lib(), name)(*args)


def launch_count() -> int:
    return int(lib().gs_launch_count())


def stream_ptr(device=None) -> int:
    import torch

    return int(torch.cuda.current_stream(device).cuda_stream)
