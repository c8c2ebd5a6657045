"""ctypes binding of ``libcubicsplat_b200.so`` (the C ABI in include/cubicsplat_b200.h).

There is no fallback: if the library is missing or a CUDA device is absent the
calls raise.  Tensors are passed as raw device pointers; the current torch CUDA
stream is passed as the launch stream.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libcubicsplat_b200.so")

CS_OK = 0
CS_ERR_ARG = 1
CS_ERR_CAPACITY = 2
CS_ERR_CUDA = 3
CS_ERR_UNSUPPORTED = 4
CS_ERR_TIMEOUT = 5
_ERR_NAMES = {1: "invalid argument", 2: "intersect capacity exceeded", 3: "CUDA launch failed",
              4: "unsupported configuration", 5: "device-side wait timed out"}

_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int32
_F32 = ctypes.c_float
_SZ = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "cs_version": (ctypes.c_char_p, []),
    "cs_project_cubics": (ctypes.c_int, [_P, _P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _I32,
                                         _F32, _I32, _P]),
    "cs_flatten_bernstein": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _P]),
    "cs_primitive_tile_ranges": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I32, _I32, _P]),
    "cs_map_cubic_to_intersects": (ctypes.c_int, [_P, _P, _P, _P, _P, _I64, _I32, _P]),
    "cs_tile_bin_edges": (ctypes.c_int, [_P, _I64, _P, _I64, _P]),
    "cs_isect_edge_ranges": (ctypes.c_int, [_P, _P, _P, _I64, _P]),
    "cs_bin_workspace_size": (_SZ, [_I64]),
    "cs_unit_lists_size": (_SZ, [_I64]),
    "cs_bin_count": (ctypes.c_int, [_P] * 15 + [_I64, _I64, _I64, _I64, _I32, _I32, _I32, _I32,
                                                _I32, _F32, _I32, _P, _I32, _P]),
    "cs_bin_sort": (ctypes.c_int, [_P] * 7 + [_I64, _I64, _I32, _I32, _I32, _I32] + [_P] * 12
                    + [_I64, _P, _P]),
    "cs_stage_workspace_size": (_SZ, [_I64]),
    "cs_tile_stage": (ctypes.c_int, [_P] * 18 + [_I64, _I32, _I32, _P]),
    "cs_raster_workspace_size": (_SZ, [_I64]),
    "cs_de_casteljau_max_depth": (_I32, [_I32]),
    "cs_de_casteljau_edge_capacity": (_I64, [_I64, _I32]),
    "cs_flatten_de_casteljau": (ctypes.c_int, [_P, _P, _I64, _I64, _I32, _F32, _P, _P, _P, _P,
                                               _P, _I64, _P, _P]),
    "cs_edge_grads_to_cubics_csr": (ctypes.c_int, [_P] * 5 + [_I64, _F32, _F32, _P]),
    "cs_cubic_flatness_flags": (ctypes.c_int, [_P, _P, _I64, _F32, _I32, _P]),
    "cs_cubic_split_half": (ctypes.c_int, [_P, _P, _P, _I64, _P]),
    "cs_aa_widths_forward": (ctypes.c_int, [_P, _P, _P, _I64, _P]),
    "cs_aa_widths_backward": (ctypes.c_int, [_P, _P, _P, _P, _I64, _P]),
    "cs_visit_lists_size": (_SZ, [_I64, _I64]),
    "cs_visit_winners_size": (_SZ, [_I64, _I64]),
    "cs_fill_forward": (ctypes.c_int, [_P] * 20 + [_I32, _I32, _I32, _I32, _P]),
    "cs_fill_backward": (ctypes.c_int, [_P] * 25 + [_I32, _I32, _I32, _I32, _P]),
    "cs_stroke_forward": (ctypes.c_int, [_P] * 19 + [_I32, _I32, _I32, _I32, _P]),
    "cs_stroke_backward": (ctypes.c_int, [_P] * 25 + [_I32, _I32, _I32, _I32, _P]),
    "cs_edge_grads_to_cubics": (ctypes.c_int, [_P, _P, _I64, _I32, _F32, _F32, _P]),
    "cs_ring_to_cubics": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _I32, _P]),
    "cs_edge_grads_to_ring": (ctypes.c_int, [_P, _P, _I64, _I32, _I32, _I32, _I32, _I32, _P,
                                             _I32, _I32, _P]),
    "cs_adan_step": (ctypes.c_int, [_P] * 6 + [_I64, _I32] + [_F32] * 10 + [_I32, _P]),
    "cs_regularization_workspace_size": (_SZ, []),
    "cs_ccl_workspace_size": (_SZ, [_I64]),
    "cs_ccl_labels_4": (ctypes.c_int, [_P, _I32, _I32, _P, _P, _P, _P]),
    "cs_ccl_compact_4": (ctypes.c_int, [_P, _I32, _I32, _P, _P, _P, _P, _P]),
    "cs_ccl_stats_4": (ctypes.c_int, [_I32, _I32, _I32, _P, _P, _P, _P]),
    "cs_regularization_forward": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _I64, _I32, _I32,
                                                 _I32, _F32, _I32, _F32, _F32, _F32, _P, _P,
                                                 _P]),
    "cs_regularization_backward": (ctypes.c_int, [_P, _P, _P, _I64, _I64, _I64, _I64, _I32,
                                                  _I32, _I32, _F32, _I32, _F32, _F32, _F32, _P,
                                                  _P, _P, _P, _P]),
    "cs_adam_workspace_size": (_SZ, []),
    "cs_adam_step": (ctypes.c_int, [_P, _P, _P, _P, _I64, _I64, _F32, _F32, _F32, _F32, _F32, _P,
                                    _P, _I32, _P]),
    "cs_ring_segments_forward": (ctypes.c_int, [_P, _P, _P, _P, _P, _I64, _I32, _I32, _P]),
    "cs_ring_segments_backward": (ctypes.c_int, [_P, _P, _P, _P, _P, _I64, _I32, _I32, _P]),
    "cs_mse_workspace_size": (_SZ, [_I64]),
    "cs_mse_forward": (ctypes.c_int, [_P, _P, _I64, _P, _P, _P, _P]),
    "cs_mse_backward": (ctypes.c_int, [_P, _P, _P, _F32, _P, _I64, _P]),
    "cs_ssim_workspace_size": (_SZ, [_I64, _I32, _I32, _I32]),
    "cs_ssim": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _I32, _F32, _F32, _P, _P, _P, _P]),
    "cs_ssim_noalloc": (ctypes.c_int, [_P, _P, _P, _I64, _I32, _I32, _I32, _F32, _F32, _P, _P,
                                       _P]),
    "cs_allreduce_adam_workspace_size": (_SZ, []),
    "cs_peer_signal": (ctypes.c_int, [_P, _I32, _I32, _I32, _P, _I32, _I32, _P]),
    "cs_peer_wait_copy": (ctypes.c_int, [_P, _I32, _I32, _I32, _P, _I32, _I64, _P, _P, _I64, _P,
                                         _I64, _I64, _I32, _P]),
    "cs_allreduce_adam": (ctypes.c_int, [_P, _I32, _P, _P, _P, _I64, _I64, _I32, _P, _P, _F32,
                                         _F32, _F32, _F32, _F32, _P, _P, _I32, _I64, _P, _P,
                                         _P]),
    "cs_stream_is_capturing": (ctypes.c_int, [_P]),
    "cs_poison_on_status": (ctypes.c_int, [_P, _P, _I64, _P]),
}

_lock = threading.Lock()
_lib = None


class NativeError(RuntimeError):
    pass


def library_path() -> str:
    return LIB_PATH


def load():
    """Load the CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise NativeError(
                f"{LIB_PATH} is missing: build it with `python -m repo_b200.build` "
                "(there is no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int, what: str) -> None:
    if status != CS_OK:
        raise NativeError(f"{what} failed: {_ERR_NAMES.get(status, status)} (status {status})")


def ptr(t) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    return t.data_ptr()


def stream(device=None) -> int:
    """The current torch CUDA stream of `device` (default: the current
    device) as a raw cudaStream_t, without building a torch Stream object."""
    if device is None:
        idx = torch.cuda.current_device()
    elif isinstance(device, int):
        idx = device
    else:
        idx = torch.device(device).index
        if idx is None:
            idx = torch.cuda.current_device()
    return torch._C._cuda_getCurrentRawStream(idx)


def call(name: str, *args) -> int:
    return getattr(load(), name)(*args)


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the B200 renderer has no CPU path)")
