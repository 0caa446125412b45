"""ctypes binding of the C ABI declared in include/kf_sm100.h.

There is no fallback: if the shared library is missing or no sm_100 GPU is
present, calls raise. Callers that want the reference answer on failure (the
drop-in `submission.UserOptimizedTransformer`) catch that explicitly and say
so.
"""
from __future__ import annotations

import ctypes
import os
import threading

from .build import LIB_PATH

_c_i64 = ctypes.c_int64
_c_int = ctypes.c_int
_c_float = ctypes.c_float
_c_ptr = ctypes.c_void_p

# name -> (restype, argtypes); must mirror include/kf_sm100.h exactly.
SIGNATURES = {
    "kf_version": (_c_int, []),
    "kf_last_error": (ctypes.c_char_p, []),
    "kf_device_status": (_c_int, [_c_int]),
    "kf_device_status_async": (_c_int, [_c_ptr, _c_ptr]),
    "kf_set_wait_limit": (_c_int, [_c_i64]),
    "kf_ln_add_mask": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_ptr,
                                _c_ptr, _c_i64, _c_ptr, _c_i64, _c_i64, _c_i64, _c_float,
                                _c_int, _c_ptr]),
    "kf_gemm_tf32": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_i64,
                              _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int,
                              _c_ptr, _c_ptr, _c_ptr]),
    "kf_live_row_tiles": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_ptr, _c_ptr]),
    "kf_ln_add_mask_rows": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_ptr,
                                     _c_ptr, _c_i64, _c_ptr, _c_i64, _c_i64, _c_i64, _c_float,
                                     _c_int, _c_ptr, _c_ptr]),
    "kf_pack_rows": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_ptr]),
    "kf_gemm_bf16x3": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_i64,
                                _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int, _c_int,
                                _c_ptr, _c_ptr, _c_ptr]),
    "kf_gemm_bf16x3_sk": (_c_int, [_c_ptr, _c_i64, _c_ptr, _c_i64, _c_ptr, _c_ptr, _c_i64,
                                   _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_int, _c_int,
                                   _c_int, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_ptr]),
    "kf_gemm_sk_workspace_bytes": (_c_i64, [_c_i64, _c_i64, _c_int]),
    "kf_split_bf16x2": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_i64, _c_ptr]),
    "kf_keep_bits_words": (ctypes.c_size_t, [_c_i64, _c_i64]),
    "kf_keep_bits": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_ptr]),
    "kf_flash_fwd_tf32": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_i64,
                                   _c_ptr, _c_i64, _c_i64, _c_i64,
                                   _c_ptr, _c_i64, _c_i64, _c_i64,
                                   _c_ptr, _c_i64, _c_i64, _c_i64,
                                   _c_ptr, _c_i64, _c_i64, _c_i64, _c_int, _c_int, _c_float,
                                   _c_int, _c_ptr]),
    "kf_batch_order": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr]),
    "kf_flash_fwd_tf32_ordered": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_i64,
                                           _c_ptr, _c_i64, _c_i64, _c_i64,
                                           _c_ptr, _c_i64, _c_i64, _c_i64,
                                           _c_ptr, _c_i64, _c_i64, _c_i64,
                                           _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_int,
                                           _c_int, _c_float, _c_int, _c_ptr]),
    "kf_round_tf32": (_c_int, [_c_ptr, _c_ptr, _c_i64, _c_ptr]),
    "kf_attn_schedule_words": (ctypes.c_size_t, [_c_i64, _c_i64, _c_i64]),
    "kf_attn_schedule": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_i64, _c_ptr, _c_ptr]),
    "kf_flash_fwd_tf32_sched": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_i64,
                                         _c_ptr, _c_i64, _c_i64, _c_i64,
                                         _c_ptr, _c_i64, _c_i64, _c_i64,
                                         _c_ptr, _c_i64, _c_i64, _c_i64,
                                         _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i64, _c_int,
                                         _c_int, _c_float, _c_int, _c_ptr]),
    "kf_flash_fwd_tf32_keep_noalloc": (_c_int, [_c_ptr, _c_i64, _c_i64, _c_i64,
                                                _c_ptr, _c_i64, _c_i64, _c_i64,
                                                _c_ptr, _c_i64, _c_i64, _c_i64,
                                                _c_ptr, _c_i64, _c_i64, _c_i64,
                                                _c_ptr, _c_i64, _c_i64, _c_i64, _c_i64,
                                                _c_int, _c_int, _c_float, _c_int, _c_ptr]),
}

# C-ABI constants (include/kf_sm100.h)
KF_OK = 0
KF_E_INVALID = 1
KF_E_UNSUPPORTED = 2
KF_E_CUDA = 3
KF_E_NO_DEVICE = 4
KF_LN_MASK_OUT = 1
KF_LN_ROUND_TF32 = 2
KF_LN_SKIP_PADDED = 4
KF_LN_OUT_BF16X2 = 8
KF_LN_STATIC_PARAMS = 16
KF_LN_Y_MAPPED = 32
KF_LN_H_MAPPED = 64
KF_EPI_BIAS = 0
KF_EPI_BIAS_GELU = 1
KF_GEMM_ROUND_TF32 = 1
KF_GEMM_SPLIT3 = 2
KF_GEMM_BF16X3 = 4

GEMM_PRECISION_FLAGS = {"tf32": 0, "3xtf32": KF_GEMM_SPLIT3, "bf16x3": KF_GEMM_BF16X3}
KF_ATTN_CAUSAL = 1
KF_ATTN_SKIP_EMPTY_Q = 2
KF_ATTN_ROUND_TF32 = 4
KF_ATTN_OUT_BF16X2 = 8
KF_ATTN_EMPTY_Q_UNTOUCHED = 16
KF_GEMM_OUT_BF16X2 = 8
KF_GEMM_PAIR = 32
KF_GEMM_W_STATIC = 64
KF_NOALLOC_KEEP_WORDS_MAX = 262144

_lib = None
_lock = threading.Lock()


class KernelError(RuntimeError):
    """A C-ABI call returned a non-zero status."""


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Load the library and bind every declared symbol (no GPU needed)."""
    global _lib
    with _lock:
        if _lib is not None and path == LIB_PATH:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} is missing: build it with `python -m techjam2026_b200.build` "
                "(or __graft_entry__.build())")
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if path == LIB_PATH:
            _lib = lib
        return lib


def lib() -> ctypes.CDLL:
    return _lib if _lib is not None else load()


def check(rc: int, what: str) -> None:
    if rc != KF_OK:
        msg = lib().kf_last_error().decode(errors="replace")
        raise KernelError(f"{what} failed with status {rc}: {msg}")


def stream_ptr(stream=None) -> int:
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)
