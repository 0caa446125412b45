"""The C-ABI library: it builds for sm_100a, loads without a GPU, exports
every symbol include/kf_sm100.h declares, and rejects bad arguments before
touching the device. No kernel is launched here. CPU only."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from techjam2026_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "kf_sm100.h")


def declared_symbols():
    src = open(HEADER, encoding="utf-8").read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(kf_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(build.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(raw, name), name


def test_library_has_no_libcuda_link_dependency():
    import subprocess
    out = subprocess.run(["ldd", build.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out


def test_version_and_workspace_size(lib):
    assert lib.kf_version() == 100
    assert lib.kf_keep_bits_words(2, 33) == 4
    assert lib.kf_keep_bits_words(0, 33) == 0


def test_invalid_arguments_are_rejected_without_a_device(lib):
    assert lib.kf_gemm_tf32(None, 4, None, 4, None, None, 4, 4, 4, 4, 0, 0, 0, 0, 0, None, None, None) == \
        _lib.KF_E_INVALID
    assert b"invalid" in lib.kf_last_error()
    assert lib.kf_ln_add_mask(None, 8, None, 0, None, None, None, None, 0, None, 8, 4, 8, 1e-5,
                              0, None) == _lib.KF_E_INVALID
    assert lib.kf_keep_bits(None, 8, 1, 8, None, None) == _lib.KF_E_INVALID
    assert lib.kf_flash_fwd_tf32(None, 1, 1, 1, None, 1, 1, 1, None, 1, 1, 1, None, 1, 1, 1,
                                 None, 1, 1, 1, 64, 64, 0.125, 0, None) == _lib.KF_E_INVALID
    assert lib.kf_round_tf32(None, None, 4, None) == _lib.KF_E_INVALID
    assert lib.kf_batch_order(None, 4, 64, None, None) == _lib.KF_E_INVALID
    fake = ctypes.c_void_p(0x1000)   # never dereferenced: rejected before any launch
    assert lib.kf_batch_order(fake, 0, 64, fake, None) == _lib.KF_E_INVALID
    assert lib.kf_flash_fwd_tf32_ordered(fake, 64, 64, 64, fake, 64, 64, 64, fake, 64, 64, 64,
                                         fake, 64, 64, 64, fake, None, 1, 1, 8, 64, 64, 0.125,
                                         0, None) == _lib.KF_E_INVALID
    assert b"batch_order is null" in lib.kf_last_error()


def test_unsupported_shapes_are_reported(lib):
    fake = ctypes.c_void_p(0x1000)   # never dereferenced: rejected by the shape checks
    rc = lib.kf_gemm_tf32(fake, 6, fake, 6, None, fake, 8, 8, 8, 6, 0, 0, 0, 0, 0, None, None, None)
    assert rc == _lib.KF_E_UNSUPPORTED and b"K % 4" in lib.kf_last_error()
    rc = lib.kf_flash_fwd_tf32(fake, 64, 64, 64, fake, 64, 64, 64, fake, 64, 64, 64,
                               fake, 64, 64, 64, None, 1, 1, 8, 48, 48, 0.1, 0, None)
    assert rc == _lib.KF_E_UNSUPPORTED
    rc = lib.kf_gemm_tf32(fake, 8, fake, 8, None, fake, 8, 8, 8, 8, 7, 0, 0, 0, 0, None, None, None)
    assert rc == _lib.KF_E_INVALID


def test_empty_problems_are_no_ops(lib):
    fake = ctypes.c_void_p(0x1000)
    assert lib.kf_gemm_tf32(fake, 8, fake, 8, None, fake, 8, 0, 8, 8, 0, 0, 0, 0, 0, None, None, None) == 0
    assert lib.kf_ln_add_mask(fake, 8, None, 0, None, fake, fake, None, 0, fake, 8, 0, 8, 1e-5,
                              0, None) == 0


def test_bf16x3_gemm_rejects_unknown_flags_before_any_launch():
    """kf_gemm_bf16x3 and its stream-K form refuse flag bits they do not know
    (bit 16 is no longer a GEMM flag) with an error code and no CUDA call,
    instead of silently ignoring them."""
    lib = _lib.lib()
    fake = ctypes.c_void_p(0x1000)
    for bits in (16, 128, 1 << 12):
        assert lib.kf_gemm_bf16x3(fake, 64, fake, 64, None, fake, 64, 128, 64, 64, 0, bits, 0, 0,
                                  0, None, None, None) == _lib.KF_E_INVALID
        assert b"unknown flags" in lib.kf_last_error()
        assert lib.kf_gemm_bf16x3_sk(fake, 64, fake, 64, None, fake, 64, 128, 64, 64, 0, bits,
                                     64, 0, 0, None, None, fake, 1 << 20,
                                     None) == _lib.KF_E_INVALID


def test_packed_row_entries_reject_bad_arguments_before_any_launch():
    """kf_pack_rows and kf_ln_add_mask_rows check their arguments on the
    host: null buffers, B outside [1, 65535], a missing row map or no map
    flag are refused with KF_E_INVALID and no CUDA call; kf_ln_add_mask
    refuses the map flags (they need the map)."""
    lib = _lib.lib()
    fake = ctypes.c_void_p(0x1000)
    assert lib.kf_pack_rows(None, 2, 8, fake, fake, fake, fake, None) == _lib.KF_E_INVALID
    assert lib.kf_pack_rows(fake, 0, 8, fake, fake, fake, fake, None) == _lib.KF_E_INVALID
    assert lib.kf_pack_rows(fake, 65536, 8, fake, fake, fake, fake, None) == _lib.KF_E_INVALID
    assert lib.kf_pack_rows(fake, 2, 8, fake, None, fake, fake, None) == _lib.KF_E_INVALID
    ln = lambda fn, flags, rmap: fn(fake, 8, fake, 8, None, fake, fake, None, 0, fake, 8, 4, 8,
                                    1e-5, flags, *(() if rmap is False else (rmap,)), None)
    assert ln(lib.kf_ln_add_mask_rows, _lib.KF_LN_Y_MAPPED, None) == _lib.KF_E_INVALID
    assert ln(lib.kf_ln_add_mask_rows, 0, fake) == _lib.KF_E_INVALID
    assert b"row_map" in lib.kf_last_error()
    assert ln(lib.kf_ln_add_mask, _lib.KF_LN_H_MAPPED, False) == _lib.KF_E_INVALID


def test_noalloc_entry_rejects_bad_attention_arguments_before_any_launch():
    """kf_flash_fwd_tf32_keep_noalloc runs every check of the attention call
    before it queues the key-bit packer: an unsupported head_dim, an odd
    stride or a short keep row stride is refused with no CUDA call at all
    (this runs without a GPU, so any launch or device query would fail with
    a CUDA error code instead)."""
    lib = _lib.lib()
    fake = ctypes.c_void_p(0x1000)   # never dereferenced

    def call(dh=64, q_sm=64, ld_keep=8, S=8):
        return lib.kf_flash_fwd_tf32_keep_noalloc(
            fake, 4096, 512, q_sm, fake, 4096, 512, 64, fake, 4096, 512, 64,
            fake, 4096, 512, 64, fake, ld_keep, 1, 1, S, dh, dh, 0.125, 0, None)

    assert call(dh=48) == _lib.KF_E_UNSUPPORTED
    assert b"head_dim" in lib.kf_last_error()
    assert call(q_sm=6) == _lib.KF_E_UNSUPPORTED
    assert b"strides" in lib.kf_last_error()
    assert call(ld_keep=4) == _lib.KF_E_INVALID
    assert b"ld_keep" in lib.kf_last_error()


def test_persistent_attention_entries_reject_before_any_launch():
    lib = _lib.lib()
    fake = ctypes.c_void_p(0x1000)   # never dereferenced
    assert lib.kf_attn_schedule_words(2, 3, 129) == 8 + 2 * 2 * 3 * 2
    assert lib.kf_attn_schedule_words(0, 3, 129) == 0
    assert lib.kf_attn_schedule(None, 2, 3, 100, None, None) == _lib.KF_E_INVALID
    assert lib.kf_attn_schedule(None, 20000, 1, 100, fake, None) == _lib.KF_E_UNSUPPORTED
    assert lib.kf_attn_schedule(None, 2, 1, 100, ctypes.c_void_p(0x1004), None) == \
        _lib.KF_E_INVALID
    assert lib.kf_attn_schedule(None, 1000, 100, 100, fake, None) == _lib.KF_E_UNSUPPORTED
    args = (fake, 4096, 512, 64, fake, 4096, 512, 64, fake, 4096, 512, 64, fake, 4096, 512, 64,
            None)
    assert lib.kf_flash_fwd_tf32_sched(*args, None, 1, 1, 8, 64, 64, 0.125, 0, None) == \
        _lib.KF_E_INVALID
    assert b"sched is null" in lib.kf_last_error()
    assert lib.kf_flash_fwd_tf32_sched(*args, fake, 1, 1, 8, 48, 48, 0.125, 0, None) == \
        _lib.KF_E_UNSUPPORTED


def test_status_entries_reject_a_null_destination():
    lib = _lib.lib()
    assert lib.kf_device_status_async(None, None) == _lib.KF_E_INVALID
    assert b"null" in lib.kf_last_error()
