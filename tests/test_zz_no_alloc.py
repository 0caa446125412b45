"""kf_flash_fwd_tf32_keep_noalloc: the attention forward for callers that
cannot allocate device memory (a serving process whose GPU memory is all in a
fixed arena, a latency-bound path that cannot take cudaMalloc's device-wide
synchronisation, an FFI caller with no device allocator). It packs the key
bits into the library's static device scratch instead of a caller workspace.

Checked through the C ABI against the existing entry points
(kf_keep_bits + kf_flash_fwd_tf32 with a caller-allocated workspace) on two
calls in a row with different shapes and masks, so stale scratch from the
first call would show in the second. This file sorts last so a run that stops
at the first failure has run every other test before it; it needs no state
from them.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from techjam2026_b200 import _lib
from techjam2026_b200.numerics import check

pytestmark = pytest.mark.gpu


def _strides(t):
    return t.stride(0), t.stride(1), t.stride(2)


def _existing(q, k, v, keep, causal):
    L = _lib.lib()
    B, H, S, Dh = q.shape
    o = torch.empty_like(q)
    bits = torch.empty(int(L.kf_keep_bits_words(B, S)), dtype=torch.int32, device=q.device)
    st = _lib.stream_ptr()
    _lib.check(L.kf_keep_bits(keep.data_ptr(), keep.stride(0), B, S, bits.data_ptr(), st),
               "kf_keep_bits")
    _lib.check(L.kf_flash_fwd_tf32(q.data_ptr(), *_strides(q), k.data_ptr(), *_strides(k),
                                   v.data_ptr(), *_strides(v), o.data_ptr(), *_strides(o),
                                   bits.data_ptr(), B, H, S, Dh, Dh, Dh ** -0.5,
                                   1 if causal else 0, st), "kf_flash_fwd_tf32")
    return o


def _noalloc(q, k, v, keep, causal):
    L = _lib.lib()
    B, H, S, Dh = q.shape
    o = torch.empty_like(q)
    rc = L.kf_flash_fwd_tf32_keep_noalloc(
        q.data_ptr(), *_strides(q), k.data_ptr(), *_strides(k), v.data_ptr(), *_strides(v),
        o.data_ptr(), *_strides(o), keep.data_ptr(), keep.stride(0), B, H, S, Dh, Dh,
        Dh ** -0.5, 1 if causal else 0, _lib.stream_ptr())
    _lib.check(rc, "kf_flash_fwd_tf32_keep_noalloc")
    return o


def test_noalloc_matches_the_existing_entry_point_on_two_calls_in_a_row():
    cases = [(0, 4, 8, 700, 64, True), (1, 3, 4, 333, 32, False)]
    for seed, B, H, S, Dh, causal in cases:
        g = torch.Generator(device="cpu").manual_seed(seed)
        q, k, v = (torch.randn(B, H, S, Dh, generator=g).cuda() for _ in range(3))
        lens = torch.randint(1, S + 1, (B,), generator=g)
        keep = (torch.arange(S)[None, :] < lens[:, None]).to(torch.uint8).cuda()
        got = _noalloc(q, k, v, keep, causal)
        want = _existing(q, k, v, keep, causal)
        torch.cuda.synchronize()
        res = check(want, got)
        assert res.passed, str(res)
        assert (got - want).abs().max().item() < 5e-3
        assert torch.equal(got, want), "same kernels, same inputs: identical output expected"
    assert _lib.lib().kf_device_status(0) == 0


def test_noalloc_rejects_sizes_beyond_its_static_scratch():
    L = _lib.lib()
    q = torch.zeros(1, 1, 32, 64, device="cuda")
    keep = torch.ones(1, 32, dtype=torch.uint8, device="cuda")
    B, S = 2, 32 * _lib.KF_NOALLOC_KEEP_WORDS_MAX   # twice the capacity
    rc = L.kf_flash_fwd_tf32_keep_noalloc(
        q.data_ptr(), 2048, 2048, 64, q.data_ptr(), 2048, 2048, 64, q.data_ptr(), 2048, 2048, 64,
        q.data_ptr(), 2048, 2048, 64, keep.data_ptr(), S, B, 1, S, 64, 64, 0.125, 0,
        _lib.stream_ptr())
    assert rc == _lib.KF_E_UNSUPPORTED
    assert b"static scratch" in L.kf_last_error()
