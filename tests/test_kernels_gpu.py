"""The CUDA kernels through the C ABI against exact torch references.

Traps targeted, as the reference's own kernel tests do
(kernelforge tests/test_kernels.py): all-zero rows and mask ordering around
the norm, row counts and sequence lengths that are not tile multiples, causal
crossed with padding, fully masked softmax rows, strided QKV views, head_dim
8 (zero-padded) through 256.

Operands are pre-rounded to TF32 so the GEMM can be checked against a float64
product to fp32-accumulation accuracy: any descriptor, swizzle or tiling error
shows up as an O(1) difference, not as noise inside a loose tolerance.
"""
from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from conftest import tf32_round
from techjam2026_b200.numerics import check
from techjam2026_b200.ops import add_mask_layernorm, flash_attention, linear

pytestmark = pytest.mark.gpu


# --------------------------------------------------------------- layernorm

@pytest.mark.parametrize("d", [128, 256, 512, 768, 1024, 100])
@pytest.mark.parametrize("mask_out", [False, True])
def test_fused_add_mask_layernorm(d, mask_out):
    torch.manual_seed(0)
    M = 517
    x = torch.randn(M, d, device="cuda")
    y = torch.randn(M, d, device="cuda")
    keep = (torch.rand(M, device="cuda") > 0.3).float()
    w = torch.randn(d, device="cuda")
    b = torch.randn(d, device="cuda")
    s, h = add_mask_layernorm(x, y, keep, w, b, 1e-5, mask_out=mask_out)
    ref_s = (x + y) * keep[:, None]                     # fp32 add: bit-exact target
    ref_h = F.layer_norm(ref_s.double(), (d,), w.double(), b.double(), 1e-5)
    if mask_out:
        ref_h = ref_h * keep[:, None].double()
    assert torch.equal(s, ref_s)
    assert (h.double() - ref_h).abs().max().item() < 2e-5
    # padded rows: residual exactly 0; h exactly 0 under mask_out
    dead = keep == 0
    assert torch.count_nonzero(s[dead]) == 0
    if mask_out:
        assert torch.count_nonzero(h[dead]) == 0


def test_layernorm_of_an_all_zero_row_returns_bias():
    d = 256
    x = torch.zeros(8, d, device="cuda")
    w = torch.randn(d, device="cuda")
    b = torch.randn(d, device="cuda")
    _, h = add_mask_layernorm(x, None, None, w, b, 1e-5, mask_out=False)
    assert torch.equal(h, b.expand_as(h))
    keep = torch.zeros(8, device="cuda")
    _, h_masked = add_mask_layernorm(x, None, keep, w, b, 1e-5, mask_out=True)
    assert torch.count_nonzero(h_masked) == 0


def test_layernorm_mask_is_a_select_not_a_multiply():
    """A padded row holding NaN/Inf still comes out exactly 0 (masked_fill)."""
    d = 128
    x = torch.randn(4, d, device="cuda")
    x[1] = float("nan")
    x[2] = float("inf")
    keep = torch.tensor([1, 0, 0, 1], device="cuda", dtype=torch.bool)
    w, b = torch.ones(d, device="cuda"), torch.zeros(d, device="cuda")
    s, h = add_mask_layernorm(x, None, keep, w, b, mask_out=True)
    assert torch.count_nonzero(s[1:3]) == 0 and torch.count_nonzero(h[1:3]) == 0
    assert torch.isfinite(h).all()


@pytest.mark.parametrize("d", [128, 512, 1024, 4096])
@pytest.mark.parametrize("skip", [False, True])
def test_layernorm_static_params_identical(d, skip):
    """KF_LN_STATIC_PARAMS loads keep, gamma and beta before the wait on the
    previous kernel (and lets skipped padded rows leave early): same bits."""
    from techjam2026_b200 import _lib
    L = _lib.lib()
    torch.manual_seed(d)
    M = 517
    x, y = torch.randn(M, d, device="cuda"), torch.randn(M, d, device="cuda")
    keep = (torch.rand(M, device="cuda") > 0.3).to(torch.uint8)
    w, b = torch.randn(d, device="cuda"), torch.randn(d, device="cuda")
    torch.cuda.synchronize()
    outs = []
    for static in (False, True):
        s = torch.full((M, d), 5.0, device="cuda")
        h = torch.full((M, d), 7.0, device="cuda")
        flags = (_lib.KF_LN_SKIP_PADDED if skip else 0) | (_lib.KF_LN_STATIC_PARAMS if static else 0)
        _lib.check(L.kf_ln_add_mask(x.data_ptr(), d, y.data_ptr(), d, keep.data_ptr(),
                                    w.data_ptr(), b.data_ptr(), s.data_ptr(), d, h.data_ptr(), d,
                                    M, d, 1e-5, flags, _lib.stream_ptr()), "kf_ln_add_mask")
        outs.append((s, h))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])
    if skip:
        dead = keep == 0
        assert torch.all(outs[1][0][dead] == 5.0) and torch.all(outs[1][1][dead] == 7.0)


def test_layernorm_in_place_residual():
    """The stack updates its residual stream in place (x is s_out)."""
    from techjam2026_b200 import _lib
    torch.manual_seed(1)
    M, d = 300, 512
    x = torch.randn(M, d, device="cuda")
    y = torch.randn(M, d, device="cuda")
    w, b = torch.randn(d, device="cuda"), torch.randn(d, device="cuda")
    ref_s = x + y
    ref_h = F.layer_norm(ref_s, (d,), w, b, 1e-5)
    h = torch.empty_like(x)
    rc = _lib.lib().kf_ln_add_mask(x.data_ptr(), d, y.data_ptr(), d, None, w.data_ptr(),
                                   b.data_ptr(), x.data_ptr(), d, h.data_ptr(), d, M, d, 1e-5,
                                   0, _lib.stream_ptr())
    _lib.check(rc, "kf_ln_add_mask")
    assert torch.equal(x, ref_s)
    assert (h - ref_h).abs().max().item() < 2e-5


# --------------------------------------------------------------- GEMM

@pytest.mark.parametrize("M,N,K", [(128, 64, 32), (517, 384, 512), (4096, 1536, 512),
                                   (300, 200, 132), (1, 2304, 768), (2048, 512, 2048)])
@pytest.mark.parametrize("bn", [0, 64, 128, 256])
def test_gemm_exact_on_tf32_operands(M, N, K, bn):
    torch.manual_seed(M + N + K)
    a = tf32_round(torch.randn(M, K, device="cuda"))
    w = tf32_round(torch.randn(N, K, device="cuda") / math.sqrt(K))
    bias = torch.randn(N, device="cuda")
    out = linear(a, w, bias, bn=bn, precision="tf32")
    ref = a.double() @ w.double().t() + bias.double()
    err = (out.double() - ref).abs().max().item()
    assert err < 1e-4, f"max abs err {err}"


@pytest.mark.parametrize("M,N,K", [(128, 64, 32), (517, 384, 512), (4096, 1536, 512),
                                   (300, 200, 132), (2048, 512, 2048)])
@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("gelu", [False, True])
@pytest.mark.parametrize("precision", ["3xtf32", "bf16x3"])
def test_gemm_split_modes_accuracy(M, N, K, bn, gelu, precision):
    """Compensated modes on unrounded operands: near-fp32 error."""
    torch.manual_seed(M + 7 * N + K)
    a = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / math.sqrt(K)
    bias = torch.randn(N, device="cuda")
    out = linear(a, w, bias, gelu=gelu, bn=bn, precision=precision)
    ref = a.double() @ w.double().t() + bias.double()
    if gelu:
        ref = F.gelu(ref, approximate="none")
    err = (out.double() - ref).abs().max().item()
    # 3xtf32 ~2^-20 and bf16x3 ~2^-17 per product, plus fp32 accumulation
    # inside the tensor core over K terms of O(1/sqrt(K)).
    assert err < (2e-4 if precision == "3xtf32" else 5e-4), f"max abs err {err}"


def test_gemm_plain_tf32_is_tf32_level():
    torch.manual_seed(9)
    a = torch.randn(1000, 768, device="cuda")
    w = torch.randn(768, 768, device="cuda") / math.sqrt(768)
    one = linear(a, w, None, precision="tf32")
    three = linear(a, w, None, precision="3xtf32")
    bf3 = linear(a, w, None, precision="bf16x3")
    ref = a.double() @ w.double().t()
    e1 = (one.double() - ref).abs().max().item()
    e3 = (three.double() - ref).abs().max().item()
    eb = (bf3.double() - ref).abs().max().item()
    assert 1e-4 < e1 < 1e-2 and e3 < 1e-4 and e3 < e1 / 20 and eb < e1 / 8


@pytest.mark.parametrize("M,N,K", [(517, 2048, 512), (128, 512, 128)])
def test_gemm_gelu_epilogue(M, N, K):
    torch.manual_seed(3)
    a = tf32_round(torch.randn(M, K, device="cuda"))
    w = tf32_round(torch.randn(N, K, device="cuda") / math.sqrt(K))
    bias = torch.randn(N, device="cuda")
    out = linear(a, w, bias, gelu=True)
    ref = F.gelu(a.double() @ w.double().t() + bias.double(), approximate="none")
    assert (out.double() - ref).abs().max().item() < 1e-4


def test_gemm_unrounded_operands_within_tf32_error():
    torch.manual_seed(4)
    M, N, K = 1000, 768, 768
    a = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / math.sqrt(K)
    out = linear(a, w, None, precision="tf32")
    ref = a.double() @ w.double().t()
    # TF32 keeps 10 explicit mantissa bits: |err| ~ 2^-11 * sqrt(K) * |a||w|
    assert (out.double() - ref).abs().max().item() < 1e-2


def test_gemm_head_padded_output():
    """head_dim 8 columns land in 16-wide slots; pad columns stay untouched."""
    from techjam2026_b200 import _lib
    torch.manual_seed(5)
    M, N, K = 256, 3 * 128, 128        # 3 x (16 heads x 8)
    a = tf32_round(torch.randn(M, K, device="cuda"))
    w = tf32_round(torch.randn(N, K, device="cuda") / math.sqrt(K))
    out = torch.full((M, 3 * 16 * 16), 7.0, device="cuda")
    rc = _lib.lib().kf_gemm_tf32(a.data_ptr(), K, w.data_ptr(), K, None, out.data_ptr(),
                                 out.stride(0), M, N, K, 0, 0, 0, 8, 16, None, None, _lib.stream_ptr())
    _lib.check(rc, "kf_gemm_tf32")
    ref = (a.double() @ w.double().t()).view(M, 48, 8)
    got = out.view(M, 48, 16)
    assert (got[..., :8].double() - ref).abs().max().item() < 1e-4
    assert torch.all(got[..., 8:] == 7.0)


# --------------------------------------------------------------- attention

def reference_attention(q, k, v, keep, causal, scale=None):
    """float64 transcription of BaselineSelfAttention's core (softmax(QK^T)V)."""
    scale = q.shape[-1] ** -0.5 if scale is None else scale
    scores = torch.matmul(q.double(), k.double().transpose(-2, -1)) * scale
    S = q.shape[2]
    if causal:
        cm = torch.ones((S, S), device=q.device, dtype=torch.bool).triu(1)
        scores = scores.masked_fill(cm, float("-inf"))
    if keep is not None:
        scores = scores.masked_fill(~keep.bool()[:, None, None, :], float("-inf"))
    p = torch.softmax(scores, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)     # fully masked rows -> 0 (kernel contract)
    return torch.matmul(p, v.double())


@pytest.mark.parametrize("shape", [
    (2, 8, 128, 64), (1, 4, 1, 64), (2, 8, 333, 64), (1, 8, 2048, 64),
    (1, 4, 100, 128), (2, 4, 64, 32), (2, 4, 200, 16), (1, 2, 300, 256), (2, 16, 257, 8),
    (1, 4, 1023, 64), (2, 2, 777, 32),
])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("pad", [0.0, 0.4])
def test_flash_attention_matches_reference(shape, causal, pad):
    torch.manual_seed(0)
    B, H, S, Dh = shape
    q, k, v = (torch.randn(B, H, S, Dh, device="cuda") for _ in range(3))
    keep = None
    if pad > 0:
        lens = torch.randint(1, S + 1, (B,), device="cuda")
        keep = (torch.arange(S, device="cuda")[None, :] < lens[:, None]).to(torch.uint8)
    out = flash_attention(q, k, v, keep=keep, causal=causal)
    ref = reference_attention(q, k, v, keep, causal)
    res = check(ref.float(), out)
    assert res.passed, str(res)
    assert (out.double() - ref).abs().max().item() < 5e-3


def test_flash_fully_masked_row_yields_zero_not_nan():
    torch.manual_seed(1)
    B, H, S, Dh = 1, 2, 64, 32
    q, k, v = (torch.randn(B, H, S, Dh, device="cuda") for _ in range(3))
    keep = torch.zeros(B, S, dtype=torch.uint8, device="cuda")
    keep[0, 40:] = 1      # rows < 40 see no valid key under the causal mask
    out = flash_attention(q, k, v, keep=keep, causal=True)
    assert torch.isfinite(out).all()
    assert torch.count_nonzero(out[:, :, :40]) == 0


def test_flash_random_non_prefix_mask():
    torch.manual_seed(2)
    B, H, S, Dh = 2, 4, 400, 64
    q, k, v = (torch.randn(B, H, S, Dh, device="cuda") for _ in range(3))
    keep = (torch.rand(B, S, device="cuda") > 0.5).to(torch.uint8)
    keep[:, 0] = 1
    keep[0, 128:256] = 0           # one fully masked KV tile in the middle
    for causal in (False, True):
        out = flash_attention(q, k, v, keep=keep, causal=causal)
        ref = reference_attention(q, k, v, keep, causal)
        assert (out.double() - ref).abs().max().item() < 5e-3


def test_flash_on_strided_qkv_views():
    """Q/K/V as views of one fused [B, S, 3, H, Dh] buffer, output into [B, S, H, Dh]."""
    torch.manual_seed(3)
    B, S, H, Dh = 2, 300, 8, 64
    qkv = torch.randn(B, S, 3, H, Dh, device="cuda")
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    ctx = torch.empty(B, S, H, Dh, device="cuda")
    flash_attention(q, k, v, causal=True, out=ctx.permute(0, 2, 1, 3))
    ref = reference_attention(q.contiguous(), k.contiguous(), v.contiguous(), None, True)
    assert (ctx.permute(0, 2, 1, 3).double() - ref).abs().max().item() < 5e-3


def test_flash_long_sequence_causal_padded():
    torch.manual_seed(4)
    B, H, S, Dh = 1, 2, 4096, 64
    q, k, v = (torch.randn(B, H, S, Dh, device="cuda") for _ in range(3))
    keep = (torch.arange(S, device="cuda")[None, :] < 3000).to(torch.uint8)
    out = flash_attention(q, k, v, keep=keep, causal=True)
    ref = reference_attention(q, k, v, keep, True)
    assert (out.double() - ref).abs().max().item() < 5e-3


def test_device_status_clean_after_kernels():
    from techjam2026_b200 import _lib
    assert _lib.lib().kf_device_status(0) == 0


# --------------------------------------------------------------- padded-row skipping

def _live_tiles(keep_u8):
    from techjam2026_b200 import _lib
    M = keep_u8.numel()
    tiles = torch.full(((M + 127) // 128,), -1, dtype=torch.int32, device="cuda")
    count = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.check(_lib.lib().kf_live_row_tiles(keep_u8.data_ptr(), M, tiles.data_ptr(),
                                            count.data_ptr(), _lib.stream_ptr()),
               "kf_live_row_tiles")
    return tiles, count


@pytest.mark.parametrize("M", [1, 127, 128, 4096, 131072 + 77])
def test_live_row_tiles_lists_exactly_the_tiles_with_a_real_row(M):
    g = torch.Generator().manual_seed(M)
    keep = (torch.rand(M, generator=g) < 0.002).to(torch.uint8)
    keep[: min(M, 5)] = 1 if M > 300 else keep[: min(M, 5)]
    tiles, count = _live_tiles(keep.cuda())
    want = [t for t in range((M + 127) // 128) if bool(keep[t * 128:(t + 1) * 128].any())]
    n = int(count.item())
    assert tiles[:n].tolist() == want


def test_gemm_computes_only_live_row_tiles():
    from techjam2026_b200 import _lib
    torch.manual_seed(6)
    M, N, K = 1000, 384, 256
    a = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / math.sqrt(K)
    keep = torch.zeros(M, dtype=torch.uint8, device="cuda")
    keep[5] = 1          # tile 0
    keep[300:310] = 1    # tile 2
    keep[999] = 1        # tile 7 (ragged last tile)
    tiles, count = _live_tiles(keep)
    out = torch.full((M, N), 7.0, device="cuda")
    rc = _lib.lib().kf_gemm_tf32(a.data_ptr(), K, w.data_ptr(), K, None, out.data_ptr(), N, M,
                                 N, K, 0, _lib.KF_GEMM_SPLIT3, 0, 0, 0, tiles.data_ptr(),
                                 count.data_ptr(), _lib.stream_ptr())
    _lib.check(rc, "kf_gemm_tf32")
    ref = a.double() @ w.double().t()
    for t in range(8):
        rows = slice(t * 128, min(M, (t + 1) * 128))
        if t in (0, 2, 7):
            assert (out[rows].double() - ref[rows]).abs().max().item() < 2e-4
        else:
            assert torch.all(out[rows] == 7.0)


def test_layernorm_skip_padded_leaves_padded_rows_untouched():
    from techjam2026_b200 import _lib
    M, d = 64, 128
    x = torch.randn(M, d, device="cuda")
    keep = (torch.arange(M, device="cuda") % 3 != 0).to(torch.uint8)
    w, b = torch.ones(d, device="cuda"), torch.zeros(d, device="cuda")
    s = torch.full((M, d), 5.0, device="cuda")
    h = torch.full((M, d), 6.0, device="cuda")
    rc = _lib.lib().kf_ln_add_mask(x.data_ptr(), d, None, 0, keep.data_ptr(), w.data_ptr(),
                                   b.data_ptr(), s.data_ptr(), d, h.data_ptr(), d, M, d, 1e-5,
                                   _lib.KF_LN_SKIP_PADDED, _lib.stream_ptr())
    _lib.check(rc, "kf_ln_add_mask")
    dead = keep == 0
    assert torch.all(s[dead] == 5.0) and torch.all(h[dead] == 6.0)
    assert torch.equal(s[~dead], x[~dead])


# --------------------------------------------------------------- pre-split bf16x3

def to_planes(t: torch.Tensor) -> torch.Tensor:
    """fp32 [..] -> int16 [2, ..] bf16 planes: hi = bf16_rn(t), lo = bf16_rn(t - hi)."""
    hi = t.to(torch.bfloat16)
    lo = (t - hi.float()).to(torch.bfloat16)
    return torch.stack([hi.view(torch.int16), lo.view(torch.int16)])


def from_planes(p: torch.Tensor) -> torch.Tensor:
    return p[0].view(torch.bfloat16).float() + p[1].view(torch.bfloat16).float()


@pytest.mark.parametrize("M,N,K", [(128, 64, 64), (517, 384, 512), (4096, 2048, 512),
                                   (300, 200, 136), (2048, 512, 2048)])
@pytest.mark.parametrize("bn", [64, 96, 128, 256])
@pytest.mark.parametrize("gelu", [False, True])
@pytest.mark.parametrize("out_split", [False, True])
def test_gemm_bf16x3_presplit(M, N, K, bn, gelu, out_split):
    from techjam2026_b200 import _lib
    torch.manual_seed(M + N + K + bn)
    a = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / math.sqrt(K)
    bias = torch.randn(N, device="cuda")
    a2, w2 = to_planes(a).contiguous(), to_planes(w).contiguous()
    if out_split:
        c = torch.zeros(2, M, N, dtype=torch.int16, device="cuda")
    else:
        c = torch.zeros(M, N, device="cuda")
    flags = _lib.KF_GEMM_OUT_BF16X2 if out_split else 0
    rc = _lib.lib().kf_gemm_bf16x3(a2.data_ptr(), K, w2.data_ptr(), K, bias.data_ptr(),
                                   c.data_ptr(), N, M, N, K, 1 if gelu else 0, flags, bn, 0, 0,
                                   None, None, _lib.stream_ptr())
    _lib.check(rc, "kf_gemm_bf16x3")
    got = from_planes(c) if out_split else c
    ref = a.double() @ w.double().t() + bias.double()
    if gelu:
        ref = F.gelu(ref, approximate="none")
    err = (got.double() - ref).abs().max().item()
    assert err < 6e-4, f"max abs err {err}"


@pytest.mark.parametrize("M,N,K", [(128, 64, 64), (517, 384, 512), (300, 200, 136),
                                   (256, 256, 24), (2048, 512, 2048), (1000, 1024, 1000)])
@pytest.mark.parametrize("bn", [64, 96, 128, 256])
@pytest.mark.parametrize("gelu,out_split", [(False, False), (True, True)])
def test_gemm_bf16x3_tiles_and_ragged_k(M, N, K, bn, gelu, out_split):
    """Every N tile, a ragged last k block (K % 64 != 0) and K below one
    block: fp32-class accuracy against fp64, in fp32 and in bf16-plane
    output."""
    from techjam2026_b200 import _lib
    torch.manual_seed(M * 7 + N + K + bn)
    a = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / math.sqrt(K)
    bias = torch.randn(N, device="cuda")
    a2, w2 = to_planes(a).contiguous(), to_planes(w).contiguous()
    shape = (2, M, N) if out_split else (M, N)
    c = torch.full(shape, 3, dtype=torch.int16 if out_split else torch.float32, device="cuda")
    flags = _lib.KF_GEMM_OUT_BF16X2 if out_split else 0
    rc = _lib.lib().kf_gemm_bf16x3(a2.data_ptr(), K, w2.data_ptr(), K, bias.data_ptr(),
                                   c.data_ptr(), N, M, N, K, 1 if gelu else 0, flags, bn, 0,
                                   0, None, None, _lib.stream_ptr())
    _lib.check(rc, "kf_gemm_bf16x3")
    got = from_planes(c) if out_split else c
    ref = a.double() @ w.double().t() + bias.double()
    if gelu:
        ref = F.gelu(ref, approximate="none")
    assert (got.double() - ref).abs().max().item() < 6e-4


@pytest.mark.parametrize("M,N,K", [(256, 256, 64), (517, 384, 512), (300, 200, 136),
                                   (1000, 1024, 1000), (4096, 2048, 512), (2048, 512, 2048)])
@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("gelu,out_split", [(False, False), (True, True)])
@pytest.mark.parametrize("live", [False, True])
def test_gemm_bf16x3_pair_bit_identical(M, N, K, bn, gelu, out_split, live):
    """KF_GEMM_PAIR (256 x bn tiles on CTA pairs, cta_group::2) gives the same
    bits as the one-CTA kernel: same products, same order. Covers an odd
    number of row tiles (the last pair's second CTA stores nothing), N and K
    not multiples of the tile, and a live-tile list with gaps (rows of the
    other tiles keep their contents)."""
    from techjam2026_b200 import _lib
    L = _lib.lib()
    torch.manual_seed(M * 3 + N + K + bn)
    a = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / math.sqrt(K)
    bias = torch.randn(N, device="cuda")
    a2, w2 = to_planes(a).contiguous(), to_planes(w).contiguous()
    lt = lc = None
    n_rt = (M + 127) // 128
    if live:
        keep = torch.zeros(M, dtype=torch.uint8, device="cuda")
        for t in range(0, n_rt, 3):  # tiles 0, 3, 6, ... live
            keep[t * 128] = 1
        lt = torch.empty(n_rt, dtype=torch.int32, device="cuda")
        lc = torch.zeros(1, dtype=torch.int32, device="cuda")
        _lib.check(L.kf_live_row_tiles(keep.data_ptr(), M, lt.data_ptr(), lc.data_ptr(),
                                       _lib.stream_ptr()), "live tiles")
    outs = []
    for pair in (False, True):
        shape = (2, M, N) if out_split else (M, N)
        c = torch.full(shape, 3, dtype=torch.int16 if out_split else torch.float32, device="cuda")
        flags = (_lib.KF_GEMM_OUT_BF16X2 if out_split else 0) | (_lib.KF_GEMM_PAIR if pair else 0)
        rc = L.kf_gemm_bf16x3(a2.data_ptr(), K, w2.data_ptr(), K, bias.data_ptr(), c.data_ptr(), N,
                              M, N, K, 1 if gelu else 0, flags, bn, 0, 0,
                              lt.data_ptr() if live else None, lc.data_ptr() if live else None,
                              _lib.stream_ptr())
        _lib.check(rc, "kf_gemm_bf16x3")
        outs.append(c)
    assert torch.equal(outs[0], outs[1])
    assert L.kf_device_status(0) == 0
    got = from_planes(outs[1]) if out_split else outs[1]
    ref = a.double() @ w.double().t() + bias.double()
    if gelu:
        ref = F.gelu(ref, approximate="none")
    rows = torch.arange(M, device="cuda")
    computed = ((rows // 128) % 3 == 0) if live else torch.ones(M, dtype=torch.bool, device="cuda")
    assert (got[computed].double() - ref[computed]).abs().max().item() < 6e-4
    if live:
        untouched = outs[1][:, ~computed] if out_split else outs[1][~computed]
        assert torch.all(untouched == 3)


@pytest.mark.parametrize("M,N,K", [(517, 384, 512), (300, 200, 136), (2048, 512, 2048),
                                   (256, 256, 24)])
@pytest.mark.parametrize("bn", [64, 96, 128, 256])
@pytest.mark.parametrize("live", [False, True])
def test_gemm_bf16x3_static_w_prefetch_bit_identical(M, N, K, bn, live):
    """KF_GEMM_W_STATIC loads the first W stages before waiting for the
    previous kernel: same bits, including CTAs that end up with no tile (a
    sparse live-tile list) and so must drain their prefetched stages."""
    from techjam2026_b200 import _lib
    L = _lib.lib()
    torch.manual_seed(M + 5 * N + K + bn)
    a = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / math.sqrt(K)
    bias = torch.randn(N, device="cuda")
    a2, w2 = to_planes(a).contiguous(), to_planes(w).contiguous()
    torch.cuda.synchronize()  # W is written before the GEMM's predecessor starts
    lt = lc = None
    if live:
        n_rt = (M + 127) // 128
        keep = torch.zeros(M, dtype=torch.uint8, device="cuda")
        keep[(n_rt - 1) * 128] = 1  # only the last row tile is live
        lt = torch.empty(n_rt, dtype=torch.int32, device="cuda")
        lc = torch.zeros(1, dtype=torch.int32, device="cuda")
        _lib.check(L.kf_live_row_tiles(keep.data_ptr(), M, lt.data_ptr(), lc.data_ptr(),
                                       _lib.stream_ptr()), "live tiles")
    outs = []
    for static in (False, True):
        c = torch.full((M, N), 3.0, device="cuda")
        flags = _lib.KF_GEMM_W_STATIC if static else 0
        rc = L.kf_gemm_bf16x3(a2.data_ptr(), K, w2.data_ptr(), K, bias.data_ptr(), c.data_ptr(), N,
                              M, N, K, 0, flags, bn, 0, 0, lt.data_ptr() if live else None,
                              lc.data_ptr() if live else None, _lib.stream_ptr())
        _lib.check(rc, "kf_gemm_bf16x3")
        outs.append(c)
    assert torch.equal(outs[0], outs[1])
    assert L.kf_device_status(0) == 0


@pytest.mark.parametrize("M,N,K", [(4096, 512, 512), (517, 384, 512), (300, 200, 136),
                                   (1000, 1000, 1000), (256, 112, 64), (128, 16, 32)])
@pytest.mark.parametrize("gelu", [False, True])
@pytest.mark.parametrize("static", [False, True])
def test_gemm_bf16x3_bn112_bit_identical(M, N, K, gelu, static):
    """N tile 112 (one wave for N = 512 on 148 SMs: 5 column tiles): the last
    16-column chunk of each tile is stored directly, bounded by the tile.
    Same bits as N tile 128 (a tile only moves work between CTAs)."""
    from techjam2026_b200 import _lib
    L = _lib.lib()
    torch.manual_seed(M + 3 * N + K)
    a = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / math.sqrt(K)
    bias = torch.randn(N, device="cuda")
    a2, w2 = to_planes(a).contiguous(), to_planes(w).contiguous()
    torch.cuda.synchronize()
    outs = []
    for bn in (128, 112):
        c = torch.full((M, N), 3.0, device="cuda")
        rc = L.kf_gemm_bf16x3(a2.data_ptr(), K, w2.data_ptr(), K, bias.data_ptr(), c.data_ptr(), N,
                              M, N, K, 1 if gelu else 0,
                              _lib.KF_GEMM_W_STATIC if static else 0, bn, 0, 0, None, None,
                              _lib.stream_ptr())
        _lib.check(rc, "kf_gemm_bf16x3")
        outs.append(c)
    assert torch.equal(outs[0], outs[1])
    assert L.kf_device_status(0) == 0


def test_gemm_bf16x3_bn112_rejects_split_output_and_pairs():
    from techjam2026_b200 import _lib
    L = _lib.lib()
    a2 = torch.zeros(2, 128, 64, dtype=torch.int16, device="cuda")
    w2 = torch.zeros(2, 112, 64, dtype=torch.int16, device="cuda")
    c = torch.zeros(2, 128, 112, dtype=torch.int16, device="cuda")
    for flags in (_lib.KF_GEMM_OUT_BF16X2, _lib.KF_GEMM_PAIR):
        rc = L.kf_gemm_bf16x3(a2.data_ptr(), 64, w2.data_ptr(), 64, None, c.data_ptr(), 112, 128,
                              112, 64, 0, flags, 112, 0, 0, None, None, _lib.stream_ptr())
        assert rc == _lib.KF_E_INVALID


@pytest.mark.parametrize("M,N,K", [(4096, 512, 512), (4096, 512, 2048), (300, 200, 136),
                                   (128, 64, 64), (1000, 1000, 1000), (256, 256, 24),
                                   (4096, 2048, 512)])
@pytest.mark.parametrize("bn", [64, 128, 256])
@pytest.mark.parametrize("gelu", [False, True])
@pytest.mark.parametrize("live", [False, True])
def test_gemm_bf16x3_stream_k(M, N, K, bn, gelu, live):
    """Stream-K: every SM takes an even share of the (tile, k block) pairs and
    a split tile is finished by its first part. Deterministic (two runs agree
    bit for bit), within fp32 reassociation of the one-CTA kernel, padded row
    tiles untouched, and the workspace's counters are zero again afterwards."""
    from techjam2026_b200 import _lib
    L = _lib.lib()
    torch.manual_seed(M + N + 7 * K + bn)
    a = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / math.sqrt(K)
    bias = torch.randn(N, device="cuda")
    a2, w2 = to_planes(a).contiguous(), to_planes(w).contiguous()
    lt = lc = None
    n_rt = (M + 127) // 128
    computed = torch.ones(M, dtype=torch.bool, device="cuda")
    if live:
        keep = torch.zeros(M, dtype=torch.uint8, device="cuda")
        for t in range(0, n_rt, 2):
            keep[t * 128] = 1
        lt = torch.empty(n_rt, dtype=torch.int32, device="cuda")
        lc = torch.zeros(1, dtype=torch.int32, device="cuda")
        _lib.check(L.kf_live_row_tiles(keep.data_ptr(), M, lt.data_ptr(), lc.data_ptr(),
                                       _lib.stream_ptr()), "live tiles")
        computed = (torch.arange(M, device="cuda") // 128) % 2 == 0
    nbytes = int(L.kf_gemm_sk_workspace_bytes(M, N, bn))
    ws = torch.zeros(nbytes // 4, dtype=torch.int32, device="cuda")
    tiles = n_rt * ((N + bn - 1) // bn)
    flags_view = ws[tiles * 2 * 128 * bn:]
    args = lambda c: (a2.data_ptr(), K, w2.data_ptr(), K, bias.data_ptr(), c.data_ptr(), N, M, N,
                      K, 1 if gelu else 0, 0, bn, 0, 0, lt.data_ptr() if live else None,
                      lc.data_ptr() if live else None)
    ref = torch.full((M, N), 3.0, device="cuda")
    _lib.check(L.kf_gemm_bf16x3(*args(ref), _lib.stream_ptr()), "kf_gemm_bf16x3")
    outs = []
    for _ in range(2):
        c = torch.full((M, N), 3.0, device="cuda")
        _lib.check(L.kf_gemm_bf16x3_sk(*args(c), ws.data_ptr(), nbytes, _lib.stream_ptr()),
                   "kf_gemm_bf16x3_sk")
        outs.append(c)
        torch.cuda.synchronize()
        assert torch.count_nonzero(flags_view) == 0
    assert L.kf_device_status(0) == 0
    assert torch.equal(outs[0], outs[1])
    err = (outs[0][computed] - ref[computed]).abs().max().item()
    assert err <= 1e-5 * max(1.0, ref[computed].abs().max().item()), err
    assert torch.all(outs[0][~computed] == 3.0)


def test_gemm_bf16x3_stream_k_rejects_bad_workspace():
    from techjam2026_b200 import _lib
    L = _lib.lib()
    a2 = torch.zeros(2, 128, 64, dtype=torch.int16, device="cuda")
    w2 = torch.zeros(2, 64, 64, dtype=torch.int16, device="cuda")
    c = torch.zeros(128, 64, device="cuda")
    need = int(L.kf_gemm_sk_workspace_bytes(128, 64, 64))
    ws = torch.zeros(need // 4, dtype=torch.int32, device="cuda")
    for wptr, wbytes, bn in ((None, need, 64), (ws.data_ptr(), need - 4, 64),
                             (ws.data_ptr(), need, 96)):
        rc = L.kf_gemm_bf16x3_sk(a2.data_ptr(), 64, w2.data_ptr(), 64, None, c.data_ptr(), 64, 128,
                                 64, 64, 0, 0, bn, 0, 0, None, None, wptr, wbytes,
                                 _lib.stream_ptr())
        assert rc == _lib.KF_E_INVALID


def test_gemm_bf16x3_pair_rejects_bad_tiles():
    from techjam2026_b200 import _lib
    L = _lib.lib()
    a2 = torch.zeros(2, 128, 64, dtype=torch.int16, device="cuda")
    w2 = torch.zeros(2, 64, 64, dtype=torch.int16, device="cuda")
    c = torch.zeros(128, 64, device="cuda")
    # bn 64 and 96 have no pair form; bit 16 is no flag of this GEMM.
    for bn, extra in ((64, 0), (96, 0), (128, 16)):
        rc = L.kf_gemm_bf16x3(a2.data_ptr(), 64, w2.data_ptr(), 64, None, c.data_ptr(), 64, 128,
                              64, 64, 0, _lib.KF_GEMM_PAIR | extra, bn, 0, 0, None, None,
                              _lib.stream_ptr())
        assert rc == _lib.KF_E_INVALID


def test_gemm_bf16x3_head_padded_output():
    from techjam2026_b200 import _lib
    torch.manual_seed(11)
    M, N, K = 256, 3 * 128, 128
    a = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / math.sqrt(K)
    out = torch.full((M, 3 * 16 * 16), 7.0, device="cuda")
    a2, w2 = to_planes(a).contiguous(), to_planes(w).contiguous()   # keep them alive
    rc = _lib.lib().kf_gemm_bf16x3(a2.data_ptr(), K, w2.data_ptr(), K, None,
                                   out.data_ptr(), out.stride(0), M, N, K, 0, 0, 0, 8, 16,
                                   None, None, _lib.stream_ptr())
    _lib.check(rc, "kf_gemm_bf16x3")
    ref = (a.double() @ w.double().t()).view(M, 48, 8)
    got = out.view(M, 48, 16)
    assert (got[..., :8].double() - ref).abs().max().item() < 6e-4
    assert torch.all(got[..., 8:] == 7.0)


def test_layernorm_split_output():
    from techjam2026_b200 import _lib
    torch.manual_seed(12)
    M, d = 517, 512
    x, y = torch.randn(M, d, device="cuda"), torch.randn(M, d, device="cuda")
    w, b = torch.randn(d, device="cuda"), torch.randn(d, device="cuda")
    h2 = torch.zeros(2, M, d, dtype=torch.int16, device="cuda")
    rc = _lib.lib().kf_ln_add_mask(x.data_ptr(), d, y.data_ptr(), d, None, w.data_ptr(),
                                   b.data_ptr(), None, 0, h2.data_ptr(), d, M, d, 1e-5,
                                   _lib.KF_LN_OUT_BF16X2, _lib.stream_ptr())
    _lib.check(rc, "kf_ln_add_mask")
    ref = F.layer_norm((x + y).double(), (d,), w.double(), b.double(), 1e-5)
    assert torch.equal(h2, to_planes(F.layer_norm(x + y, (d,), w, b, 1e-5))) or \
        (from_planes(h2).double() - ref).abs().max().item() < 1e-4


def test_attention_split_output():
    from techjam2026_b200 import _lib
    torch.manual_seed(13)
    B, H, S, Dh = 2, 4, 300, 64
    q, k, v = (torch.randn(B, H, S, Dh, device="cuda") for _ in range(3))
    keep = (torch.arange(S, device="cuda")[None, :] < torch.tensor([[300], [170]],
                                                                    device="cuda")).to(torch.uint8)
    ref = flash_attention(q, k, v, keep=keep, causal=True)
    L = _lib.lib()
    bits = torch.empty(int(L.kf_keep_bits_words(B, S)), dtype=torch.int32, device="cuda")
    _lib.check(L.kf_keep_bits(keep.data_ptr(), S, B, S, bits.data_ptr(), _lib.stream_ptr()), "b")
    o2 = torch.zeros(2, B, H, S, Dh, dtype=torch.int16, device="cuda")
    st = q.stride()
    rc = L.kf_flash_fwd_tf32(q.data_ptr(), *st[:3], k.data_ptr(), *st[:3], v.data_ptr(), *st[:3],
                             o2.data_ptr(), *o2[0].stride()[:3], bits.data_ptr(), B, H, S, Dh, Dh,
                             Dh ** -0.5, _lib.KF_ATTN_CAUSAL | _lib.KF_ATTN_OUT_BF16X2,
                             _lib.stream_ptr())
    _lib.check(rc, "kf_flash_fwd_tf32")
    assert (from_planes(o2) - ref).abs().max().item() < 1e-4


def _flash_raw(q, k, v, keep, o, flags, o_strides=None, dh_out=None):
    """kf_flash_fwd_tf32 on [B, H, S, Dh] views with an explicit output
    buffer and strides (batch, head, row)."""
    from techjam2026_b200 import _lib
    L = _lib.lib()
    B, H, S, Dh = q.shape
    bits = None
    if keep is not None:
        bits = torch.empty(int(L.kf_keep_bits_words(B, S)), dtype=torch.int32, device="cuda")
        _lib.check(L.kf_keep_bits(keep.data_ptr(), S, B, S, bits.data_ptr(), _lib.stream_ptr()),
                   "kf_keep_bits")
    st = q.stride()
    rc = L.kf_flash_fwd_tf32(q.data_ptr(), *st[:3], k.data_ptr(), *st[:3], v.data_ptr(), *st[:3],
                             o.data_ptr(), *o_strides, bits.data_ptr() if bits is not None else None,
                             B, H, S, Dh, dh_out or Dh, Dh ** -0.5, flags, _lib.stream_ptr())
    _lib.check(rc, "kf_flash_fwd_tf32")
    torch.cuda.synchronize()
    return bits


@pytest.mark.parametrize("Dh", [32, 64, 128, 256])
@pytest.mark.parametrize("split", [False, True])
@pytest.mark.parametrize("row_pad", [0, 4])
def test_flash_output_paths(Dh, split, row_pad):
    """The output tile is written by TMA stores when rows are whole 128-byte
    swizzle rows with 16-byte aligned strides, else by per-thread stores
    (row_pad = 4 elements breaks the alignment for bf16 planes, and an odd
    row stride for fp32). Both write the same values, into [B, S, H, Dh]
    rows, bf16 hi/lo planes B batches apart, and nothing outside the rows."""
    from techjam2026_b200 import _lib
    torch.manual_seed(20 + Dh)
    B, H, S = 2, 3, 333
    q, k, v = (torch.randn(B, H, S, Dh, device="cuda") for _ in range(3))
    keep = (torch.arange(S, device="cuda")[None, :] < torch.tensor([[333], [150]],
                                                                    device="cuda")).to(torch.uint8)
    ref = reference_attention(q, k, v, keep, True)
    pad = row_pad if split else (row_pad // 4)     # fp32: 1 element -> unaligned rows
    row = H * Dh + pad
    flags = _lib.KF_ATTN_CAUSAL
    if split:
        flags |= _lib.KF_ATTN_OUT_BF16X2
        buf = torch.full((2 * B, S, row), 0x1234, dtype=torch.int16, device="cuda")
    else:
        buf = torch.full((B, S, row), 7.0, device="cuda")
    _flash_raw(q, k, v, keep, buf, flags, (S * row, Dh, row))
    got_rows = buf[..., :H * Dh]
    if split:
        got = from_planes(got_rows.reshape(2, B, S, H * Dh))
        if pad:
            assert torch.all(buf[..., H * Dh:] == 0x1234)
        tol = 1e-4                            # the bf16 pair carries ~2^-17 relative error
    else:
        got = got_rows
        if pad:
            assert torch.all(buf[..., H * Dh:] == 7.0)
        tol = 5e-3
    got = got.reshape(B, S, H, Dh).permute(0, 2, 1, 3).double()
    fa = flash_attention(q, k, v, keep=keep, causal=True)
    if split:
        assert (got - fa.double()).abs().max().item() < tol
    assert (got - ref).abs().max().item() < 5e-3


def _reference_rows(q, k, v, keep, causal, rows):
    """float64 attention for the query rows `rows` only (against all keys)."""
    scale = q.shape[-1] ** -0.5
    qs = q[:, :, rows].double()
    scores = qs @ k.double().transpose(-2, -1) * scale
    S = k.shape[2]
    if causal:
        r = torch.as_tensor(rows, device=q.device)[:, None]
        scores = scores.masked_fill(torch.arange(S, device=q.device)[None, :] > r, float("-inf"))
    if keep is not None:
        scores = scores.masked_fill(~keep.bool()[:, None, None, :], float("-inf"))
    p = torch.nan_to_num(torch.softmax(scores, dim=-1), nan=0.0)
    return p @ v.double()


@pytest.mark.parametrize("Dh,S", [(16, 777), (64, 777), (128, 777), (256, 777), (64, 66000)])
@pytest.mark.parametrize("causal", [False, True])
def test_flash_skip_empty_query_tiles(Dh, S, causal):
    """KF_ATTN_SKIP_EMPTY_Q: tiles holding a valid query are bit-identical to
    the unskipped kernel and a tile without one is zeroed. Valid rows are not
    a prefix; one tile is empty in the middle of a sequence; S = 66000 keeps
    the key bits in global memory (too long for the shared-memory staging)."""
    from techjam2026_b200 import _lib
    torch.manual_seed(Dh + S)
    B, H = 3, 2
    q, k, v = (torch.randn(B, H, S, Dh, device="cuda") for _ in range(3))
    keep = (torch.rand(B, S, device="cuda") > 0.2).to(torch.uint8)
    keep[0, 128:256] = 0          # an empty tile inside sequence 0
    keep[1, 300:] = 0             # sequence 1 ends at 300: tiles 3.. are empty
    keep[2] = 0                   # sequence 2 has no valid token at all
    flags = _lib.KF_ATTN_CAUSAL if causal else 0
    full = torch.empty(B, H, S, Dh, device="cuda")
    _flash_raw(q, k, v, keep, full, flags, full.stride()[:3])
    o = torch.full((B, H, S, Dh), 7.0, device="cuda")
    _flash_raw(q, k, v, keep, o, flags | _lib.KF_ATTN_SKIP_EMPTY_Q, o.stride()[:3])
    n_t = (S + 127) // 128
    tile_live = torch.zeros(B, n_t, dtype=torch.bool, device="cuda")
    for t in range(n_t):
        tile_live[:, t] = keep[:, t * 128:(t + 1) * 128].any(dim=1)
    row_live = tile_live.repeat_interleave(128, dim=1)[:, :S]
    live = row_live[:, None, :, None].expand_as(o)
    assert torch.equal(o[live], full[live])
    assert torch.all(o[~live] == 0.0)
    assert int((~row_live).sum()) > 0


@pytest.mark.parametrize("B,S", [(1, 100), (7, 333), (64, 2048), (300, 64), (4097, 32)])
def test_batch_order_ranks_rows_longest_first(B, S):
    """kf_batch_order: a permutation of the rows by valid-key count, longest
    first, ties by row index; identity above 4096 rows."""
    from techjam2026_b200 import _lib
    L = _lib.lib()
    g = torch.Generator().manual_seed(B + S)
    lengths = torch.randint(0, S + 1, (B,), generator=g)
    lengths[: B // 3] = lengths[0]                      # ties
    keep = (torch.rand(B, S, generator=g) < 0.7).to(torch.uint8)
    keep &= (torch.arange(S)[None, :] < lengths[:, None]).to(torch.uint8)
    keep = keep.cuda()
    bits = torch.empty(int(L.kf_keep_bits_words(B, S)), dtype=torch.int32, device="cuda")
    st = _lib.stream_ptr()
    _lib.check(L.kf_keep_bits(keep.data_ptr(), S, B, S, bits.data_ptr(), st), "kf_keep_bits")
    order = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    _lib.check(L.kf_batch_order(bits.data_ptr(), B, S, order.data_ptr(), st), "kf_batch_order")
    got = order.cpu().tolist()
    if B > 4096:
        assert got == list(range(B))
        return
    n = keep.sum(dim=1).cpu().tolist()
    assert got == sorted(range(B), key=lambda b: (-n[b], b))


@pytest.mark.parametrize("Dh", [16, 64, 128, 256])
def test_flash_ordered_rows_are_bit_identical(Dh):
    """kf_flash_fwd_tf32_ordered only changes which CTA runs when: same bits
    as kf_flash_fwd_tf32 on ragged, non-prefix masks (split output)."""
    from techjam2026_b200 import _lib
    L = _lib.lib()
    torch.manual_seed(Dh)
    B, H, S = 6, 2, 700
    d = H * Dh
    qkv = torch.randn(B, S, 3, H, Dh, device="cuda")
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    lengths = torch.tensor([700, 5, 333, 0, 699, 128])
    keep = (torch.arange(S)[None, :] < lengths[:, None]).to(torch.uint8)
    keep &= (torch.rand(B, S) < 0.9).to(torch.uint8)
    keep = keep.cuda()
    st = _lib.stream_ptr()
    bits = torch.empty(int(L.kf_keep_bits_words(B, S)), dtype=torch.int32, device="cuda")
    _lib.check(L.kf_keep_bits(keep.data_ptr(), S, B, S, bits.data_ptr(), st), "kf_keep_bits")
    order = torch.empty(B, dtype=torch.int32, device="cuda")
    _lib.check(L.kf_batch_order(bits.data_ptr(), B, S, order.data_ptr(), st), "kf_batch_order")
    flags = _lib.KF_ATTN_CAUSAL | _lib.KF_ATTN_SKIP_EMPTY_Q | _lib.KF_ATTN_OUT_BF16X2
    qs = q.stride()
    outs = []
    for ordered in (False, True):
        o = torch.full((2, B, S, d), 7, dtype=torch.int16, device="cuda")
        args = [q.data_ptr(), *qs[:3], k.data_ptr(), *qs[:3], v.data_ptr(), *qs[:3],
                o.data_ptr(), S * d, Dh, d, bits.data_ptr()]
        if ordered:
            rc = L.kf_flash_fwd_tf32_ordered(*args, order.data_ptr(), B, H, S, Dh, Dh,
                                             Dh ** -0.5, flags, st)
        else:
            rc = L.kf_flash_fwd_tf32(*args, B, H, S, Dh, Dh, Dh ** -0.5, flags, st)
        _lib.check(rc, "attention")
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    assert order.cpu().tolist()[-1] == 3          # the row without a valid key runs last


@pytest.mark.parametrize("Dh,S", [(64, 66000), (256, 15000)])
def test_flash_key_bits_beyond_shared_memory_staging(Dh, S):
    """Rows whose key bits exceed the shared-memory staging area (2048 words
    at Dh 64, 448 at Dh 256) read them from global memory; a non-prefix mask
    makes every tile's bits matter."""
    from techjam2026_b200 import _lib
    torch.manual_seed(30)
    B, H = 1, 1
    q, k, v = (torch.randn(B, H, S, Dh, device="cuda") for _ in range(3))
    keep = (torch.rand(B, S, device="cuda") > 0.3).to(torch.uint8)
    keep[:, 5000:9000] = 0
    o = torch.empty(B, H, S, Dh, device="cuda")
    _flash_raw(q, k, v, keep, o, _lib.KF_ATTN_CAUSAL, o.stride()[:3])
    rows = list(range(0, 64)) + list(range(6000, 6100)) + list(range(S - 200, S))
    ref = _reference_rows(q, k, v, keep, True, rows)
    assert (o[:, :, rows].double() - ref).abs().max().item() < 5e-3


@pytest.mark.parametrize("out_split", [False, True])
def test_gemm_gelu_epilogue_error_bound(out_split):
    """The GELU epilogue evaluates erf with Abramowitz & Stegun 7.1.26
    (|error| <= 1.5e-7). Inputs exactly representable in bf16 and an identity
    weight make the GEMM itself exact, so the output isolates the epilogue:
    within 3e-7 * max(1, |x|) of float64 GELU (erf) for fp32 output, plus the
    bf16 hi/lo pair's own rounding (2^-16 relative) for split output."""
    from techjam2026_b200 import _lib
    torch.manual_seed(14)
    M, K = 4096, 16
    x = (torch.rand(M, K, device="cuda") * 20 - 10).to(torch.bfloat16).float()
    x[0, :8] = torch.tensor([0.0, -0.0, 1e-3, -1e-3, 5.0, -5.0, 9.5, -9.5])
    w = torch.eye(K, device="cuda")
    bias = torch.zeros(K, device="cuda")
    a2, w2 = to_planes(x).contiguous(), to_planes(w).contiguous()
    if out_split:
        out = torch.zeros(2, M, K, dtype=torch.int16, device="cuda")
        flags = _lib.KF_GEMM_OUT_BF16X2
    else:
        out = torch.zeros(M, K, device="cuda")
        flags = 0
    rc = _lib.lib().kf_gemm_bf16x3(a2.data_ptr(), K, w2.data_ptr(), K, bias.data_ptr(),
                                   out.data_ptr(), K, M, K, K, _lib.KF_EPI_BIAS_GELU, flags, 0, 0,
                                   0, None, None, _lib.stream_ptr())
    _lib.check(rc, "kf_gemm_bf16x3")
    torch.cuda.synchronize()
    got = (from_planes(out) if out_split else out).double()
    xd = x.double()
    ref = 0.5 * xd * (1 + torch.erf(xd / math.sqrt(2)))
    err = (got - ref).abs()
    bound = 3e-7 * xd.abs().clamp(min=1)
    if out_split:
        bound = bound + 2.0 ** -16 * ref.abs()
    assert bool((err <= bound).all()), f"max err {err.max().item()}"
    # and against the fp32 erf GELU that torch computes on the GPU
    assert (got - F.gelu(x).double()).abs().max().item() < 2e-5


# --------------------------------------------------------------- ops surface options

def test_add_mask_layernorm_options():
    """want_residual=False returns (None, h) with the same h; keep given as
    float, bool or uint8 gives the same bits; a strided x is accepted;
    non-fp32 outputs are refused (the reference's fp16 options are out of
    this fp32 path)."""
    torch.manual_seed(21)
    M, d = 300, 256
    wide = torch.randn(M, 2 * d, device="cuda")
    x = wide[:, :d]                                   # row stride 2d
    y = torch.randn(M, d, device="cuda")
    w, b = torch.randn(d, device="cuda"), torch.randn(d, device="cuda")
    keep_f = (torch.rand(M, device="cuda") > 0.25).float()
    s, h = add_mask_layernorm(x, y, keep_f, w, b, mask_out=True)
    none, h2 = add_mask_layernorm(x, y, keep_f, w, b, mask_out=True, want_residual=False)
    assert none is None and torch.equal(h, h2)
    for keep in (keep_f.bool(), keep_f.to(torch.uint8)):
        s3, h3 = add_mask_layernorm(x, y, keep, w, b, mask_out=True)
        assert torch.equal(s3, s) and torch.equal(h3, h)
    assert torch.equal(s, (x + y) * keep_f[:, None])
    with pytest.raises(TypeError):
        add_mask_layernorm(x, y, keep_f, w, b, out_dtype=torch.float16)


@pytest.mark.parametrize("causal", [False, True])
def test_flash_attention_options(causal):
    """sm_scale other than Dh^-1/2, keep=None, a caller-provided `out` view,
    and the reference's tuning hints (smem_kb, block) accepted and ignored;
    round_scores_to (fp16/bf16 I/O only) refused."""
    torch.manual_seed(22)
    B, H, S, Dh = 2, 3, 200, 64
    q, k, v = (torch.randn(B, H, S, Dh, device="cuda") for _ in range(3))
    scale = 0.3
    ref = _reference_rows(q * (scale / Dh ** -0.5), k, v, None, causal, list(range(S)))
    buf = torch.full((B, S, H, Dh), 5.0, device="cuda")
    o = flash_attention(q, k, v, causal=causal, sm_scale=scale, smem_kb=99.0,
                        block=(128, 64, 2, 2), out=buf.permute(0, 2, 1, 3))
    assert o.data_ptr() == buf.data_ptr()
    assert (buf.permute(0, 2, 1, 3).double() - ref).abs().max().item() < 5e-3
    with pytest.raises(NotImplementedError):
        flash_attention(q, k, v, causal=causal, round_scores_to=torch.float16)


# ------------------------------------------------------------ persistent attention

def _bits_of(keep):
    from techjam2026_b200 import _lib
    L = _lib.lib()
    B, S = keep.shape
    bits = torch.empty(int(L.kf_keep_bits_words(B, S)), dtype=torch.int32, device="cuda")
    _lib.check(L.kf_keep_bits(keep.data_ptr(), keep.stride(0), B, S, bits.data_ptr(),
                              _lib.stream_ptr()), "kf_keep_bits")
    return bits


def _expected_schedule(keep, B, H, S):
    """The work list kf_attn_schedule documents, built on the host: rows by
    valid-key count (longest first, ties by index), per row its heads, per
    head the query tiles holding a valid token from the last to the first;
    then the tiles without one, in the same row and head order."""
    n_qt = (S + 127) // 128
    if keep is None:
        counts = [S] * B
        live = [[True] * n_qt for _ in range(B)]
    else:
        kc = keep.cpu().bool()
        counts = kc.sum(1).tolist()
        live = [[bool(kc[b, t * 128:(t + 1) * 128].any()) for t in range(n_qt)] for b in range(B)]
    order = sorted(range(B), key=lambda b: (-counts[b], b)) if B <= 4096 else list(range(B))
    items = []
    for b in order:
        for h in range(H):
            items += [(b * H + h, t) for t in reversed(range(n_qt)) if live[b][t]]
    n_live = len(items)
    for b in order:
        for h in range(H):
            items += [(b * H + h, t) for t in range(n_qt) if not live[b][t]]
    return n_live, items


@pytest.mark.parametrize("B,H,S,masked", [(1, 1, 100, True), (7, 3, 333, True), (64, 12, 2048, True),
                                          (5, 2, 66000, True), (300, 2, 200, True),
                                          (3, 4, 1000, False)])
def test_attn_schedule_matches_its_definition(B, H, S, masked):
    from techjam2026_b200.ops.flash import attn_schedule
    g = torch.Generator().manual_seed(B * 7 + S)
    keep = None
    if masked:
        lengths = torch.randint(0, S + 1, (B,), generator=g)
        lengths[: B // 3] = lengths[0]                          # ties
        keep = (torch.rand(B, S, generator=g) < 0.8).to(torch.uint8)
        keep &= (torch.arange(S)[None, :] < lengths[:, None]).to(torch.uint8)
        if S > 300:
            keep[0, 128:256] = 0                                # an empty tile mid-row
        keep = keep.cuda()
    bits = _bits_of(keep) if keep is not None else None
    sched = attn_schedule(bits, B, H, S)
    torch.cuda.synchronize()
    n_live, items = _expected_schedule(keep, B, H, S)
    s = sched.cpu()
    assert s[0].item() == 0 and s[1].item() == 0
    assert s[2].item() == n_live and s[3].item() == len(items) == B * H * ((S + 127) // 128)
    got = s[8:8 + 2 * len(items)].view(-1, 2).tolist()
    assert [tuple(x) for x in got] == items


def _attn_call(q, k, v, o, bits, flags, sched=None, o_strides=None, dh_out=None):
    from techjam2026_b200 import _lib
    L = _lib.lib()
    B, H, S, Dh = q.shape
    qs = q.stride()
    args = [q.data_ptr(), *qs[:3], k.data_ptr(), *k.stride()[:3], v.data_ptr(), *v.stride()[:3],
            o.data_ptr(), *(o_strides or o.stride()[:3]),
            bits.data_ptr() if bits is not None else None]
    if sched is None:
        rc = L.kf_flash_fwd_tf32(*args, B, H, S, Dh, dh_out or Dh, Dh ** -0.5, flags,
                                 _lib.stream_ptr())
    else:
        rc = L.kf_flash_fwd_tf32_sched(*args, sched.data_ptr(), B, H, S, Dh, dh_out or Dh,
                                       Dh ** -0.5, flags, _lib.stream_ptr())
    _lib.check(rc, "attention")


@pytest.mark.parametrize("Dh", [16, 32, 64, 128, 256])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("mode", ["zeros", "compute", "untouched"])
def test_flash_sched_is_bit_identical_to_one_cta_per_tile(Dh, causal, mode):
    """kf_flash_fwd_tf32_sched gives the bits of kf_flash_fwd_tf32 for every
    row it writes, on ragged non-prefix masks with empty query tiles (inside
    a row, at its end, a row without any valid token), twice in a row on one
    work list (its counters reset themselves). Empty query tiles: zeros
    (KF_ATTN_SKIP_EMPTY_Q), computed like any tile, or left untouched
    (KF_ATTN_EMPTY_Q_UNTOUCHED)."""
    from techjam2026_b200 import _lib
    from techjam2026_b200.ops.flash import attn_schedule
    torch.manual_seed(Dh * 3 + causal)
    B, H, S = (5, 3, 777) if Dh < 256 else (3, 2, 500)
    q, k, v = (torch.randn(B, H, S, Dh, device="cuda") for _ in range(3))
    keep = (torch.rand(B, S, device="cuda") > 0.2).to(torch.uint8)
    keep[0, 128:256] = 0
    keep[1, 300:] = 0
    keep[2] = 0
    bits = _bits_of(keep)
    base = _lib.KF_ATTN_CAUSAL if causal else 0
    ref_flags = base | (_lib.KF_ATTN_SKIP_EMPTY_Q if mode != "compute" else 0)
    ref = torch.full((B, H, S, Dh), 7.0, device="cuda")
    _attn_call(q, k, v, ref, bits, ref_flags)
    flags = base | {"zeros": _lib.KF_ATTN_SKIP_EMPTY_Q, "compute": 0,
                    "untouched": _lib.KF_ATTN_EMPTY_Q_UNTOUCHED}[mode]
    sched = attn_schedule(bits, B, H, S)
    outs = []
    for _ in range(2):
        o = torch.full((B, H, S, Dh), 7.0, device="cuda")
        _attn_call(q, k, v, o, bits, flags, sched)
        outs.append(o)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    o = outs[0]
    if mode == "untouched":
        n_t = (S + 127) // 128
        kb = keep.bool()
        tile_live = torch.stack([kb[:, t * 128:(t + 1) * 128].any(1) for t in range(n_t)], 1)
        row_live = tile_live.repeat_interleave(128, dim=1)[:, :S][:, None, :, None].expand_as(o)
        assert torch.equal(o[row_live], ref[row_live])
        assert torch.all(o[~row_live] == 7.0)
    else:
        assert torch.equal(o, ref)
    assert sched[:2].cpu().tolist() == [0, 0]
    assert _lib.lib().kf_device_status(0) == 0


@pytest.mark.parametrize("Dh,H", [(64, 12), (16, 8), (32, 8), (128, 4), (256, 2)])
@pytest.mark.parametrize("split", [False, True])
def test_flash_sched_many_items_per_cta(split, Dh, H):
    """More items than resident CTAs (c4's rows: 16 rows x 16 query tiles
    per head, lengths from 1 to 2048, so items of 1 to 32 key tiles follow
    one another in every CTA) on strided views of a fused QKV buffer with
    [B, S, H, Dh] output rows, fp32 or bf16 hi/lo planes: the persistent
    kernel matches the one-CTA-per-tile kernel bit for bit, call after call
    on one list, and the float64 reference."""
    from techjam2026_b200 import _lib
    from techjam2026_b200.ops.flash import attn_schedule
    torch.manual_seed(41 + split + Dh)
    B, S = 16, 2048
    d = H * Dh
    qkv = torch.randn(B, S, 3, H, Dh, device="cuda")
    q, k, v = (qkv[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    lengths = torch.randint(1, S + 1, (B,))
    keep = (torch.arange(S)[None, :] < lengths[:, None]).to(torch.uint8).cuda()
    bits = _bits_of(keep)
    flags = _lib.KF_ATTN_CAUSAL | _lib.KF_ATTN_SKIP_EMPTY_Q
    if split:
        flags |= _lib.KF_ATTN_OUT_BF16X2
        mk = lambda: torch.full((2, B, S, d), 7, dtype=torch.int16, device="cuda")  # noqa: E731
    else:
        mk = lambda: torch.full((B, S, d), 7.0, device="cuda")  # noqa: E731
    strides = (S * d, Dh, d)
    ref = mk()
    _attn_call(q, k, v, ref, bits, flags, o_strides=strides)
    sched = attn_schedule(bits, B, H, S)
    for _ in range(3):
        o = mk()
        _attn_call(q, k, v, o, bits, flags, sched, o_strides=strides)
        torch.cuda.synchronize()
        assert torch.equal(o, ref)
    got = from_planes(o) if split else o
    got = got.reshape(B, S, H, Dh).permute(0, 2, 1, 3)
    rows = [0, 127, 128, 1000, 2047]
    want = _reference_rows(q, k, v, keep, True, rows)
    # rows of query tiles without a valid query are zeros (KF_ATTN_SKIP_EMPTY_Q)
    lens = lengths.cuda()
    live = (torch.tensor(rows, device="cuda")[None, :] // 128 * 128 < lens[:, None])
    live = live[:, None, :, None].expand_as(want)
    assert (got[:, :, rows].double() - want)[live].abs().max().item() < 5e-3
    assert torch.all(got[:, :, rows][~live] == 0)
    assert _lib.lib().kf_device_status(0) == 0


def test_flash_sched_without_mask_and_long_rows():
    """No key mask (every tile live) and a row long enough that the key bits
    do not fit the one-CTA kernel's shared-memory staging (S = 66000)."""
    from techjam2026_b200 import _lib
    from techjam2026_b200.ops.flash import attn_schedule
    torch.manual_seed(43)
    for (B, H, S, masked) in [(2, 4, 1000, False), (1, 2, 66000, True)]:
        q, k, v = (torch.randn(B, H, S, 64, device="cuda") for _ in range(3))
        keep = bits = None
        if masked:
            keep = (torch.rand(B, S, device="cuda") > 0.3).to(torch.uint8)
            keep[:, 5000:9000] = 0
            bits = _bits_of(keep)
        ref = torch.empty(B, H, S, 64, device="cuda")
        _attn_call(q, k, v, ref, bits, _lib.KF_ATTN_CAUSAL)
        o = torch.empty_like(ref)
        _attn_call(q, k, v, o, bits, _lib.KF_ATTN_CAUSAL, attn_schedule(bits, B, H, S))
        torch.cuda.synchronize()
        assert torch.equal(o, ref)


def _pack_reference(keep):
    """row_map, row_off and the packed tile count of a [B, S] keep mask."""
    B, S = keep.shape
    flat = keep.reshape(-1).bool()
    rank = torch.cumsum(flat.to(torch.int64), 0) - 1
    row_map = torch.where(flat, rank, torch.full_like(rank, -1)).to(torch.int32)
    counts = keep.bool().sum(1).to(torch.int64)
    row_off = torch.cat([torch.zeros(1, dtype=torch.int64, device=keep.device),
                         torch.cumsum(counts, 0)]).to(torch.int32)
    return row_map, row_off, (int(counts.sum()) + 127) // 128


@pytest.mark.parametrize("B,S", [(1, 1), (3, 5), (8, 512), (64, 2048), (5, 3000), (2, 65536),
                                 (40, 33)])
@pytest.mark.parametrize("kind", ["prefix", "random", "empty_rows"])
def test_pack_rows_matches_its_definition(B, S, kind):
    """kf_pack_rows: each valid token's rank among all valid tokens in
    row-major order, -1 for padding, the rows' offsets and the tile list of
    the packed rows, for prefix masks, arbitrary masks and empty rows."""
    from techjam2026_b200 import _lib
    L = _lib.lib()
    torch.manual_seed(B * 7 + S)
    if kind == "prefix":
        lens = torch.randint(0, S + 1, (B,))
        keep = (torch.arange(S)[None, :] < lens[:, None])
    else:
        keep = torch.rand(B, S) > 0.4
        if kind == "empty_rows":
            keep[::2] = False
    keep = keep.to(torch.uint8).cuda()
    bits = _bits_of(keep)
    M = B * S
    row_map = torch.full((M,), 7, dtype=torch.int32, device="cuda")
    row_off = torch.full((B + 1,), 7, dtype=torch.int32, device="cuda")
    tiles = torch.full(((M + 127) // 128,), -7, dtype=torch.int32, device="cuda")
    count = torch.full((1,), -7, dtype=torch.int32, device="cuda")
    _lib.check(L.kf_pack_rows(bits.data_ptr(), B, S, row_map.data_ptr(), row_off.data_ptr(),
                              tiles.data_ptr(), count.data_ptr(), _lib.stream_ptr()), "pack")
    torch.cuda.synchronize()
    want_map, want_off, n = _pack_reference(keep)
    assert torch.equal(row_map, want_map)
    assert torch.equal(row_off, want_off)
    assert count.item() == n
    assert torch.equal(tiles[:n].cpu(), torch.arange(n, dtype=torch.int32))


@pytest.mark.parametrize("M,d", [(300, 768), (517, 512), (1024, 1024), (200, 40)])
@pytest.mark.parametrize("mode", ["h_planes", "y_mask_out", "both_fp32"])
def test_ln_rows_map_matches_unmapped(M, d, mode):
    """kf_ln_add_mask_rows equals kf_ln_add_mask bit for bit on every row:
    its y read from, and / or its h written to, the row's packed position
    (rows mapped to -1 have no y and write no h)."""
    from techjam2026_b200 import _lib
    L = _lib.lib()
    torch.manual_seed(M + d)
    x = torch.randn(M, d, device="cuda")
    y = torch.randn(M, d, device="cuda")
    g, b = torch.randn(d, device="cuda"), torch.randn(d, device="cuda")
    keep = (torch.rand(M, device="cuda") > 0.3).to(torch.uint8)
    row_map, _, _ = _pack_reference(keep[None, :])
    T = int(keep.sum())
    valid = keep.bool()
    mapped = row_map[valid].long()
    planes = mode == "h_planes"
    flags = {"h_planes": _lib.KF_LN_OUT_BF16X2 | _lib.KF_LN_SKIP_PADDED,
             "y_mask_out": _lib.KF_LN_MASK_OUT,
             "both_fp32": _lib.KF_LN_SKIP_PADDED}[mode]
    mflags = {"h_planes": _lib.KF_LN_H_MAPPED, "y_mask_out": _lib.KF_LN_Y_MAPPED,
              "both_fp32": _lib.KF_LN_Y_MAPPED | _lib.KF_LN_H_MAPPED}[mode]

    def new_h():
        return (torch.full((2, M, d), 3, dtype=torch.int16, device="cuda") if planes
                else torch.full((M, d), 3.0, device="cuda"))
    s_a, h_a = x.clone(), new_h()
    _lib.check(L.kf_ln_add_mask(s_a.data_ptr(), d, y.data_ptr(), d, keep.data_ptr(), g.data_ptr(),
                                b.data_ptr(), s_a.data_ptr(), d, h_a.data_ptr(), d, M, d, 1e-5,
                                flags, _lib.stream_ptr()), "ln")
    # y in packed order for the mapped call
    yp = torch.full((M, d), float("nan"), device="cuda")
    if mflags & _lib.KF_LN_Y_MAPPED:
        yp[mapped] = y[valid]
    else:
        yp = y
    s_b, h_b = x.clone(), new_h()
    _lib.check(L.kf_ln_add_mask_rows(s_b.data_ptr(), d, yp.data_ptr(), d, keep.data_ptr(),
                                     g.data_ptr(), b.data_ptr(), s_b.data_ptr(), d, h_b.data_ptr(),
                                     d, M, d, 1e-5, flags | mflags, row_map.data_ptr(),
                                     _lib.stream_ptr()), "ln rows")
    torch.cuda.synchronize()
    assert torch.equal(s_a, s_b)
    if mflags & _lib.KF_LN_H_MAPPED:
        got = h_b[:, mapped] if planes else h_b[mapped]
        want = h_a[:, valid] if planes else h_a[valid]
        assert torch.equal(got, want)
        rest = h_b[:, T:] if planes else h_b[T:]
        assert torch.all(rest == 3)
    else:
        assert torch.equal(h_a, h_b)
