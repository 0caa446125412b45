"""The layer-stack forward on sm_100a: every op is a call into libkf_sm100.

Per forward (fp32 I/O, residual stream fp32 throughout):

  keep bits  <- kf_keep_bits(valid_token_mask)                  (once)
  res, h     <- kf_ln_add_mask(x, -, keep, LN1[0])              (entry norm)
  per layer i:
    qkv      <- kf_gemm_tf32(h, [Wq;Wk;Wv], b)                  fused QKV
    ctx      <- kf_flash_fwd_tf32(q, k, v views of qkv, keep bits, causal)
    y        <- kf_gemm_tf32(ctx, Wo, bo)                       out_proj
    res, h   <- kf_ln_add_mask(res, y, keep, LN2[i])            in place
    ffn      <- kf_gemm_tf32(h, W1, b1, GELU(erf))
    y        <- kf_gemm_tf32(ffn, W2, b2)
    res, h   <- kf_ln_add_mask(res, y, keep, LN1[i+1])          (last layer:
                final_norm with mask_out, written to the output)

That is the reference's fused structure (kernelforge/optimized.py:397-458),
with cuBLAS replaced by the tcgen05 GEMM and the GELU fused into FFN1's
epilogue. Masking the residual at the entry norm and inside every norm is
exact: padded rows never feed a valid row (keys are masked in attention, all
other ops are per row) and the reference zeroes them at every block end.

The whole forward is captured once per (shape, mask presence) into one CUDA
graph (kernelforge/optimized.py:588-625 pattern): static input buffers, one
replay, output cloned for the caller. There is no fallback: a failing
kernel raises.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch

from . import _lib
from .dispatch import DEFAULT_PLAN, Plan
from .model import LayerStack

SUPPORTED_HEAD_DIMS = (8, 16, 32, 64, 128, 256)


class _Weights:
    """Device copies laid out for the kernels, built once per device.

    [Wq;Wk;Wv] is fused. A GEMM running "bf16x3" gets its weight split into
    bf16 hi/lo planes [2, N, K]; a "tf32" GEMM gets it rounded to TF32; a
    "3xtf32" GEMM keeps all fp32 bits."""

    def __init__(self, model: LayerStack, device: torch.device, plan: Plan):
        from .ops.gemm import round_tf32 as rnd

        def prep_w(w: torch.Tensor, prec: str) -> torch.Tensor:
            w = w.detach().to(device=device, dtype=torch.float32).contiguous()
            if prec == "bf16x3":
                N, K = w.shape
                out = torch.empty(2, N, K, dtype=torch.int16, device=device)
                _lib.check(_lib.lib().kf_split_bf16x2(w.data_ptr(), N, K, K, out.data_ptr(), K,
                                                      _lib.stream_ptr()), "kf_split_bf16x2")
                return out
            return rnd(w) if (plan.round_tf32 and prec == "tf32") else w.clone()

        def prep_b(b: torch.Tensor) -> torch.Tensor:
            return b.detach().to(device=device, dtype=torch.float32).contiguous().clone()

        self.layers = []
        for layer in model.layers:
            a = layer.attention
            self.layers.append(dict(
                wqkv=prep_w(torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0),
                            plan.prec_qkv),
                bqkv=prep_b(torch.cat([a.q_proj.bias, a.k_proj.bias, a.v_proj.bias], 0)),
                wo=prep_w(a.out_proj.weight, plan.prec_out), bo=prep_b(a.out_proj.bias),
                w1=prep_w(layer.ffn_in.weight, plan.prec_ffn1), b1=prep_b(layer.ffn_in.bias),
                w2=prep_w(layer.ffn_out.weight, plan.prec_ffn2), b2=prep_b(layer.ffn_out.bias),
                ln1w=prep_b(layer.norm1.weight), ln1b=prep_b(layer.norm1.bias),
                ln2w=prep_b(layer.norm2.weight), ln2b=prep_b(layer.norm2.bias),
                eps1=float(layer.norm1.eps), eps2=float(layer.norm2.eps)))
        self.finw = prep_b(model.final_norm.weight)
        self.finb = prep_b(model.final_norm.bias)
        self.fin_eps = float(model.final_norm.eps)
        # Once every prepared weight is written, later GEMMs may load their
        # first W tiles before waiting for the previous kernel
        # (KF_GEMM_W_STATIC). Not inside a stream capture (no sync there).
        self.static = not torch.cuda.is_current_stream_capturing()
        if self.static:
            torch.cuda.current_stream(device).synchronize()


class _Workspace:
    """Activation buffers for one (B, S): allocated once, reused every call.

    An activation that feeds a "bf16x3" GEMM is kept as bf16 hi/lo planes
    [2, M, width] (same 4 bytes per value as fp32); otherwise fp32.

    Zeroed once at allocation: the head-padding columns of the QKV buffer
    (head_dim 8 stored as 16) must stay exactly zero, and rows of padded
    tokens that the plan skips keep whatever an earlier call left -- always
    finite values, so a masked key (P = 0) times its stale V stays 0."""

    def __init__(self, cfg, B: int, S: int, device: torch.device, plan: Plan):
        d, F, H = cfg.d_model, cfg.ffn_dim, cfg.num_heads
        self.dh = d // H
        self.dh_store = max(16, self.dh)
        M = B * S
        f32 = dict(dtype=torch.float32, device=device)
        pl = dict(dtype=torch.int16, device=device)
        split = {g: p == "bf16x3" for g, p in plan.gemm_precisions().items()}
        self.res = torch.zeros(M, d, **f32)
        self.h = torch.zeros(M, d, **f32) if not (split["qkv"] and split["ffn1"]) else None
        self.h2 = torch.zeros(2, M, d, **pl) if (split["qkv"] or split["ffn1"]) else None
        self.qkv = torch.zeros(M, 3 * H * self.dh_store, **f32)
        self.ctx = torch.zeros(2, M, d, **pl) if split["out"] else torch.zeros(M, d, **f32)
        self.y = torch.zeros(M, d, **f32)
        self.ffn = torch.zeros(2, M, F, **pl) if split["ffn2"] else torch.zeros(M, F, **f32)
        words = (S + 31) // 32
        i32 = dict(dtype=torch.int32, device=device)
        self.bits = torch.zeros(B * words, **i32)
        self.live_tiles = torch.zeros((M + 127) // 128, **i32)
        self.live_count = torch.zeros(1, **i32)
        self.order = torch.zeros(B, **i32)
        # Packed row order of the valid tokens for the FFN GEMMs (kf_pack_rows).
        self.row_map = torch.zeros(M, **i32) if plan.packed_ffn else None
        self.row_off = torch.zeros(B + 1, **i32) if plan.packed_ffn else None
        self.packed_tiles = torch.zeros((M + 127) // 128, **i32) if plan.packed_ffn else None
        self.packed_count = torch.zeros(1, **i32) if plan.packed_ffn else None
        # Work list of the persistent attention (kf_attn_schedule), built once
        # per forward; zeroed so its counters start at 0.
        self.sched = (torch.zeros(int(_lib.lib().kf_attn_schedule_words(B, H, S)), **i32)
                      if plan.attn_persistent else None)
        # Stream-K GEMMs share one zeroed workspace (partials + counters);
        # the kernels leave its counters zero, and they run one after another.
        sk_bytes = _Workspace.sk_bytes(cfg, M, plan)
        self.sk = torch.zeros(sk_bytes // 4, **i32) if sk_bytes else None

    @staticmethod
    def sk_bytes(cfg, M: int, plan: Plan) -> int:
        """One stream-K workspace for every stream-K GEMM of the plan: the
        largest partial area plus the largest counter area."""
        d, F = cfg.d_model, cfg.ffn_dim
        widths = {"qkv": 3 * d, "out": d, "ffn1": F, "ffn2": d}
        prec = plan.gemm_precisions()
        partials = counters = 0
        for g, n in widths.items():
            if getattr(plan, f"sk_{g}") and prec[g] == "bf16x3":
                bn = getattr(plan, f"bn_{g}") or 128
                tiles = ((M + 127) // 128) * ((n + bn - 1) // bn)
                partials = max(partials, tiles * 2 * 128 * bn * 4)
                counters = max(counters, tiles * 2 * 4)
        # partials at the start, counters at the end (kf_gemm_bf16x3_sk)
        return partials + ((counters + 15) // 16) * 16 + (16 if counters else 0)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size()
                   for t in (self.res, self.h, self.h2, self.qkv, self.ctx, self.y, self.ffn,
                             self.bits, self.live_tiles, self.live_count, self.order,
                             self.sk, self.sched, self.row_map, self.row_off, self.packed_tiles,
                             self.packed_count)
                   if t is not None)

    @staticmethod
    def estimate(cfg, B: int, S: int, plan: Plan) -> int:
        """Bytes __init__ would allocate for (B, S), without allocating."""
        d, F, H = cfg.d_model, cfg.ffn_dim, cfg.num_heads
        dh_store = max(16, d // H)
        M = B * S
        split = {g: p == "bf16x3" for g, p in plan.gemm_precisions().items()}
        per_row = 4 * d                                        # res
        per_row += 0 if (split["qkv"] and split["ffn1"]) else 4 * d   # h
        per_row += 4 * d if (split["qkv"] or split["ffn1"]) else 0    # h2 planes
        per_row += 4 * 3 * H * dh_store + 4 * d + 4 * d + 4 * F       # qkv, ctx, y, ffn
        words = (S + 31) // 32
        sched = 4 * (8 + 2 * B * H * ((S + 127) // 128)) if plan.attn_persistent else 0
        packed = (4 * M + 4 * (B + 1) + 4 * ((M + 127) // 128) + 4) if plan.packed_ffn else 0
        return (M * per_row + 4 * B * words + 4 * B + 4 * ((M + 127) // 128) + 4
                + _Workspace.sk_bytes(cfg, M, plan) + sched + packed)


class FusedTransformer(LayerStack):
    """Drop-in for BaselineTransformer (identical state_dict keys).

    `forward(x, valid_token_mask=None) -> Tensor[B, S, d]` with x fp32 on an
    sm_100 GPU and valid_token_mask bool [B, S] (True = real token).
    """

    def __init__(self, config, plan: Optional[Plan] = None,
                 memory_budget_bytes: Optional[int] = None):
        super().__init__(config)
        self.plan = plan or DEFAULT_PLAN
        # Device bytes one forward may use for its workspace and its input /
        # output staging; a batch that needs more runs in slices of whole
        # sequences (no op mixes batch elements, so slicing is exact).
        # None = 90% of the device memory free at the first call of a shape.
        self.memory_budget_bytes = memory_budget_bytes
        self._slice_rows: Dict[Tuple, int] = {}
        self._weights: Optional[_Weights] = None
        self._weights_key = None
        self._workspaces: Dict[Tuple, _Workspace] = {}
        self._graphs: Dict[Tuple, "GraphRunner"] = {}
        self.launches_per_forward = 0

    # ------------------------------------------------------------ preparation

    def _param_key(self, device) -> tuple:
        # Parameter storage identity; call invalidate() after editing weights
        # in place (inference tensors carry no version counter to watch).
        return (str(device),) + tuple(p.data_ptr() for p in self.parameters())

    def invalidate(self) -> None:
        """Drop prepared weights and captured graphs (after in-place edits)."""
        self._weights = None
        self._weights_key = None
        self._graphs.clear()

    def prepare(self, device: torch.device) -> _Weights:
        key = self._param_key(device)
        if self._weights is None or self._weights_key != key:
            self._weights = _Weights(self, device, self.plan)
            self._weights_key = key
            self._graphs.clear()
        return self._weights

    def workspace(self, B: int, S: int, device: torch.device) -> _Workspace:
        key = (B, S, str(device))
        ws = self._workspaces.get(key)
        if ws is None:
            ws = _Workspace(self.config, B, S, device, self.plan)
            self._workspaces[key] = ws
        return ws

    def release_buffers(self) -> None:
        self._graphs.clear()
        self._workspaces.clear()
        self._slice_rows.clear()

    # ------------------------------------------------------------ the forward

    def _check_inputs(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> None:
        cfg = self.config
        if x.dim() != 3 or x.shape[-1] != cfg.d_model:
            raise ValueError(f"x must be [B, S, {cfg.d_model}], got {tuple(x.shape)}")
        if x.dtype != torch.float32:
            raise TypeError("only float32 I/O is implemented")
        if not x.is_cuda:
            raise RuntimeError("FusedTransformer runs on an sm_100 GPU only (no CPU path)")
        if mask is not None and tuple(mask.shape) != tuple(x.shape[:2]):
            raise ValueError("valid_token_mask must be [B, S]")
        if cfg.d_model // cfg.num_heads not in SUPPORTED_HEAD_DIMS:
            raise RuntimeError(f"head_dim {cfg.d_model // cfg.num_heads} unsupported")

    def launch(self, x: torch.Tensor, keep_u8: Optional[torch.Tensor], out: torch.Tensor,
               ws: _Workspace, w: _Weights, timer=None) -> int:
        """Issue the whole forward on the current stream; returns launches.

        `timer(kind) -> (start_event, end_event)`, when given, brackets every
        launch with CUDA events (used for the live per-kernel breakdown)."""
        cfg, plan = self.config, self.plan
        B, S, d = x.shape
        M, H, F = B * S, cfg.num_heads, cfg.ffn_dim
        dh, dhs = ws.dh, ws.dh_store
        L = _lib.lib()
        st = _lib.stream_ptr()
        R = plan.round_tf32
        P = _lib.GEMM_PRECISION_FLAGS
        prec = plan.gemm_precisions()
        split = {g: p == "bf16x3" for g, p in prec.items()}
        keep = keep_u8.data_ptr() if keep_u8 is not None else None
        bits = ws.bits.data_ptr() if keep_u8 is not None else None
        # Padded rows: GEMMs compute only 128-row tiles holding a real token
        # and the (non-final) norms leave padded rows alone.
        skip_rows = keep_u8 is not None and plan.skip_padded_rows
        lt = lt0 = ws.live_tiles.data_ptr() if skip_rows else None
        lc = lc0 = ws.live_count.data_ptr() if skip_rows else None
        # FFN over packed rows: a token's row in h_ffn1, ffn and FFN2's y is
        # its rank among the batch's valid tokens (map built below).
        pack = (keep is not None and plan.packed_ffn and split["ffn1"] and split["ffn2"])
        rmap = ws.row_map.data_ptr() if pack else None
        ptiles = (ws.packed_tiles.data_ptr(), ws.packed_count.data_ptr()) if pack else None
        # keep, gamma and beta are static for the forward (inputs copied and
        # weights synchronised before it starts): the norms load them before
        # waiting for the previous kernel.
        ln_static = _lib.KF_LN_STATIC_PARAMS if w.static else 0
        ln_skip = (_lib.KF_LN_SKIP_PADDED if skip_rows else 0) | ln_static

        # Producer output formats follow their consumer's precision: bf16
        # hi/lo planes for "bf16x3", TF32-rounded fp32 for "tf32" (the tensor
        # core would truncate those bits), plain fp32 for "3xtf32".
        def ln_out(consumer):
            if split[consumer]:
                return ws.h2.data_ptr(), _lib.KF_LN_OUT_BF16X2 | ln_skip
            rnd = _lib.KF_LN_ROUND_TF32 if (R and prec[consumer] == "tf32") else 0
            return ws.h.data_ptr(), rnd | ln_skip

        h_qkv, f_ln1 = ln_out("qkv")
        h_ffn1, f_ln2 = ln_out("ffn1")
        attn_flags = (_lib.KF_ATTN_CAUSAL if cfg.causal else 0)
        if split["out"]:
            attn_flags |= _lib.KF_ATTN_OUT_BF16X2
        elif R and prec["out"] == "tf32":
            attn_flags |= _lib.KF_ATTN_ROUND_TF32
        if keep_u8 is not None and plan.skip_empty_queries:
            attn_flags |= _lib.KF_ATTN_SKIP_EMPTY_Q
        res, y, qkv = ws.res.data_ptr(), ws.y.data_ptr(), ws.qkv.data_ptr()
        ctx, ffn = ws.ctx.data_ptr(), ws.ffn.data_ptr()
        ldq = 3 * H * dhs
        hd, hs = (dh, dhs) if dhs != dh else (0, 0)
        n = 0

        def run(kind, fn, *a):
            nonlocal n
            if timer is not None:
                ev0, ev1 = timer(kind)
                ev0.record()
            _lib.check(fn(*a), fn.__name__)
            if timer is not None:
                ev1.record()
            n += 1

        def gemm(kind, g, A, lda, W, bias, C, ldc, N, K, epi, flags, bn, hd_=0, hs_=0,
                 tiles=None):
            lt, lc = tiles if tiles is not None else (lt0, lc0)
            if split[g]:
                if getattr(plan, f"sk_{g}"):
                    run(kind, L.kf_gemm_bf16x3_sk, A, lda, W.data_ptr(), K, bias.data_ptr(), C,
                        ldc, M, N, K, epi, flags, bn or 128, hd_, hs_, lt, lc,
                        ws.sk.data_ptr(), ws.sk.numel() * 4, st)
                    return
                if getattr(plan, f"pair_{g}") and bn in (128, 256):
                    flags |= _lib.KF_GEMM_PAIR
                elif w.static:
                    flags |= _lib.KF_GEMM_W_STATIC
                run(kind, L.kf_gemm_bf16x3, A, lda, W.data_ptr(), K, bias.data_ptr(), C, ldc,
                    M, N, K, epi, flags, bn, hd_, hs_, lt, lc, st)
            else:
                run(kind, L.kf_gemm_tf32, A, lda, W.data_ptr(), K, bias.data_ptr(), C, ldc, M,
                    N, K, epi, flags | P[prec[g]], bn, hd_, hs_, lt, lc, st)

        if keep is not None:
            run("keep_bits", L.kf_keep_bits, keep, S, B, S, bits, st)
        if pack:
            run("keep_bits", L.kf_pack_rows, bits, B, S, rmap, ws.row_off.data_ptr(), ptiles[0],
                ptiles[1], st)
        if skip_rows:
            run("keep_bits", L.kf_live_row_tiles, keep, M, lt, lc, st)
        sched = ws.sched.data_ptr() if plan.attn_persistent else None
        order = (ws.order.data_ptr() if (sched is None and keep is not None and plan.order_rows
                                         and B > 1) else None)
        if order is not None:
            run("keep_bits", L.kf_batch_order, bits, B, S, order, st)
        if sched is not None:
            run("keep_bits", L.kf_attn_schedule, bits, B, H, S, sched, st)
            if keep is not None and plan.skip_empty_queries:
                # rows of query tiles without a valid query are padding: not written
                attn_flags = (attn_flags & ~_lib.KF_ATTN_SKIP_EMPTY_Q) | _lib.KF_ATTN_EMPTY_Q_UNTOUCHED
        l0 = w.layers[0]
        run("ln", L.kf_ln_add_mask, x.data_ptr(), d, None, 0, keep, l0["ln1w"].data_ptr(),
            l0["ln1b"].data_ptr(), res, d, h_qkv, d, M, d, l0["eps1"], f_ln1, st)
        nl = len(w.layers)
        f_ffn1_out = _lib.KF_GEMM_OUT_BF16X2 if split["ffn2"] else (
            _lib.KF_GEMM_ROUND_TF32 if (R and prec["ffn2"] == "tf32") else 0)
        for i, lw in enumerate(w.layers):
            gemm("qkv", "qkv", h_qkv, d, lw["wqkv"], lw["bqkv"], qkv, ldq, 3 * d, d,
                 _lib.KF_EPI_BIAS, _lib.KF_GEMM_ROUND_TF32 if R else 0, plan.bn_qkv, hd, hs)
            if sched is not None:
                run("attention", L.kf_flash_fwd_tf32_sched, qkv, S * ldq, dhs, ldq,
                    qkv + 4 * H * dhs, S * ldq, dhs, ldq, qkv + 8 * H * dhs, S * ldq, dhs,
                    ldq, ctx, S * d, dh, d, bits, sched, B, H, S, dhs, dh, dh ** -0.5,
                    attn_flags, st)
            elif order is not None:
                run("attention", L.kf_flash_fwd_tf32_ordered, qkv, S * ldq, dhs, ldq,
                    qkv + 4 * H * dhs, S * ldq, dhs, ldq, qkv + 8 * H * dhs, S * ldq, dhs,
                    ldq, ctx, S * d, dh, d, bits, order, B, H, S, dhs, dh, dh ** -0.5,
                    attn_flags, st)
            else:
                run("attention", L.kf_flash_fwd_tf32, qkv, S * ldq, dhs, ldq,
                    qkv + 4 * H * dhs, S * ldq, dhs, ldq, qkv + 8 * H * dhs, S * ldq, dhs,
                    ldq, ctx, S * d, dh, d, bits, B, H, S, dhs, dh, dh ** -0.5, attn_flags, st)
            # out_proj, then the residual add + mask + LN2 (its output at the
            # tokens' packed rows when the FFN runs packed).
            gemm("out_proj", "out", ctx, d, lw["wo"], lw["bo"], y, d, d, d,
                 _lib.KF_EPI_BIAS, 0, plan.bn_out)
            if pack:
                run("ln", L.kf_ln_add_mask_rows, res, d, y, d, keep, lw["ln2w"].data_ptr(),
                    lw["ln2b"].data_ptr(), res, d, h_ffn1, d, M, d, lw["eps2"],
                    f_ln2 | _lib.KF_LN_H_MAPPED, rmap, st)
            else:
                run("ln", L.kf_ln_add_mask, res, d, y, d, keep, lw["ln2w"].data_ptr(),
                    lw["ln2b"].data_ptr(), res, d, h_ffn1, d, M, d, lw["eps2"], f_ln2, st)
            gemm("ffn1", "ffn1", h_ffn1, d, lw["w1"], lw["b1"], ffn, F, F, d,
                 _lib.KF_EPI_BIAS_GELU, f_ffn1_out, plan.bn_ffn1, tiles=ptiles)
            # FFN2, then the next layer's LN1 (or the final norm).
            if i == nl - 1:
                nw, nb, ne = w.finw.data_ptr(), w.finb.data_ptr(), w.fin_eps
                s_out, h_out, f_next = None, out.data_ptr(), _lib.KF_LN_MASK_OUT | ln_static
            else:
                nx = w.layers[i + 1]
                nw, nb, ne = nx["ln1w"].data_ptr(), nx["ln1b"].data_ptr(), nx["eps1"]
                s_out, h_out, f_next = res, h_qkv, f_ln1
            gemm("ffn2", "ffn2", ffn, F, lw["w2"], lw["b2"], y, d, d, F, _lib.KF_EPI_BIAS, 0,
                 plan.bn_ffn2, tiles=ptiles)
            if pack:
                run("ln", L.kf_ln_add_mask_rows, res, d, y, d, keep, nw, nb, s_out, d, h_out, d,
                    M, d, ne, f_next | _lib.KF_LN_Y_MAPPED, rmap, st)
            else:
                run("ln", L.kf_ln_add_mask, res, d, y, d, keep, nw, nb, s_out, d, h_out, d, M, d,
                    ne, f_next, st)
        self.launches_per_forward = n
        return n

    @staticmethod
    def _keep_u8(mask: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
        if mask is None:
            return None
        if mask.dtype == torch.bool:
            return mask.contiguous().view(torch.uint8)
        return (mask != 0).to(torch.uint8).contiguous()

    def eager_forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None,
                      out: Optional[torch.Tensor] = None) -> torch.Tensor:
        self._check_inputs(x, valid_token_mask)
        x = x.contiguous()
        w = self.prepare(x.device)
        B, S, d = x.shape
        ws = self.workspace(B, S, x.device)
        out = torch.empty_like(x) if out is None else out
        self.launch(x, self._keep_u8(valid_token_mask), out, ws, w)
        return out

    def bytes_per_sequence(self, S: int) -> int:
        """Device bytes one sequence of length S costs a forward: its share of
        the workspace plus the graph's static input and output and the
        returned copy (3 x S x d fp32)."""
        return (_Workspace.estimate(self.config, 1, S, self.plan)
                + 3 * 4 * S * self.config.d_model)

    def slice_rows(self, B: int, S: int, device: torch.device) -> int:
        """Sequences per slice for a [B, S] batch under the memory budget
        (decided once per shape and device)."""
        key = (B, S, str(device))
        rows = self._slice_rows.get(key)
        if rows is None:
            budget = self.memory_budget_bytes
            if budget is None:
                free, _ = torch.cuda.mem_get_info(device)
                budget = int(0.9 * free) + sum(
                    w.nbytes() for k, w in self._workspaces.items() if k[2] == str(device))
            rows = max(1, min(B, budget // max(1, self.bytes_per_sequence(S))))
            self._slice_rows[key] = rows
        return rows

    def _forward_whole(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]
                       ) -> torch.Tensor:
        if self.plan.cuda_graph and not torch.cuda.is_current_stream_capturing():
            return self.graph_runner(x, valid_token_mask)(x, valid_token_mask)
        return self.eager_forward(x, valid_token_mask)

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None
                ) -> torch.Tensor:
        self._check_inputs(x, valid_token_mask)
        B, S, _ = x.shape
        rows = self.slice_rows(B, S, x.device) if B > 1 else 1
        if rows >= B:
            return self._forward_whole(x, valid_token_mask)
        # Batch streaming: whole sequences per slice, results written into
        # one output (at most two captured graphs: full slices and the rest).
        out = torch.empty_like(x)
        for b0 in range(0, B, rows):
            b1 = min(B, b0 + rows)
            m = None if valid_token_mask is None else valid_token_mask[b0:b1]
            out[b0:b1].copy_(self._forward_whole(x[b0:b1], m))
        return out

    def graph_runner(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor]
                     ) -> "GraphRunner":
        key = (tuple(x.shape), str(x.device), valid_token_mask is None)
        runner = self._graphs.get(key)
        if runner is None:
            runner = GraphRunner(self, x, valid_token_mask)
            self._graphs[key] = runner
        return runner


class GraphRunner:
    """One CUDA graph holding the whole multi-layer forward for a fixed shape.

    Inputs are copied into static device buffers, the graph is replayed, and
    the output is cloned (the next replay overwrites the static output, and
    callers legitimately hold results)."""

    def __init__(self, model: FusedTransformer, x: torch.Tensor,
                 mask: Optional[torch.Tensor], out: Optional[torch.Tensor] = None,
                 ws: Optional["_Workspace"] = None):
        """With `out` given, x, mask and out themselves are the graph's
        buffers (no copies: the caller writes inputs into x and mask and reads
        results from out; mask must then be a contiguous bool tensor, read
        as bytes in place), and `ws` may be a workspace shared with other
        runners that never run at the same time."""
        self.model = model
        B, S, d = x.shape
        if out is None:
            self.static_x = x.detach().clone().contiguous()
            self.static_keep = None if mask is None else model._keep_u8(mask).clone()
            self.static_out = torch.empty_like(self.static_x)
        else:
            if not (x.is_contiguous() and out.is_contiguous() and out.shape == x.shape
                    and out.dtype == x.dtype and out.device == x.device):
                raise ValueError("bound buffers must be contiguous tensors of one shape")
            if mask is not None and (mask.dtype != torch.bool or not mask.is_contiguous()):
                raise ValueError("a bound mask must be a contiguous bool tensor")
            self.static_x = x
            self.static_keep = None if mask is None else model._keep_u8(mask)
            self.static_out = out
        self.weights = model.prepare(x.device)
        # A workspace of its own unless shared: eager calls of other shapes
        # never alias it.
        self.ws = ws if ws is not None else _Workspace(model.config, B, S, x.device, model.plan)
        side = torch.cuda.Stream(device=x.device)
        side.wait_stream(torch.cuda.current_stream(x.device))
        with torch.cuda.stream(side):
            # Warm-up outside capture: sets kernel attributes, checks arguments.
            self.launches = model.launch(self.static_x, self.static_keep, self.static_out,
                                         self.ws, self.weights)
        torch.cuda.current_stream(x.device).wait_stream(side)
        torch.cuda.synchronize(x.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            model.launch(self.static_x, self.static_keep, self.static_out, self.ws,
                         self.weights)

    def load_inputs(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> None:
        self.static_x.copy_(x, non_blocking=True)
        if self.static_keep is not None and mask is not None:
            self.static_keep.copy_(FusedTransformer._keep_u8(mask), non_blocking=True)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.static_out

    def __call__(self, x: torch.Tensor, mask: Optional[torch.Tensor]) -> torch.Tensor:
        self.load_inputs(x, mask)
        return self.replay().clone()
