/*
 * kf_sm100.h -- C ABI of the B200 (sm_100a) layer-stack forward library.
 *
 * The library implements the hot path of the pre-norm Transformer stack of
 * torch_transformer_benchmark.py (BaselineTransformer, :125-172) as four
 * kernels: a fused residual-add + padding-mask + LayerNorm, a tcgen05 TF32
 * GEMM with bias / bias+GELU(erf) epilogues, a key-padding bit packer and a
 * tcgen05 TF32 FlashAttention forward with in-register causal and key-padding
 * masks.
 *
 * Conventions shared by every entry point:
 *   - all pointers are device pointers owned by the caller (the library never
 *     allocates, frees or synchronises on the hot path; every call is
 *     stream-ordered on `stream`, a cudaStream_t, and may be captured in a CUDA
 *     graph);
 *   - strides and leading dimensions are in ELEMENTS, not bytes;
 *   - the return value is KF_OK (0) or a KF_E_* code; kf_last_error() gives the
 *     message of the last failure on the calling thread;
 *   - kernels that spin on barriers give up after a bounded time and record a
 *     device status word, read back (with a device sync) by kf_device_status().
 */
#ifndef KF_SM100_H_
#define KF_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KF_OK 0
#define KF_E_INVALID 1     /* bad argument: null pointer, negative size, bad stride */
#define KF_E_UNSUPPORTED 2 /* valid request outside what the kernels implement */
#define KF_E_CUDA 3        /* a CUDA runtime / driver call failed */
#define KF_E_NO_DEVICE 4   /* no sm_100 device is current */

/* ----------------------------------------------------------- housekeeping */

/* Library ABI version (major * 100 + minor). */
int kf_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* kf_last_error(void);

/* Reads the device-side status word of the current device (synchronises the
 * device). 0 = no kernel has failed since the last reset; otherwise the code
 * of the first failure: 1-4 a bounded wait gave up (1 TMA producer, 2 MMA
 * issuer, 3 GEMM epilogue, 4 attention softmax), 5 an ordered attention
 * call got a batch_order entry outside [0, B). `reset` != 0 clears it. */
int kf_device_status(int reset);

/* The same status word copied into host_dst (pinned host memory, one int32)
 * by a copy queued on `stream`, without synchronising: it holds the status
 * once that stream reaches the copy. Lets a caller check the library's health
 * after each call at no cost to the call (submission.py reads it one call
 * later and falls back when it is nonzero). */
int kf_device_status_async(int32_t* host_dst, void* stream);

/* Time limit of every bounded wait of the current device's kernels, in SM
 * cycles (synchronous; takes effect for later launches). cycles <= 0 restores
 * the default (~2 s). Waits that drain in-flight copies while a CTA unwinds
 * keep the default, so a short limit only makes a stuck wait give up sooner.
 * For tests of the failure path: a real wait takes microseconds. */
int kf_set_wait_limit(int64_t cycles);

/* ----------------------------------------------------------- LayerNorm */

#define KF_LN_MASK_OUT 1   /* zero h on rows whose keep byte is 0 (final norm) */
#define KF_LN_ROUND_TF32 2 /* round h to TF32 (it only feeds a TF32 GEMM) */
#define KF_LN_SKIP_PADDED 4 /* leave s and h of padded rows untouched (valid
                               only when every consumer masks those rows) */
#define KF_LN_OUT_BF16X2 8  /* write h as bf16 hi/lo planes: h_out is then a
                               uint16 [2][M][ldh] buffer (kf_gemm_bf16x3 input) */
#define KF_LN_STATIC_PARAMS 16 /* keep, w and b (and row_map) were written before the
                                  kernel that precedes this call in the stream started:
                                  they are loaded before waiting for that kernel */
#define KF_LN_Y_MAPPED 32 /* kf_ln_add_mask_rows: y of row r is row row_map[r] of y */
#define KF_LN_H_MAPPED 64 /* kf_ln_add_mask_rows: h of row r goes to row row_map[r] */

/* Fused residual-add + row mask + LayerNorm over rows of width d:
 *     s = keep[r] ? x[r] + y[r] : 0          (y optional, keep optional)
 *     h = (s - mean(s)) / sqrt(var_biased(s) + eps) * w + b
 *     h = (MASK_OUT && !keep[r]) ? 0 : h
 * s_out is written when non-null. fp32 in and out.
 * Replaces kernelforge/ops/layernorm.py:101-156 (add_mask_layernorm) and its
 * Triton kernel _add_mask_ln_kernel (layernorm.py:40-86); semantics of
 * torch_transformer_benchmark.py:128,140-144,169-171. */
int kf_ln_add_mask(const float* x, int64_t ldx, const float* y, int64_t ldy, const uint8_t* keep,
                   const float* w, const float* b, float* s_out, int64_t lds, float* h_out,
                   int64_t ldh, int64_t M, int64_t d, float eps, int flags, void* stream);

/* kf_ln_add_mask with y and / or h in a packed row order: row_map[r] (int32,
 * M entries, e.g. from kf_pack_rows) is the row of y read for row r
 * (KF_LN_Y_MAPPED) and the row of h written for it (KF_LN_H_MAPPED); an entry
 * of -1 means row r has no y (s = keep ? x : 0) and writes no h. x, keep and
 * s_out stay in the unpacked order; h's bf16 planes keep the stride M * ldh.
 * The arithmetic of every row is that of kf_ln_add_mask. Lets the FFN GEMMs
 * run over valid tokens only (no reference counterpart: the reference keeps
 * the padded layout, kernelforge/optimized.py:441-446). */
int kf_ln_add_mask_rows(const float* x, int64_t ldx, const float* y, int64_t ldy,
                        const uint8_t* keep, const float* w, const float* b, float* s_out,
                        int64_t lds, float* h_out, int64_t ldh, int64_t M, int64_t d, float eps,
                        int flags, const int32_t* row_map, void* stream);

/* Packed row order of the valid tokens of a [B, S] key mask (its kf_keep_bits
 * words): row_map[b*S + s] = the rank of token (b, s) among all valid tokens
 * in row-major order, or -1 for a padded one; row_off[0..B] the prefix sums
 * of the rows' valid counts (row_off[B] = T); tiles[i] = i for the
 * ceil(T / 128) 128-row tiles that hold packed rows, *tile_count that number
 * (the live_tiles / live_count form of the GEMMs). row_map holds B*S int32,
 * row_off B+1, tiles ceil(B*S/128). B <= 65535. Two small kernels. No
 * reference counterpart (see kf_ln_add_mask_rows). */
int kf_pack_rows(const uint32_t* bits, int64_t B, int64_t S, int32_t* row_map, int32_t* row_off,
                 int32_t* tiles, int32_t* tile_count, void* stream);

/* ----------------------------------------------------------- GEMM */

#define KF_EPI_BIAS 0      /* C = A W^T + bias */
#define KF_EPI_BIAS_GELU 1 /* C = gelu_erf(A W^T + bias) */

#define KF_GEMM_ROUND_TF32 1 /* round C to TF32 (it only feeds a TF32 MMA) */
#define KF_GEMM_SPLIT3 2     /* error-compensated 3xTF32: hi*hi + hi*lo + lo*hi
                                (~2^-20 relative, 3 TF32 MMAs per k step) */
#define KF_GEMM_BF16X3 4     /* error-compensated BF16x3: bf16 hi/lo split of the
                                fp32 operands, hi*hi + hi*lo + lo*hi on the BF16
                                tensor path (~2^-17 relative, 1.5x one TF32
                                pass); exclusive with KF_GEMM_SPLIT3 */

/* Compact list of the 128-row tiles of an [M] keep-byte vector that hold at
 * least one nonzero byte: tiles[0..*count) in ascending order. `tiles` needs
 * ceil(M/128) entries. Feeds kf_gemm_tf32's live-tile schedule. */
int kf_live_row_tiles(const uint8_t* keep, int64_t M, int32_t* tiles, int32_t* count,
                      void* stream);

/* C[M,N] = epilogue(A[M,K] . W[N,K]^T + bias[N]) on tcgen05 TF32 tensor cores
 * with an FP32 TMEM accumulator (nn.Linear layout: W row-major [N,K]).
 * flags: KF_GEMM_ROUND_TF32 | (KF_GEMM_SPLIT3 or KF_GEMM_BF16X3).
 * `bias` may be null. Requires K % 4 == 0, lda/ldw % 4 == 0 and 16-byte
 * aligned A/W (TMA constraints). `bn` selects the N tile (0 = automatic,
 * 64/128/256). When head_dim > 0, output column n is written to column
 * (n / head_dim) * head_stride + n % head_dim of its row (used to zero-pad
 * head_dim 8 to 16 for the attention MMA); columns never written keep their
 * contents. live_tiles/live_count (both null, or both device pointers from
 * kf_live_row_tiles): compute only those 128-row tiles; rows of other tiles
 * keep their contents.
 * Replaces the cuBLAS F.linear calls of kernelforge/optimized.py:441-446
 * (FFN1 + F.gelu, FFN2), :483 (fused QKV) and :573 (out_proj). */
int kf_gemm_tf32(const float* A, int64_t lda, const float* W, int64_t ldw, const float* bias,
                 float* C, int64_t ldc, int64_t M, int64_t N, int64_t K, int epilogue, int flags,
                 int bn, int head_dim, int head_stride, const int32_t* live_tiles,
                 const int32_t* live_count, void* stream);

#define KF_GEMM_OUT_BF16X2 8 /* kf_gemm_bf16x3: write C as bf16 hi/lo planes */
#define KF_GEMM_W_STATIC 64  /* kf_gemm_bf16x3: W was written before the kernel that
                                precedes this call in the stream started (weights
                                prepared once), so the first W tiles may be loaded
                                before waiting for that kernel; one-CTA tiles only */
#define KF_GEMM_PAIR 32      /* kf_gemm_bf16x3: 256 x bn tiles on CTA pairs
                                (tcgen05 cta_group::2; bn 128 or 256): each SM
                                stages its 128 A rows and half of the B rows, so
                                shared-memory operand traffic per product drops
                                by a third (bn 256); same accumulation order */

/* Error-compensated GEMM on operands already split into bf16 planes:
 * A2 = [2][M][lda] (hi plane, then lo plane, with hi + lo = the fp32 value to
 * ~2^-17), W2 = [2][N][ldw] likewise; C = epilogue(A.W^T + bias) computed as
 * hi(A)hi(W) + hi(A)lo(W) + lo(A)hi(W) on the BF16 tensor path with an FP32
 * TMEM accumulator. C is fp32 [M][ldc], or with KF_GEMM_OUT_BF16X2 bf16
 * planes [2][M][ldc] in the same split format (to feed another
 * kf_gemm_bf16x3). Needs K, lda, ldw % 8 == 0 and 16-byte aligned pointers.
 * head_dim/head_stride (fp32 output only) and live_tiles/live_count as
 * kf_gemm_tf32; `bn` as kf_gemm_tf32 plus 96 (fewer partial waves when
 * N / 128 tiles leave the last wave nearly empty). Replaces the same F.linear calls
 * as kf_gemm_tf32, at fp32-class accuracy. */
int kf_gemm_bf16x3(const uint16_t* A2, int64_t lda, const uint16_t* W2, int64_t ldw,
                   const float* bias, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                   int epilogue, int flags, int bn, int head_dim, int head_stride,
                   const int32_t* live_tiles, const int32_t* live_count, void* stream);

/* kf_gemm_bf16x3 with stream-K scheduling: one CTA per SM, each computing an
 * even share of all (tile, k block) pairs, so a GEMM with fewer tiles than
 * SMs (or a ragged last wave) still keeps every SM busy for a share of the
 * K loop. A tile split between CTAs is finished by the CTA holding its first
 * k blocks, which adds the other parts (fp32, in a fixed order: results are
 * deterministic, not bit-identical to kf_gemm_bf16x3). `bn` 64, 128 or 256
 * (0 = 128), no KF_GEMM_PAIR. `workspace`: at least
 * kf_gemm_sk_workspace_bytes(M, N, bn) bytes, 16-byte aligned, ZEROED before
 * its first use (the kernel leaves its counters zero again); partials go at
 * its start and the per-tile counters at its end, so GEMMs of several shapes
 * can share one buffer of max(partial bytes) + max(counter bytes); calls
 * sharing it must not overlap on the GPU. Replaces the same F.linear calls as kf_gemm_bf16x3
 * (kernelforge/optimized.py:441-446, 573). */
int kf_gemm_bf16x3_sk(const uint16_t* A2, int64_t lda, const uint16_t* W2, int64_t ldw,
                      const float* bias, void* C, int64_t ldc, int64_t M, int64_t N, int64_t K,
                      int epilogue, int flags, int bn, int head_dim, int head_stride,
                      const int32_t* live_tiles, const int32_t* live_count, void* workspace,
                      int64_t workspace_bytes, void* stream);
int64_t kf_gemm_sk_workspace_bytes(int64_t M, int64_t N, int bn);

/* ----------------------------------------------------------- attention */

/* Words of the packed key-validity workspace for a [B, S] keep mask. */
size_t kf_keep_bits_words(int64_t B, int64_t S);

/* Pack a uint8 keep mask [B, S] (row stride ld_keep) into bits[B][ceil(S/32)]
 * (bit k%32 of word k/32 = keep[b][k] != 0; bits past S are 0). This is the
 * caller-owned workspace kf_flash_fwd_tf32 reads. */
int kf_keep_bits(const uint8_t* keep, int64_t ld_keep, int64_t B, int64_t S, uint32_t* bits,
                 void* stream);

#define KF_ATTN_CAUSAL 1      /* mask keys after the query (triu(1) = -inf) */
#define KF_ATTN_SKIP_EMPTY_Q 2 /* write 0 for query tiles with no valid query
                                  (valid only when the caller masks those rows
                                  afterwards, as the layer stack does) */
#define KF_ATTN_ROUND_TF32 4  /* round O to TF32 (it only feeds a TF32 GEMM) */
#define KF_ATTN_OUT_BF16X2 8  /* write O as bf16 hi/lo planes: o is then a uint16
                                 buffer with the given strides (in bf16
                                 elements), lo plane B * o_sb elements after
                                 the hi plane (kf_gemm_bf16x3 input) */

/* O = softmax(Q K^T * sm_scale + causal(-inf) + keypad(-inf)) V per (b, h),
 * softmax in fp32, TF32 tensor-core contractions, FP32 accumulation in TMEM.
 * Q/K/V/O are strided [B, H, S, Dh] views with unit stride on Dh and the
 * other strides given as (batch, head, row) in elements (multiples of 4).
 * `dh` is the stored head width of Q/K/V (16, 32, 64, 128 or 256), `dh_out`
 * the number of O columns written (<= dh; dh_out < dh means Q/K/V carry
 * zero padding up to dh). keep_bits may be null (no key mask) or a
 * kf_keep_bits workspace. KV tiles without a valid key are skipped; a query
 * row with no valid key yields 0, not NaN.
 * Replaces kernelforge/ops/flash.py:363-422 (flash_attention) and its Triton
 * kernel _flash_fwd_kernel (flash.py:41-249); semantics of
 * torch_transformer_benchmark.py:97-112. */
int kf_flash_fwd_tf32(const float* q, int64_t q_sb, int64_t q_sh, int64_t q_sm, const float* k,
                      int64_t k_sb, int64_t k_sh, int64_t k_sm, const float* v, int64_t v_sb,
                      int64_t v_sh, int64_t v_sm, float* o, int64_t o_sb, int64_t o_sh,
                      int64_t o_sm, const uint32_t* keep_bits, int64_t B, int64_t H, int64_t S,
                      int dh, int dh_out, float sm_scale, int flags, void* stream);

/* Batch rows of a kf_keep_bits workspace ranked by valid-key count, longest
 * first (ties by row index): order[rank] = b, order holding B int32. One
 * CTA; batches of more than 4096 rows get the identity order. No reference
 * counterpart (the reference's Triton grid runs rows in batch order). */
int kf_batch_order(const uint32_t* bits, int64_t B, int64_t S, int32_t* order, void* stream);

/* kf_flash_fwd_tf32 with the grid's batch rows taken in the order of
 * batch_order (a kf_batch_order result written by an earlier kernel in the
 * stream): the longest rows' heavy causal tiles start first, so the launch
 * ends on short rows instead of waiting for a late long one. Results are
 * the same bit for bit as kf_flash_fwd_tf32's; only the schedule changes.
 * batch_order must be a permutation of [0, B) (kf_batch_order's output for
 * the same B and key bits); an entry outside [0, B) is not used as an index
 * -- that grid row runs its own batch row -- and sets device status 5.
 * Stands in for the same reference call as kf_flash_fwd_tf32
 * (kernelforge/ops/flash.py:363-422). */
int kf_flash_fwd_tf32_ordered(const float* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                              const float* k, int64_t k_sb, int64_t k_sh, int64_t k_sm,
                              const float* v, int64_t v_sb, int64_t v_sh, int64_t v_sm, float* o,
                              int64_t o_sb, int64_t o_sh, int64_t o_sm, const uint32_t* keep_bits,
                              const int32_t* batch_order, int64_t B, int64_t H, int64_t S, int dh,
                              int dh_out, float sm_scale, int flags, void* stream);

/* ----------------------------------------------------------- persistent attention */

#define KF_ATTN_EMPTY_Q_UNTOUCHED 16 /* kf_flash_fwd_tf32_sched: leave the rows of
                                        query tiles without a valid query as they
                                        are (no work at all for those tiles) */

/* int32 words of a kf_attn_schedule work list for [B, S] rows of H heads:
 * 8 header words plus two per (row, head, 128-query tile). */
size_t kf_attn_schedule_words(int64_t B, int64_t H, int64_t S);

/* Builds the work list of kf_flash_fwd_tf32_sched from a kf_keep_bits
 * workspace (keep_bits may be null: every key valid) in `sched`
 * (kf_attn_schedule_words int32 words, caller-owned, 8-byte aligned). One item per (row,
 * head, 128-query tile): the rows by valid length, longest first, their heads
 * in order, and within a head the query tiles that hold a valid query from
 * the last to the first (the heaviest under the causal mask first); the tiles
 * without a valid query come after all of those. Also zeroes the list's two
 * counters. One CTA; B <= 16384 and B * H <= 65535. The list depends only on
 * the key bits, so one list serves every layer of a forward. No reference
 * counterpart (the reference's grid runs every query tile in grid order,
 * kernelforge/ops/flash.py:397). */
int kf_attn_schedule(const uint32_t* keep_bits, int64_t B, int64_t H, int64_t S,
                     int32_t* sched, void* stream);

/* kf_flash_fwd_tf32 as a persistent kernel over a kf_attn_schedule list for
 * the same keep_bits, B, H and S: as many CTAs as fit on the GPU take items
 * from the list with an atomic counter in its header until it is exhausted,
 * keeping their barriers, TMEM and pipelines across items (the next item's Q
 * loads while the current one drains). Per query row the arithmetic is the
 * same as kf_flash_fwd_tf32's, so the output is bit-identical for the same
 * flags; with KF_ATTN_EMPTY_Q_UNTOUCHED the rows of query tiles without a
 * valid query are not written at all. The list's counters are reset by the
 * kernel's last CTA, so the list can be reused by later calls on the same
 * stream; calls that overlap on the GPU must not share a list.
 * Replaces the same reference call as kf_flash_fwd_tf32
 * (kernelforge/ops/flash.py:363-422). */
int kf_flash_fwd_tf32_sched(const float* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                            const float* k, int64_t k_sb, int64_t k_sh, int64_t k_sm,
                            const float* v, int64_t v_sb, int64_t v_sh, int64_t v_sm, float* o,
                            int64_t o_sb, int64_t o_sh, int64_t o_sm, const uint32_t* keep_bits,
                            int32_t* sched, int64_t B, int64_t H, int64_t S, int dh, int dh_out,
                            float sm_scale, int flags, void* stream);

/* ----------------------------------------------------------- no-allocation variant */

/* Capacity of the library's static key-bit scratch: 1 MiB per device. */
#define KF_NOALLOC_KEEP_WORDS_MAX 262144

/* kf_flash_fwd_tf32 for callers that cannot allocate device memory: serving
 * processes whose GPU memory is all in a fixed arena they cannot grow,
 * latency-bound paths that cannot take the device-wide synchronisation of
 * cudaMalloc/cudaFree, and FFI callers with no device allocator. It takes the
 * uint8 keep mask [B, S] (row stride ld_keep, required) instead of a
 * kf_keep_bits workspace and packs the key bits into a static device array of
 * the library (KF_NOALLOC_KEEP_WORDS_MAX words, held on every device that
 * loads the library until exit); it calls no allocator. B * ceil(S/32) above
 * the maximum returns KF_E_UNSUPPORTED, and every argument kf_flash_fwd_tf32
 * would reject is rejected, before any launch. The first call on a device
 * resolves the array's address with cudaGetSymbolAddress: make it before any
 * stream capture. That address is cached per device ordinal until the process
 * exits, so it is stale after a cudaDeviceReset of that device; do not call
 * this entry point on a device again after resetting it. All calls share the array: the packer rewrites
 * every word the kernel reads, so nothing needs clearing, but calls that
 * overlap on the GPU race -- order them on one stream or with events.
 * Other arguments, semantics and results as kf_flash_fwd_tf32.
 * No counterpart in the reference (its flash_attention allocates through
 * PyTorch). */
int kf_flash_fwd_tf32_keep_noalloc(const float* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                                   const float* k, int64_t k_sb, int64_t k_sh, int64_t k_sm,
                                   const float* v, int64_t v_sb, int64_t v_sh, int64_t v_sm,
                                   float* o, int64_t o_sb, int64_t o_sh, int64_t o_sm,
                                   const uint8_t* keep, int64_t ld_keep, int64_t B, int64_t H,
                                   int64_t S, int dh, int dh_out, float sm_scale, int flags,
                                   void* stream);

/* ----------------------------------------------------------- utilities */

/* Split src [rows][ld_src] fp32 into bf16 planes dst2 = [2][rows][ld_dst]
 * (hi = bf16_rn(x), lo = bf16_rn(x - hi)); weight preparation for
 * kf_gemm_bf16x3. */
int kf_split_bf16x2(const float* src, int64_t rows, int64_t cols, int64_t ld_src, uint16_t* dst2,
                    int64_t ld_dst, void* stream);

/* dst[i] = round_to_tf32(src[i]) for n fp32 values (weight preparation). */
int kf_round_tf32(const float* src, float* dst, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KF_SM100_H_ */
