// tcgen05 TF32 GEMM with fused epilogues:  C = epi(A . W^T + bias)
//
// A [M,K] and W [N,K] are both K-major (nn.Linear layout), fp32 in HBM, fed to
// the tensor core as TF32. The kernel is persistent (one CTA per SM, static
// round-robin over 128 x BN output tiles, N-fastest so the CTAs running at one
// time share the same A rows in L2) and warp-specialised:
//
//   warp 0      TMA producer: one elected thread streams 128x32 A and BNx32 W
//               boxes (128-byte rows, 128B swizzle) into a STAGES-deep smem
//               ring, completion tracked by mbarrier transaction counts;
//   warp 1      MMA issuer: allocates TMEM (two BN-column accumulators), one
//               thread issues 4 tcgen05.mma (K = 8 each) per 32-wide k block
//               and releases the smem stage with tcgen05.commit;
//   warps 2-9   epilogue (two halves of four, alternate 32-column chunks): tcgen05.ld the accumulator of a finished tile (warp w
//               owns TMEM lanes 32*(w%4)..+31 = 32 output rows), add bias,
//               optionally GELU(erf) and TF32 rounding, then write each
//               128x32 chunk into a 128B-swizzled shared buffer and store it
//               with one TMA bulk store (two buffers in flight), so global
//               writes are full lines instead of one 16-byte piece per row
//               per thread; then hand the accumulator back to the MMA warp.
//               Double buffering lets the epilogue of tile i overlap the main
//               loop of tile i+1;
//   warps 10-17 (split modes only) converters: once a stage has landed they
//               write a hi/lo split of both fp32 tiles next to them in shared
//               memory, so the MMA warp can issue the error-compensated
//               product  A.B ~= hi(A).hi(B) + hi(A).lo(B) + lo(A).hi(B)
//               with no extra HBM or L2 traffic:
//                 3xTF32: lo = x - trunc_tf32(x) (fp32); hi is the staged tile
//                         itself (the tensor core drops its low 13 bits);
//                         three kind::tf32 MMAs per 8-wide k step, ~2^-20;
//                 BF16x3: hi = bf16_rn(x), lo = bf16_rn(x - hi), written as
//                         64-byte swizzled bf16 rows; three kind::f16 MMAs per
//                         16-wide k step (BF16 issues at twice the TF32 rate,
//                         so 1.5x the cost of one TF32 pass), ~2^-17.
#include <cuda_bf16.h>

#include <cstring>

#include "kf_common.cuh"

namespace kf {

enum : int { KF_GEMM_VEC_OK = 1 << 8, KF_GEMM_TMA_OUT = 1 << 9, KF_GEMM_OUT_SPLIT = 1 << 10 };
// SPLIT_BF16X3_PRE: operands arrive already split into bf16 hi/lo planes
// (kf_gemm_bf16x3); TMA loads the four planes, no converter warps.
enum : int {
  SPLIT_NONE = 0,
  SPLIT_TF32X3 = 1,
  SPLIT_BF16X3 = 2,
  SPLIT_BF16X3_PRE = 3
};

// PAIR: cta_group::2 tiles of 256 x BN computed by a cluster of two CTAs;
// each CTA stages its own 128 A rows and half of the BN B rows, and holds
// the accumulator of its 128 rows (BN columns) in its own TMEM.
template <int BN, int SPLIT, bool PAIR = false>
struct GemmCfg {
  static constexpr int BM = 128;
  // One swizzle row per k block and plane: 128 bytes (32 fp32 or, pre-split,
  // 64 bf16).
  static constexpr int ROW_BYTES = 128;
  static constexpr int BK = SPLIT == SPLIT_BF16X3_PRE ? 64 : 32;
  static constexpr bool PRESPLIT = SPLIT == SPLIT_BF16X3_PRE;
  static constexpr int A_BYTES = BM * ROW_BYTES;  // one plane
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // B rows staged by this CTA
  static constexpr int B_BYTES = B_ROWS * ROW_BYTES;
  // stage layout: A | B [| lo(A) | lo(B)]
  static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * (SPLIT ? 2 : 1);
  static constexpr int STAGES_FIT = 196608 / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int CONV_THREADS = 256;  // split modes: 8 converter warps
  static constexpr bool CONVERTS = SPLIT == 1 || SPLIT == 2;
  static constexpr int EPI_WARPS = 8;       // two per TMEM lane quarter
  static constexpr int CONV_WARP0 = 2 + EPI_WARPS;
  static constexpr int THREADS = 32 * CONV_WARP0 + (CONVERTS ? CONV_THREADS : 0);
  // Two accumulators of BN columns, allocated as a power of two.
  static constexpr int TMEM_COLS = 2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512);
  static constexpr int EPI_BUF_BYTES = BM * 32 * 4;  // one 128x32 fp32 output chunk
  // Two buffers: one per epilogue half (each half stages its own chunks).
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = EPI_OFF + 2 * EPI_BUF_BYTES;
  static constexpr int BAR_BYTES = 256;
  // The tile's bias columns, staged by the epilogue before it waits for the
  // accumulator (off the critical path of the tile's epilogue).
  static constexpr int BIAS_OFF = BAR_OFF + BAR_BYTES;
  static constexpr int SMEM_BYTES = BIAS_OFF + BN * 4 + 1024;
  static_assert(BN == 64 || BN == 96 || BN == 112 || BN == 128 || BN == 256, "BN");
  static_assert(STAGES >= 2 && STAGES <= 8, "stages");
  static_assert(SMEM_BYTES <= 232448, "smem");
  static_assert(!PAIR || (SPLIT == SPLIT_BF16X3_PRE && (BN == 128 || BN == 256)), "pair shape");
};

// Low part of a TF32 split: x - trunc_tf32(x), exact in fp32.
__device__ __forceinline__ uint32_t tf32_lo_bits(uint32_t x) {
  const float f = __uint_as_float(x);
  const float hi = __uint_as_float(x & 0xFFFFE000u);
  return __float_as_uint(f - hi);
}

// Instruction descriptor for kind::f16 with BF16 A/B and an FP32 accumulator.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

__device__ __forceinline__ uint32_t pack_bf16x2(__nv_bfloat16 lo_k, __nv_bfloat16 hi_k) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(lo_k)) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(hi_k)) << 16);
}

// Split 8 consecutive k-values of one row of a staged fp32 tile (128-byte
// rows, 128B swizzle: 16-byte chunk c of row r sits at chunk c ^ (r & 7)) into
// bf16 hi and lo rows (64-byte rows, 64B swizzle: chunk m of row r sits at
// chunk m ^ ((r >> 1) & 3)).
__device__ __forceinline__ void split_bf16_chunk(const uint8_t* f32_tile, uint8_t* hi_tile,
                                                 uint8_t* lo_tile, int r, int m) {
  const float4 v0 =
      *reinterpret_cast<const float4*>(f32_tile + r * 128 + (((2 * m) ^ (r & 7)) << 4));
  const float4 v1 =
      *reinterpret_cast<const float4*>(f32_tile + r * 128 + (((2 * m + 1) ^ (r & 7)) << 4));
  const float x[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
  __nv_bfloat16 h[8], l[8];
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    h[t] = __float2bfloat16_rn(x[t]);
    l[t] = __float2bfloat16_rn(x[t] - __bfloat162float(h[t]));
  }
  const int dst = r * 64 + ((m ^ ((r >> 1) & 3)) << 4);
  *reinterpret_cast<uint4*>(hi_tile + dst) =
      make_uint4(pack_bf16x2(h[0], h[1]), pack_bf16x2(h[2], h[3]), pack_bf16x2(h[4], h[5]),
                 pack_bf16x2(h[6], h[7]));
  *reinterpret_cast<uint4*>(lo_tile + dst) =
      make_uint4(pack_bf16x2(l[0], l[1]), pack_bf16x2(l[2], l[3]), pack_bf16x2(l[4], l[5]),
                 pack_bf16x2(l[6], l[7]));
}

// cta_group::2: issued by the pair's first CTA, A rows from both CTAs, B
// columns split between them, D in both CTAs' TMEM.
__device__ __forceinline__ void mma_bf16_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// GELU(x) = x/2 (1 + erf(x / sqrt 2)), with erf from Abramowitz & Stegun,
// Handbook of Mathematical Functions, formula 7.1.26: for z >= 0,
//   erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) e^(-z^2),
//   t = 1 / (1 + p z),  |error| <= 1.5e-7,
// so with q = poly(t) e^(-z^2) and z = |x| / sqrt 2:
//   GELU(x) = x - x q / 2 for x >= 0,  x q / 2 for x < 0.
// One reciprocal and one exp2 on the multi-function unit and six FMAs; the
// GELU error stays below 1e-7 |x|, far under the bf16 hi/lo pair that
// carries the result (2^-17 relative).
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float gelu_erf(float x) {
  constexpr float kP = 0.3275911f;
  constexpr float kA1 = 0.254829592f, kA2 = -0.284496736f, kA3 = 1.421413741f;
  constexpr float kA4 = -1.453152027f, kA5 = 1.061405429f;
  constexpr float kInvSqrt2 = 0.70710678118654752440f;
  constexpr float kNegLog2e = -1.44269504088896340736f;
  const float z = fabsf(x) * kInvSqrt2;
  const float t = rcp_approx(fmaf(kP, z, 1.f));
  const float poly = t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, kA5, kA4), kA3), kA2), kA1);
  const float q = poly * fast_exp2(z * z * kNegLog2e);
  const float h = 0.5f * x * q;
  return x >= 0.f ? x - h : h;
}

// gelu_erf on a pair, the polynomial and products on packed f32x2 FMAs and
// multiplies (the same formula; the reciprocal and exp2 stay scalar).
__device__ __forceinline__ void gelu_erf2(float& x0, float& x1) {
  constexpr float kP = 0.3275911f;
  constexpr float kA1 = 0.254829592f, kA2 = -0.284496736f, kA3 = 1.421413741f;
  constexpr float kA4 = -1.453152027f, kA5 = 1.061405429f;
  constexpr float kInvSqrt2 = 0.70710678118654752440f;
  constexpr float kNegLog2e = -1.44269504088896340736f;
  const uint64_t z = f2_mul(f2_pack(fabsf(x0), fabsf(x1)), f2_pack(kInvSqrt2, kInvSqrt2));
  float u0, u1;
  f2_unpack(f2_fma(f2_pack(kP, kP), z, f2_pack(1.f, 1.f)), u0, u1);
  const uint64_t t = f2_pack(rcp_approx(u0), rcp_approx(u1));
  uint64_t poly = f2_fma(t, f2_pack(kA5, kA5), f2_pack(kA4, kA4));
  poly = f2_fma(t, poly, f2_pack(kA3, kA3));
  poly = f2_fma(t, poly, f2_pack(kA2, kA2));
  poly = f2_fma(t, poly, f2_pack(kA1, kA1));
  poly = f2_mul(t, poly);
  float e0, e1;
  f2_unpack(f2_mul(f2_mul(z, z), f2_pack(kNegLog2e, kNegLog2e)), e0, e1);
  const uint64_t q = f2_mul(poly, f2_pack(fast_exp2(e0), fast_exp2(e1)));
  const uint64_t xx = f2_pack(x0, x1);
  const uint64_t h = f2_mul(f2_mul(f2_pack(0.5f, 0.5f), xx), q);
  float h0, h1, d0, d1;
  f2_unpack(h, h0, h1);
  f2_unpack(f2_fma(h, f2_pack(-1.f, -1.f), xx), d0, d1);  // x - h
  x0 = x0 >= 0.f ? d0 : h0;
  x1 = x1 >= 0.f ? d1 : h1;
}

template <int EPI>
__device__ __forceinline__ void gemm_store_chunk(const float (&v)[32], float* __restrict__ crow,
                                                 const float* __restrict__ bias, int col0, int N,
                                                 int flags, int hd, int hs) {
  const bool rnd = (flags & KF_GEMM_ROUND_TF32) != 0;
  const bool vec = (flags & KF_GEMM_VEC_OK) != 0;
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const int col = col0 + j;
    if (col >= N) break;
    if (vec && col + 3 < N) {
      float4 bb = make_float4(0.f, 0.f, 0.f, 0.f);
      if (bias) bb = __ldg(reinterpret_cast<const float4*>(bias + col));
      float4 o = make_float4(v[j] + bb.x, v[j + 1] + bb.y, v[j + 2] + bb.z, v[j + 3] + bb.w);
      if (EPI == KF_EPI_BIAS_GELU) {
        o.x = gelu_erf(o.x);
        o.y = gelu_erf(o.y);
        o.z = gelu_erf(o.z);
        o.w = gelu_erf(o.w);
      }
      if (rnd) {
        o.x = round_tf32(o.x);
        o.y = round_tf32(o.y);
        o.z = round_tf32(o.z);
        o.w = round_tf32(o.w);
      }
      const int dst = hd ? (col / hd) * hs + (col % hd) : col;
      *reinterpret_cast<float4*>(crow + dst) = o;
    } else {
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int cc = col + t;
        if (cc < N) {
          float o = v[j + t] + (bias ? __ldg(bias + cc) : 0.f);
          if (EPI == KF_EPI_BIAS_GELU) o = gelu_erf(o);
          if (rnd) o = round_tf32(o);
          const int dst = hd ? (cc / hd) * hs + (cc % hd) : cc;
          crow[dst] = o;
        }
      }
    }
  }
}

// Stream-K workspace (SK kernels): fp32 partial accumulators of tiles split
// between CTAs, [tiles][2 parts][128 rows][BN], and per (tile, epilogue half)
// arrival counters, zero between launches.
struct SkArgs {
  float* ws;
  int* flags;
};

template <int BN, int EPI, int SPLIT, bool PAIR = false, bool SK = false>
__global__ void __launch_bounds__((SPLIT == 1 || SPLIT == 2) ? 576 : 320, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, float* __restrict__ C, int64_t ldc, const float* __restrict__ bias, int M,
                     int N, int K, int flags, int head_dim, int head_stride,
                     const int32_t* __restrict__ live_tiles, const int32_t* __restrict__ live_count,
                     const __grid_constant__ SkArgs sk) {
  using Cfg = GemmCfg<BN, SPLIT, PAIR>;
  constexpr int BM = Cfg::BM, BK = Cfg::BK, STAGES = Cfg::STAGES;
  static_assert(!SK || (SPLIT == SPLIT_BF16X3_PRE && !PAIR), "stream-K shape");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* conv = empty + STAGES;  // split mode: lo tiles written
  uint64_t* acc_full = conv + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* epi_ok = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [2], per half

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_n = (N + BN - 1) / BN;
  const int num_kb = (K + BK - 1) / BK;
  // PAIR: rank in the CTA pair; rank 0 issues the MMAs for both.
  const uint32_t crank = PAIR ? cluster_ctarank() : 0u;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], Cfg::CONV_THREADS / 32);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      // PAIR: rank 0's barrier counts the epilogue warps of both CTAs.
      mbar_init(&acc_empty[a], PAIR ? 2 * Cfg::EPI_WARPS : Cfg::EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (flags & KF_GEMM_TMA_OUT) tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // PAIR: both CTAs of the pair have initialised their barriers (and hold
  // their TMEM) before either signals the other's remotely (warp-aligned:
  // reconverge first).
  if (PAIR) {
    __syncwarp();
    cluster_sync_all();
  }

  // The next kernel is released only once every CTA of this one holds its
  // TMEM (a CTA of the next kernel may allocate before its own wait, and must
  // then only ever wait for columns that a running CTA will free).
  pdl_launch_dependents();
  // KF_GEMM_W_STATIC (the caller guarantees W was written before the
  // previous kernel in the stream started): the W tiles of the first stages
  // of this CTA's first tile are loaded before the wait, so they overlap the
  // previous kernel's tail. Their barriers expect those bytes now and the A
  // bytes and the arrival later (the phase cannot end in between).
  int pre_w = 0;
  if constexpr (Cfg::PRESPLIT && !PAIR && !SK) {
    if ((flags & KF_GEMM_W_STATIC) && warp == 0 && lane == 0) {
      const int nw0 = (static_cast<int>(blockIdx.x) % num_n) * BN;
      pre_w = num_kb < STAGES ? num_kb : STAGES;
      for (int s2 = 0; s2 < pre_w; ++s2) {
        uint8_t* sa = smem + s2 * Cfg::STAGE_BYTES;
        mbar_expect_tx(&full[s2], 2 * Cfg::B_BYTES);
        tma_load_3d(sa + Cfg::A_BYTES, &tmB, &full[s2], s2 * BK, nw0, 0);
        tma_load_3d(sa + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &tmB, &full[s2], s2 * BK, nw0, 1);
      }
    }
  }
  // Everything above overlaps the previous kernel; from here on we read its
  // outputs (the A operand and the live-tile list).
  pdl_wait();
  // Optional list of the 128-row tiles that hold at least one live row
  // (kf_live_row_tiles); other row tiles are not computed and keep their
  // contents. Every role reads the same list, so they agree on the schedule.
  const int num_m = live_tiles ? __ldg(live_count) : (M + BM - 1) / BM;
  // Work units: 128 x BN tiles, or (PAIR) 256 x BN tiles made of the row
  // tiles 2i and 2i+1 of the list (the two need not be adjacent rows). With an
  // odd count the last pair's second CTA repeats the first's rows and stores
  // nothing. Units go round-robin over CTAs (pairs), N fastest.
  const int num_tiles = (PAIR ? (num_m + 1) / 2 : num_m) * num_n;
  const int unit0 = PAIR ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int ustride = PAIR ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
  auto row_tile = [&](int tile, bool& own) -> int {
    int mi = tile / num_n;
    own = true;
    if (PAIR) {
      const int j = 2 * mi + static_cast<int>(crank);
      own = j < num_m;
      mi = own ? j : 2 * mi;
    }
    return (live_tiles ? __ldg(live_tiles + mi) : mi) * BM;
  };
  auto row0 = [&](int tile) -> int {
    bool own;
    return row_tile(tile, own);
  };
  // Segments (tile, k blocks [kb_b, kb_e)) a CTA computes, the same sequence
  // for every role. Round-robin whole tiles, or (SK, stream-K) an even share
  // of the num_tiles * num_kb k blocks: CTA c takes [c W / G, (c+1) W / G),
  // with G cut so that a share is at least half a tile (a tile then spans at
  // most three CTAs). A tile's first part (kb_b = 0) is its owner: it adds
  // the other parts, which their CTAs compute first in their ranges.
  const long long sk_W = static_cast<long long>(num_tiles) * num_kb;
  int sk_G = static_cast<int>(gridDim.x);
  if (SK && 2LL * num_tiles < sk_G) sk_G = 2 * num_tiles;
  auto sk_beg = [&](long long c) -> long long { return c * sk_W / sk_G; };
  auto sk_cta_of = [&](long long u) -> int {  // the CTA whose share holds k block u
    long long c = u * sk_G / (sk_W > 0 ? sk_W : 1);
    while (c + 1 < sk_G && sk_beg(c + 1) <= u) ++c;
    while (c > 0 && sk_beg(c) > u) --c;
    return static_cast<int>(c);
  };
  struct SegIter {
    long long u, u1;
    int rr, rr_stride, n_tiles, n_kb;
    __device__ bool next(int& tile, int& kb_b, int& kb_e) {
      if (SK) {
        if (u >= u1) return false;
        tile = static_cast<int>(u / n_kb);
        kb_b = static_cast<int>(u - static_cast<long long>(tile) * n_kb);
        const long long rem = u1 - u;
        kb_e = (kb_b + rem < n_kb) ? kb_b + static_cast<int>(rem) : n_kb;
        u += kb_e - kb_b;
        return true;
      }
      if (rr >= n_tiles) return false;
      tile = rr;
      kb_b = 0;
      kb_e = n_kb;
      rr += rr_stride;
      return true;
    }
  };
  const bool sk_active = SK && static_cast<int>(blockIdx.x) < sk_G;
  const SegIter seg0{sk_active ? sk_beg(blockIdx.x) : 0, sk_active ? sk_beg(blockIdx.x + 1) : 0,
                     unit0, ustride, num_tiles, num_kb};

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      SegIter it = seg0;
      int tile, kb_b, kb_e;
      while (ok && it.next(tile, kb_b, kb_e)) {
        const int m0 = row0(tile);
        // PAIR: this CTA stages B rows [n0 + rank * BN/2, + BN/2) of the tile.
        const int n0 = (tile % num_n) * BN + static_cast<int>(crank) * (PAIR ? Cfg::B_ROWS : 0);
        for (int kb = kb_b; kb < kb_e; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, KF_DEV_WAIT_TIMEOUT_TMA)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
          if constexpr (PAIR) {
            // Both CTAs' loads complete on rank 0's barrier, which rank 0 arms
            // with the bytes of the pair (the other CTA's bytes may land
            // first: the phase cannot end before rank 0's arrival).
            if (crank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            tma_load_3d_pair(sa, &tmA, fb, kb * BK, m0, 0);
            tma_load_3d_pair(sa + Cfg::A_BYTES, &tmB, fb, kb * BK, n0, 0);
            tma_load_3d_pair(sa + Cfg::A_BYTES + Cfg::B_BYTES, &tmA, fb, kb * BK, m0, 1);
            tma_load_3d_pair(sa + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &tmB, fb, kb * BK, n0, 1);
          } else if (Cfg::PRESPLIT && issued < pre_w) {
            // W of this stage went out before the wait: A only, and arrive.
            mbar_arrive_expect_tx(&full[stage], 2 * Cfg::A_BYTES);
            tma_load_3d(sa, &tmA, &full[stage], kb * BK, m0, 0);
            tma_load_3d(sa + Cfg::A_BYTES + Cfg::B_BYTES, &tmA, &full[stage], kb * BK, m0, 1);
          } else if (Cfg::PRESPLIT) {
            // planes: A_hi | B_hi | A_lo | B_lo (3-D maps, plane = coordinate 2)
            mbar_arrive_expect_tx(&full[stage], 2 * (Cfg::A_BYTES + Cfg::B_BYTES));
            tma_load_3d(sa, &tmA, &full[stage], kb * BK, m0, 0);
            tma_load_3d(sa + Cfg::A_BYTES, &tmB, &full[stage], kb * BK, n0, 0);
            tma_load_3d(sa + Cfg::A_BYTES + Cfg::B_BYTES, &tmA, &full[stage], kb * BK, m0, 1);
            tma_load_3d(sa + 2 * Cfg::A_BYTES + Cfg::B_BYTES, &tmB, &full[stage], kb * BK, n0,
                        1);
          } else {
            mbar_arrive_expect_tx(&full[stage], Cfg::A_BYTES + Cfg::B_BYTES);
            tma_load_2d(sa, &tmA, &full[stage], kb * BK, m0);
            tma_load_2d(sa + Cfg::A_BYTES, &tmB, &full[stage], kb * BK, n0);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Prefetched W stages that never got their A loads (no tile for this
      // CTA, or an abort): arrive, so the phase ends once the W bytes land,
      // and wait for that before the shared memory can be released.
      for (long long s2 = issued; s2 < pre_w; ++s2) {
        mbar_arrive(&full[s2]);
        mbar_wait_drain(&full[s2], 0, KF_DEV_WAIT_TIMEOUT_TMA);
      }
      if (PAIR) {
        // Rank 0's MMA thread releases the stages of both CTAs (its commits
        // arrive in this CTA's shared memory, and its products read this
        // CTA's tiles): wait for the release of the last ones before leaving.
        const long long first = issued > STAGES ? issued - STAGES : 0;
        for (long long i = first; i < issued; ++i)
          mbar_wait_drain(&empty[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1),
                          KF_DEV_WAIT_TIMEOUT_TMA);
      } else if (!ok) {
        // Drain: wait for the loads still in flight (the last <= STAGES).
        const long long first = issued > STAGES ? issued - STAGES : 0;
        for (long long i = first; i < issued; ++i)
          mbar_wait_drain(&full[i % STAGES], static_cast<uint32_t>((i / STAGES) & 1),
                          KF_DEV_WAIT_TIMEOUT_TMA);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && crank == 0) {
      // ------------------------------------------------ MMA issuer
      // (PAIR: rank 0 only; each cta_group::2 product covers both CTAs' rows)
      constexpr uint32_t idesc = make_idesc_tf32(BM, BN, 0, 0);
      constexpr uint32_t idesc_bf = make_idesc_bf16(PAIR ? 2 * BM : BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      SegIter it = seg0;
      int tile, kb_b, kb_e;
      while (ok && it.next(tile, kb_b, kb_e)) {
        // PAIR: the other CTA's epilogue warps arrive remotely (release at
        // cluster scope), so the wait acquires at cluster scope.
        if (!(PAIR ? mbar_wait_cluster(&acc_empty[acc], acc_phase ^ 1u, abort_flag,
                                       KF_DEV_WAIT_TIMEOUT_MMA)
                   : mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag,
                               KF_DEV_WAIT_TIMEOUT_MMA))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = kb_b; kb < kb_e; ++kb) {
          if (!mbar_wait(Cfg::CONVERTS ? &conv[stage] : &full[stage], phase, abort_flag,
                         KF_DEV_WAIT_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t b_addr = a_addr + Cfg::A_BYTES;
          const uint32_t alo_addr = b_addr + Cfg::B_BYTES;
          const uint32_t blo_addr = alo_addr + Cfg::A_BYTES;
          if (PAIR) {
            // As below, one cta_group::2 product per step: M = 256 rows (A
            // from both CTAs), B's BN rows split between the CTAs.
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint64_t ah = make_smem_desc(a_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
              const uint64_t bh = make_smem_desc(b_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
              const uint64_t al = make_smem_desc(alo_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
              const uint64_t bl = make_smem_desc(blo_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
              mma_bf16_ss_pair(d_tmem, al, bh, idesc_bf, (kb != kb_b || k != 0) ? 1u : 0u);
              mma_bf16_ss_pair(d_tmem, ah, bl, idesc_bf, 1u);
              mma_bf16_ss_pair(d_tmem, ah, bh, idesc_bf, 1u);
            }
          } else if (SPLIT == SPLIT_BF16X3_PRE) {
            // TMA-loaded bf16 planes, 128-byte rows (SW128): 4 k steps of 16.
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint64_t ah = make_smem_desc(a_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
              const uint64_t bh = make_smem_desc(b_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
              const uint64_t al = make_smem_desc(alo_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
              const uint64_t bl = make_smem_desc(blo_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
              mma_bf16_ss(d_tmem, al, bh, idesc_bf, (kb != kb_b || k != 0) ? 1u : 0u);
              mma_bf16_ss(d_tmem, ah, bl, idesc_bf, 1u);
              mma_bf16_ss(d_tmem, ah, bh, idesc_bf, 1u);
            }
          } else if (SPLIT == SPLIT_BF16X3) {
            // bf16 tiles: A_hi | A_lo | B_hi | B_lo, 64-byte rows (SW64).
            const uint32_t ahi = alo_addr, alo = ahi + Cfg::A_BYTES / 2;
            const uint32_t bhi = alo + Cfg::A_BYTES / 2, blo = bhi + Cfg::B_BYTES / 2;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              const uint64_t ah = make_smem_desc(ahi + k * 32, 16, 512, KF_SWIZZLE_64B);
              const uint64_t al = make_smem_desc(alo + k * 32, 16, 512, KF_SWIZZLE_64B);
              const uint64_t bh = make_smem_desc(bhi + k * 32, 16, 512, KF_SWIZZLE_64B);
              const uint64_t bl = make_smem_desc(blo + k * 32, 16, 512, KF_SWIZZLE_64B);
              mma_bf16_ss(d_tmem, al, bh, idesc_bf, (kb != kb_b || k != 0) ? 1u : 0u);
              mma_bf16_ss(d_tmem, ah, bl, idesc_bf, 1u);
              mma_bf16_ss(d_tmem, ah, bh, idesc_bf, 1u);
            }
          } else
#pragma unroll
          for (int k = 0; k < BK / 8; ++k) {
            const uint64_t ad = make_smem_desc(a_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
            const uint64_t bd = make_smem_desc(b_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
            if (SPLIT) {
              const uint64_t ald = make_smem_desc(alo_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
              const uint64_t bld = make_smem_desc(blo_addr + k * 32, 16, 1024, KF_SWIZZLE_128B);
              mma_tf32_ss(d_tmem, ald, bd, idesc, (kb != kb_b || k != 0) ? 1u : 0u);
              mma_tf32_ss(d_tmem, ad, bld, idesc, 1u);
            }
            mma_tf32_ss(d_tmem, ad, bd, idesc, (SPLIT || kb != kb_b || k != 0) ? 1u : 0u);
            (void)idesc_bf;
          }
          if constexpr (PAIR) {
            // The stage is free in both CTAs once these products complete.
            mma_commit_pair(&empty[stage]);
            mma_commit_pair_at(mapa_shared(smem_u32(&empty[stage]), 1));
          } else {
            mma_commit(&empty[stage]);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if constexpr (PAIR) {
          mma_commit_pair(&acc_full[acc]);
          mma_commit_pair_at(mapa_shared(smem_u32(&acc_full[acc]), 1));
        } else {
          mma_commit(&acc_full[acc]);
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // Every MMA this thread issued completes before TMEM is released.
      if constexpr (PAIR) {
        mma_commit_pair(drain);
      } else {
        mma_commit(drain);
      }
      mbar_wait_drain(drain, 0, KF_DEV_WAIT_TIMEOUT_MMA);
    }
  } else if (Cfg::CONVERTS && warp >= Cfg::CONV_WARP0) {
    // -------------------------------------------------- converters (warps 6..9)
    const int ct = threadIdx.x - 32 * Cfg::CONV_WARP0;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int tile = unit0; tile < num_tiles && ok; tile += ustride) {
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&full[stage], phase, abort_flag, KF_DEV_WAIT_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        uint8_t* st_base = smem + stage * Cfg::STAGE_BYTES;
        if (SPLIT == SPLIT_BF16X3) {
          uint8_t* ahi = st_base + Cfg::A_BYTES + Cfg::B_BYTES;
          uint8_t* alo = ahi + Cfg::A_BYTES / 2;
          uint8_t* bhi = alo + Cfg::A_BYTES / 2;
          uint8_t* blo = bhi + Cfg::B_BYTES / 2;
#pragma unroll 2
          for (int i = ct; i < BM * 4; i += Cfg::CONV_THREADS)
            split_bf16_chunk(st_base, ahi, alo, i >> 2, i & 3);
#pragma unroll 2
          for (int i = ct; i < BN * 4; i += Cfg::CONV_THREADS)
            split_bf16_chunk(st_base + Cfg::A_BYTES, bhi, blo, i >> 2, i & 3);
        } else {
          const uint4* src = reinterpret_cast<const uint4*>(st_base);
          uint4* dst = reinterpret_cast<uint4*>(st_base + Cfg::A_BYTES + Cfg::B_BYTES);
          constexpr int NV = (Cfg::A_BYTES + Cfg::B_BYTES) / 16 / Cfg::CONV_THREADS;
          static_assert(!Cfg::CONVERTS || NV * 16 * Cfg::CONV_THREADS == Cfg::A_BYTES + Cfg::B_BYTES,
                        "split");
          uint4 v[NV];
#pragma unroll
          for (int t = 0; t < NV; ++t) v[t] = src[ct + t * Cfg::CONV_THREADS];  // all loads in flight
#pragma unroll
          for (int t = 0; t < NV; ++t) {
            v[t].x = tf32_lo_bits(v[t].x);
            v[t].y = tf32_lo_bits(v[t].y);
            v[t].z = tf32_lo_bits(v[t].z);
            v[t].w = tf32_lo_bits(v[t].w);
            dst[ct + t * Cfg::CONV_THREADS] = v[t];
          }
        }
        fence_proxy_async_smem();  // generic-proxy stores -> tensor-core reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // ------------------------------------------ epilogue (warps 2..9, two halves)
    // Warps 2-5 and 6-9 each cover all four TMEM lane quarters (warp w reads
    // lanes 32*(w%4)..+31); half 0 takes the even 32-column chunks, half 1
    // the odd ones, each with its own leader, named barrier (ids 1, 2) and
    // staging buffer, so the two halves run independently.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int bar_id = 1 + half;
    const bool tma_out = (flags & KF_GEMM_TMA_OUT) != 0;
    const bool leader = threadIdx.x == 64 + 128 * half;
    const bool rnd = (flags & KF_GEMM_ROUND_TF32) != 0;
    uint8_t* buf = smem + Cfg::EPI_OFF + half * Cfg::EPI_BUF_BYTES;
    float* sbias = reinterpret_cast<float*>(smem + Cfg::BIAS_OFF);  // [BN], per tile
    const int ht = threadIdx.x - (64 + 128 * half);                 // 0..127 in the half
    int acc = 0;
    uint32_t acc_phase = 0;
    SegIter it = seg0;
    int tile, kb_b, kb_e;
    while (it.next(tile, kb_b, kb_e)) {
      bool own;  // PAIR: false for a repeated row tile (nothing stored)
      const int m0 = row_tile(tile, own);
      const int n0 = (tile % num_n) * BN;
      // Stage the bias of this half's chunks (columns 32*half + 64*j + 0..31)
      // while the MMAs of the tile run; 0 past N or without a bias. The
      // previous tile's readers are past the end-of-tile barrier, and the
      // barrier after the accumulator wait publishes these writes.
      if (ht < 32) {
        for (int c = 32 * half; c < BN; c += 64)
          if (c + ht < BN)
            sbias[c + ht] = (bias && n0 + c + ht < N) ? __ldg(bias + n0 + c + ht) : 0.f;
      }
      // One bounded wait by the half's leader, shared through the half's
      // named barrier, so all four warps of a half always reach the same
      // barriers (no warp can be left waiting for one that gave up).
      if (leader) epi_ok[half] = mbar_wait(&acc_full[acc], acc_phase, abort_flag,
                                           KF_DEV_WAIT_TIMEOUT_EPI) ? 1 : 0;
      named_bar_sync(bar_id, 128);
      if (!epi_ok[half]) break;
      tc_fence_after();
      // Stream-K: a later part of a tile (kb_b > 0) leaves its partial
      // accumulator in the workspace (slot = part - 1) and counts itself in
      // the tile's per-half counter; the owner (kb_b == 0, the tile's first
      // k blocks) waits for the other parts and adds them, in part order.
      int sk_part = 0, sk_np = 0;
      if constexpr (SK) {
        const long long tu = static_cast<long long>(tile) * num_kb;
        if (kb_b > 0)
          sk_part = static_cast<int>(blockIdx.x) - sk_cta_of(tu);
        else if (kb_e < num_kb)
          sk_np = sk_cta_of(tu + num_kb - 1) - static_cast<int>(blockIdx.x);
        if (sk_part > 2 || sk_np > 2) {  // the share cut makes this impossible
          if (leader) record_device_status(KF_DEV_WAIT_TIMEOUT_EPI);
          sk_part = sk_part > 2 ? 3 : sk_part;
          sk_np = sk_np > 2 ? 2 : sk_np;
        }
        if (sk_np > 0) {
          if (leader) {
            volatile int* fl = sk.flags + 2 * tile + half;
            int got = 1;
            const long long t0 = clock64();
            while (*fl < sk_np) {
              if (*abort_flag || clock64() - t0 > wait_limit()) {
                *abort_flag = 1;
                record_device_status(KF_DEV_WAIT_TIMEOUT_EPI);
                got = 0;
                break;
              }
              __nanosleep(64);
            }
            __threadfence();
            epi_ok[half] = got;
          }
          named_bar_sync(bar_id, 128);
          if (!epi_ok[half]) break;
        }
      }
      const int r = quarter * 32 + lane;
      const int row = m0 + r;
      const uint32_t tbase =
          tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * BN);
      float* crow = C + static_cast<int64_t>(row) * ldc;
#pragma unroll 1
      for (int c = 32 * half; c < BN; c += 64) {
        if (n0 + c >= N || !own) break;  // uniform over the half
        float v[32];
        // BN = 112: the last chunk holds 16 columns. Its TMEM load also reads
        // 16 columns past the accumulator (inside the allocation, unused), and
        // it is stored directly, bounded by the tile's last column.
        const bool part = (c + 32 > BN);
        tmem_ld32(tbase + static_cast<uint32_t>(c), v);
        if constexpr (SK) {
          if (sk_part > 0) {  // a later part: this thread's row of the chunk to the workspace
            if (sk_part <= 2) {
              float4* dst = reinterpret_cast<float4*>(
                  sk.ws + ((static_cast<int64_t>(tile) * 2 + sk_part - 1) * BM + r) * BN + c);
#pragma unroll
              for (int j = 0; j < 8; ++j)
                dst[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            }
            continue;
          }
          for (int pp = 0; pp < sk_np; ++pp) {  // the owner adds the later parts in order
            const float4* src = reinterpret_cast<const float4*>(
                sk.ws + ((static_cast<int64_t>(tile) * 2 + pp) * BM + r) * BN + c);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 q = __ldcg(src + j);
              v[4 * j] += q.x;
              v[4 * j + 1] += q.y;
              v[4 * j + 2] += q.z;
              v[4 * j + 3] += q.w;
            }
          }
        }
        if (part) {
          if (row < M)
            gemm_store_chunk<EPI>(v, crow, bias, n0 + c, (n0 + BN < N ? n0 + BN : N), flags,
                                  head_dim, head_stride);
        } else if (tma_out && (flags & KF_GEMM_OUT_SPLIT)) {
          // bf16 hi/lo planes: two 128x32 bf16 tiles (64-byte rows, SW64).
          // The arithmetic runs before the wait for the staging buffer, so
          // it overlaps the previous chunk's TMA store.
          uint4 hu[4], lu[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {  // 8 columns -> one 16-byte unit per plane
            float o[8];
            {
              const float4 b0 = *reinterpret_cast<const float4*>(sbias + c + 8 * j);
              const float4 b1 = *reinterpret_cast<const float4*>(sbias + c + 8 * j + 4);
              const float bs[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
              for (int t = 0; t < 8; t += 2)  // accumulator + bias, two columns per add
                f2_unpack(f2_add(f2_pack(v[8 * j + t], v[8 * j + t + 1]),
                                 f2_pack(bs[t], bs[t + 1])),
                          o[t], o[t + 1]);
            }
            if (EPI == KF_EPI_BIAS_GELU) {
#pragma unroll
              for (int t = 0; t < 8; t += 2) gelu_erf2(o[t], o[t + 1]);
            }
            uint32_t hw[4], lw[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) split_bf16x2(o[2 * t], o[2 * t + 1], hw[t], lw[t]);
            hu[j] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
            lu[j] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
          }
          if (leader) bulk_wait_group_read<0>();  // this half's last store has read `buf`
          named_bar_sync(bar_id, 128);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int off = r * 64 + ((j ^ ((r >> 1) & 3)) << 4);
            *reinterpret_cast<uint4*>(buf + off) = hu[j];
            *reinterpret_cast<uint4*>(buf + Cfg::EPI_BUF_BYTES / 2 + off) = lu[j];
          }
          fence_proxy_async_smem();
          named_bar_sync(bar_id, 128);
          if (leader) {
            tma_store_3d(&tmC, buf, n0 + c, m0, 0);
            tma_store_3d(&tmC, buf + Cfg::EPI_BUF_BYTES / 2, n0 + c, m0, 1);
            bulk_commit_group();
          }
        } else if (tma_out) {
          float4 ov[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 bb = *reinterpret_cast<const float4*>(sbias + c + 4 * j);
            float4 o;
            f2_unpack(f2_add(f2_pack(v[4 * j], v[4 * j + 1]), f2_pack(bb.x, bb.y)), o.x, o.y);
            f2_unpack(f2_add(f2_pack(v[4 * j + 2], v[4 * j + 3]), f2_pack(bb.z, bb.w)), o.z, o.w);
            if (EPI == KF_EPI_BIAS_GELU) {
              o.x = gelu_erf(o.x);
              o.y = gelu_erf(o.y);
              o.z = gelu_erf(o.z);
              o.w = gelu_erf(o.w);
            }
            if (rnd) {
              o.x = round_tf32(o.x);
              o.y = round_tf32(o.y);
              o.z = round_tf32(o.z);
              o.w = round_tf32(o.w);
            }
            ov[j] = o;
          }
          // Arithmetic done; now wait until this half's last store has read `buf`.
          if (leader) bulk_wait_group_read<0>();
          named_bar_sync(bar_id, 128);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(buf + r * 128 + ((j ^ (r & 7)) << 4)) = ov[j];
          fence_proxy_async_smem();  // generic smem writes -> TMA store reads
          named_bar_sync(bar_id, 128);
          if (leader) {
            tma_store_2d(&tmC, buf, n0 + c, m0);
            bulk_commit_group();
          }
        } else if (row < M) {
          gemm_store_chunk<EPI>(v, crow, bias, n0 + c, N, flags, head_dim, head_stride);
        }
      }
      if constexpr (SK) {
        if (sk_part > 0 && sk_part <= 2) {
          __threadfence();  // this thread's partial rows, at device scope
          named_bar_sync(bar_id, 128);
          if (leader) atomicAdd(sk.flags + 2 * tile + half, 1);
        } else if (sk_np > 0) {
          named_bar_sync(bar_id, 128);  // the half has read every part
          if (leader) atomicExch(sk.flags + 2 * tile + half, 0);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        // PAIR: the accumulator is handed back to rank 0's MMA thread.
        if (PAIR)
          mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));
        else
          mbar_arrive(&acc_empty[acc]);
      }
      named_bar_sync(bar_id, 128);  // the half has read epi_ok before it is rewritten
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    // Shared memory must outlive the stores' reads of it; the writes
    // themselves complete before the grid does (a dependent kernel's
    // griddepcontrol.wait sees them).
    if (tma_out && leader) bulk_wait_group_read<0>();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // PAIR: no CTA leaves while its peer may still write into its shared
  // memory or arrive on its barriers; the pair frees TMEM together.
  if (PAIR) {
    __syncwarp();
    cluster_sync_all();
  }
  if (warp == 1) {
    __syncwarp();
    if constexpr (PAIR)
      tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

template <int BN, int EPI, int SPLIT>
static int launch_gemm(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                       float* C, int64_t ldc,
                       const float* bias, int M, int N, int K, int flags, int hd, int hs,
                       const int32_t* live_tiles, const int32_t* live_count, cudaStream_t st) {
  using Cfg = GemmCfg<BN, SPLIT>;
  auto kern = gemm_tf32_kernel<BN, EPI, SPLIT>;
  static DeviceOnce once;
  const int rc_attr = once.run("kf_gemm_tf32", nullptr, [&](int) {
    return cuda_status(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES),
        "kf_gemm_tf32: set smem attribute");
  });
  if (rc_attr) return rc_attr;
  // With a live-tile list the count is only known on the device: launch one
  // CTA per SM and let CTAs without work exit.
  const int tiles = ((M + Cfg::BM - 1) / Cfg::BM) * ((N + BN - 1) / BN);
  const int grid = tiles < sm_count() ? tiles : sm_count();
  return cuda_status(launch_chained(kern, dim3(grid), dim3(Cfg::THREADS), Cfg::SMEM_BYTES, st, ta,
                                    tb, tc, C, ldc, bias, M, N, K, flags, hd, hs, live_tiles,
                                    live_count, SkArgs{}),
                     "kf_gemm_tf32 launch");
}

// Stream-K GEMM: one CTA per SM, each taking an even share of all k blocks
// (the share cut on the device once the live tile count is known).
template <int BN, int EPI>
static int launch_gemm_sk(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                          float* C, int64_t ldc, const float* bias, int M, int N, int K, int flags,
                          int hd, int hs, const int32_t* live_tiles, const int32_t* live_count,
                          const SkArgs& sk, cudaStream_t st) {
  using Cfg = GemmCfg<BN, SPLIT_BF16X3_PRE>;
  auto kern = gemm_tf32_kernel<BN, EPI, SPLIT_BF16X3_PRE, false, true>;
  static DeviceOnce once;
  const int rc_attr = once.run("kf_gemm_bf16x3_sk", nullptr, [&](int) {
    return cuda_status(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES),
        "kf_gemm_bf16x3_sk: set smem attribute");
  });
  if (rc_attr) return rc_attr;
  return cuda_status(launch_chained(kern, dim3(static_cast<unsigned>(sm_count())),
                                    dim3(Cfg::THREADS), Cfg::SMEM_BYTES, st, ta, tb, tc, C, ldc,
                                    bias, M, N, K, flags, hd, hs, live_tiles, live_count, sk),
                     "kf_gemm_bf16x3_sk launch");
}

// cta_group::2 GEMM: clusters of two CTAs (one 256 x BN tile per pair at a
// time), as many pairs as can be resident at once.
template <int BN, int EPI>
static int launch_gemm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc,
                            float* C, int64_t ldc, const float* bias, int M, int N, int K,
                            int flags, int hd, int hs, const int32_t* live_tiles,
                            const int32_t* live_count, cudaStream_t st) {
  using Cfg = GemmCfg<BN, SPLIT_BF16X3_PRE, true>;
  auto kern = gemm_tf32_kernel<BN, EPI, SPLIT_BF16X3_PRE, true>;
  static DeviceOnce once;
  static int max_pairs[KF_MAX_DEVICES] = {0};
  int dev = 0;
  const int rc_attr = once.run("kf_gemm_bf16x3 (pair)", &dev, [&](int d) {
    const cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return cuda_status(e, "kf_gemm_bf16x3 (pair): set smem attribute");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 8);
    cfg.blockDim = dim3(Cfg::THREADS);
    cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / 2;
    }
    max_pairs[d] = n > 0 ? n : 1;
    return static_cast<int>(KF_OK);
  });
  if (rc_attr) return rc_attr;
  // Units of 256 x BN over all row tiles (the live count is only known on
  // the device; pairs without work exit).
  const int units = (((M + Cfg::BM - 1) / Cfg::BM + 1) / 2) * ((N + BN - 1) / BN);
  const int pairs = units < max_pairs[dev] ? units : max_pairs[dev];
  return cuda_status(
      launch_chained_cluster(kern, dim3(static_cast<unsigned>(2 * pairs)), dim3(Cfg::THREADS),
                             Cfg::SMEM_BYTES, st, 2u, ta, tb, tc, C, ldc, bias, M, N, K, flags, hd,
                             hs, live_tiles, live_count, SkArgs{}),
      "kf_gemm_bf16x3 (pair) launch");
}

static int choose_bn(int64_t M, int64_t N) {
  const int sms = sm_count();
  const int64_t mt = (M + 127) / 128;
  int best = 128;
  double best_cost = 1e30;
  const int cands[3] = {256, 128, 64};
  for (int i = 0; i < 3; ++i) {
    const int bn = cands[i];
    const int64_t tiles = mt * ((N + bn - 1) / bn);
    const int64_t waves = (tiles + sms - 1) / sms;
    const double cost = static_cast<double>(waves) * (bn + 32);
    if (cost < best_cost) {
      best_cost = cost;
      best = bn;
    }
  }
  return best;
}

}  // namespace kf

using namespace kf;

extern "C" int kf_gemm_tf32(const float* A, int64_t lda, const float* W, int64_t ldw,
                            const float* bias, float* C, int64_t ldc, int64_t M, int64_t N,
                            int64_t K, int epilogue, int flags, int bn, int head_dim,
                            int head_stride, const int32_t* live_tiles,
                            const int32_t* live_count, void* stream) {
  if (!A || !W || !C || M < 0 || N < 0 || K < 0) {
    set_last_error("kf_gemm_tf32: invalid arguments");
    return KF_E_INVALID;
  }
  if (M == 0 || N == 0) return KF_OK;
  if (K == 0 || K % 4 || lda % 4 || ldw % 4 || lda < K || ldw < K ||
      (reinterpret_cast<uintptr_t>(A) & 15u) || (reinterpret_cast<uintptr_t>(W) & 15u)) {
    set_last_error(
        "kf_gemm_tf32: TMA needs K %% 4 == 0, lda/ldw %% 4 == 0, lda/ldw >= K and 16-byte "
        "aligned A/W (K=%lld lda=%lld ldw=%lld)",
        (long long)K, (long long)lda, (long long)ldw);
    return KF_E_UNSUPPORTED;
  }
  if (M > INT32_MAX || N > INT32_MAX || K > INT32_MAX) {
    set_last_error("kf_gemm_tf32: dimensions beyond 2^31");
    return KF_E_UNSUPPORTED;
  }
  if (epilogue != KF_EPI_BIAS && epilogue != KF_EPI_BIAS_GELU) {
    set_last_error("kf_gemm_tf32: unknown epilogue %d", epilogue);
    return KF_E_INVALID;
  }
  if (head_dim < 0 || (head_dim > 0 && head_stride < head_dim)) {
    set_last_error("kf_gemm_tf32: head_stride must be >= head_dim");
    return KF_E_INVALID;
  }
  const int64_t out_cols = head_dim > 0 ? ((N + head_dim - 1) / head_dim) * head_stride : N;
  if (ldc < out_cols && M > 1) {
    set_last_error("kf_gemm_tf32: ldc %lld smaller than the output row", (long long)ldc);
    return KF_E_INVALID;
  }
  if ((live_tiles == nullptr) != (live_count == nullptr)) {
    set_last_error("kf_gemm_tf32: live_tiles and live_count go together");
    return KF_E_INVALID;
  }
  if (bn == 0) bn = choose_bn(M, N);
  if (bn != 64 && bn != 128 && bn != 256) {
    set_last_error("kf_gemm_tf32: bn must be 0, 64, 128 or 256");
    return KF_E_INVALID;
  }

  CUtensorMap ta, tb;
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(lda) * 4};
    const uint32_t box[2] = {32, 128};
    int rc = encode_tensor_map(&ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, A, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }
  {
    const uint64_t dims[2] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldw) * 4};
    const uint32_t box[2] = {32, static_cast<uint32_t>(bn)};
    int rc = encode_tensor_map(&tb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, W, dims, strides, box,
                               CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
  }

  int f = flags & KF_GEMM_ROUND_TF32;
  const bool vec = (ldc % 4 == 0) && !(reinterpret_cast<uintptr_t>(C) & 15u) &&
                   !(reinterpret_cast<uintptr_t>(bias) & 15u) &&
                   (head_dim == 0 || (head_dim % 4 == 0 && head_stride % 4 == 0));
  if (vec) f |= KF_GEMM_VEC_OK;
  // TMA-store epilogue for plain row-major outputs (the head-padded scatter
  // and unaligned outputs keep direct stores).
  CUtensorMap tcm;
  memset(&tcm, 0, sizeof(tcm));
  if (vec && head_dim == 0 && (ldc * 4) % 16 == 0) {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldc) * 4};
    const uint32_t box[2] = {32, 128};
    if (encode_tensor_map(&tcm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, C, dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_128B) == KF_OK)
      f |= KF_GEMM_TMA_OUT;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  const int split = (flags & KF_GEMM_BF16X3) ? SPLIT_BF16X3
                    : (flags & KF_GEMM_SPLIT3)  ? SPLIT_TF32X3
                                                : SPLIT_NONE;
  if ((flags & KF_GEMM_BF16X3) && (flags & KF_GEMM_SPLIT3)) {
    set_last_error("kf_gemm_tf32: KF_GEMM_SPLIT3 and KF_GEMM_BF16X3 are exclusive");
    return KF_E_INVALID;
  }
#define KF_GEMM_CASE(BNV)                                                                     \
  if (bn == BNV) {                                                                            \
    if (split == SPLIT_TF32X3) {                                                              \
      if (epilogue == KF_EPI_BIAS)                                                            \
        return launch_gemm<BNV, KF_EPI_BIAS, 1>(ta, tb, tcm, C, ldc, bias, m, n, k, f, head_dim,   \
                                                head_stride, live_tiles, live_count, st);                             \
      return launch_gemm<BNV, KF_EPI_BIAS_GELU, 1>(ta, tb, tcm, C, ldc, bias, m, n, k, f,          \
                                                   head_dim, head_stride, live_tiles, live_count, st);                \
    }                                                                                         \
    if (split == SPLIT_BF16X3) {                                                              \
      if (epilogue == KF_EPI_BIAS)                                                            \
        return launch_gemm<BNV, KF_EPI_BIAS, 2>(ta, tb, tcm, C, ldc, bias, m, n, k, f, head_dim,   \
                                                head_stride, live_tiles, live_count, st);                             \
      return launch_gemm<BNV, KF_EPI_BIAS_GELU, 2>(ta, tb, tcm, C, ldc, bias, m, n, k, f,          \
                                                   head_dim, head_stride, live_tiles, live_count, st);                \
    }                                                                                         \
    if (epilogue == KF_EPI_BIAS)                                                              \
      return launch_gemm<BNV, KF_EPI_BIAS, 0>(ta, tb, tcm, C, ldc, bias, m, n, k, f, head_dim,     \
                                              head_stride, live_tiles, live_count, st);                               \
    return launch_gemm<BNV, KF_EPI_BIAS_GELU, 0>(ta, tb, tcm, C, ldc, bias, m, n, k, f, head_dim,  \
                                                 head_stride, live_tiles, live_count, st);                            \
  }
  KF_GEMM_CASE(64)
  KF_GEMM_CASE(128)
  KF_GEMM_CASE(256)
#undef KF_GEMM_CASE
  return KF_E_INVALID;
}

// Stream-K workspace bytes for an M x N output in N tiles of bn: two fp32
// partial tiles per 128 x bn tile, then two int counters per tile.
static int64_t sk_workspace_bytes(int64_t M, int64_t N, int bn) {
  const int64_t tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
  return tiles * 2 * 128 * bn * 4 + tiles * 2 * 4;
}

static int gemm_bf16x3_impl(const uint16_t* A2, int64_t lda, const uint16_t* W2, int64_t ldw,
                            const float* bias, void* C, int64_t ldc, int64_t M, int64_t N,
                            int64_t K, int epilogue, int flags, int bn, int head_dim,
                            int head_stride, const int32_t* live_tiles,
                            const int32_t* live_count, const SkArgs* sk, void* stream) {
  if (!A2 || !W2 || !C || M < 0 || N < 0 || K < 0) {
    set_last_error("kf_gemm_bf16x3: invalid arguments");
    return KF_E_INVALID;
  }
  if (flags & ~(KF_GEMM_ROUND_TF32 | KF_GEMM_BF16X3 | KF_GEMM_OUT_BF16X2 | KF_GEMM_PAIR |
                KF_GEMM_W_STATIC)) {
    set_last_error("kf_gemm_bf16x3: unknown flags 0x%x", flags);
    return KF_E_INVALID;
  }
  if (M == 0 || N == 0) return KF_OK;
  const bool out_split = (flags & KF_GEMM_OUT_BF16X2) != 0;
  if (K == 0 || K % 8 || lda % 8 || ldw % 8 || lda < K || ldw < K || ldc < N ||
      (reinterpret_cast<uintptr_t>(A2) & 15u) || (reinterpret_cast<uintptr_t>(W2) & 15u) ||
      (reinterpret_cast<uintptr_t>(C) & 15u) || (out_split ? ldc % 8 : ldc % 4) ||
      (bias && (reinterpret_cast<uintptr_t>(bias) & 15u))) {
    set_last_error(
        "kf_gemm_bf16x3: needs K, lda, ldw %% 8 == 0, ldc %% %d == 0, lda/ldw >= K, ldc >= N "
        "and 16-byte aligned pointers (K=%lld lda=%lld ldw=%lld ldc=%lld)",
        out_split ? 8 : 4, (long long)K, (long long)lda, (long long)ldw, (long long)ldc);
    return KF_E_UNSUPPORTED;
  }
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2 || K > INT32_MAX) {
    set_last_error("kf_gemm_bf16x3: dimensions beyond 2^30");
    return KF_E_UNSUPPORTED;
  }
  if (epilogue != KF_EPI_BIAS && epilogue != KF_EPI_BIAS_GELU) {
    set_last_error("kf_gemm_bf16x3: unknown epilogue %d", epilogue);
    return KF_E_INVALID;
  }
  if ((live_tiles == nullptr) != (live_count == nullptr)) {
    set_last_error("kf_gemm_bf16x3: live_tiles and live_count go together");
    return KF_E_INVALID;
  }
  if (head_dim < 0 || (head_dim > 0 && (head_stride < head_dim || out_split))) {
    set_last_error("kf_gemm_bf16x3: head padding needs head_stride >= head_dim and fp32 output");
    return KF_E_INVALID;
  }
  if (bn == 0) bn = choose_bn(M, N);
  if (bn != 64 && bn != 96 && bn != 112 && bn != 128 && bn != 256) {
    set_last_error("kf_gemm_bf16x3: bn must be 0, 64, 96, 112, 128 or 256");
    return KF_E_INVALID;
  }
  if (bn == 112 && (out_split || (flags & KF_GEMM_PAIR))) {
    set_last_error("kf_gemm_bf16x3: bn 112 needs fp32 output and one-CTA tiles");
    return KF_E_INVALID;
  }
  if (sk && (bn == 96 || bn == 112 || (flags & KF_GEMM_PAIR))) {
    set_last_error("kf_gemm_bf16x3_sk: bn must be 64, 128 or 256, without KF_GEMM_PAIR");
    return KF_E_INVALID;
  }
  // k blocks of 64 bf16 (128-byte rows): the x coordinate of every load is a
  // multiple of 64 elements.
  // KF_GEMM_PAIR: cta_group::2 tiles of 256 x bn; each CTA stages bn/2 B rows.
  const bool pair = (flags & KF_GEMM_PAIR) != 0;
  if (pair && bn != 128 && bn != 256) {
    set_last_error("kf_gemm_bf16x3: KF_GEMM_PAIR needs bn 128 or 256");
    return KF_E_INVALID;
  }
  const uint32_t kbox = 64;
  const CUtensorMapSwizzle ksw = CU_TENSOR_MAP_SWIZZLE_128B;
  CUtensorMap ta, tb, tcm;
  memset(&tcm, 0, sizeof(tcm));
  int rc;
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(M), 2};
    const uint64_t strides[2] = {static_cast<uint64_t>(lda) * 2,
                                 static_cast<uint64_t>(M) * static_cast<uint64_t>(lda) * 2};
    const uint32_t box[3] = {kbox, 128, 1};
    rc = encode_tensor_map(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, A2, dims, strides, box, ksw);
    if (rc) return rc;
  }
  {
    const uint64_t dims[3] = {static_cast<uint64_t>(K), static_cast<uint64_t>(N), 2};
    const uint64_t strides[2] = {static_cast<uint64_t>(ldw) * 2,
                                 static_cast<uint64_t>(N) * static_cast<uint64_t>(ldw) * 2};
    const uint32_t box[3] = {kbox, static_cast<uint32_t>(pair ? bn / 2 : bn), 1};
    rc = encode_tensor_map(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, W2, dims, strides, box, ksw);
    if (rc) return rc;
  }
  int f = (flags & (KF_GEMM_ROUND_TF32 | KF_GEMM_W_STATIC)) | KF_GEMM_TMA_OUT;
  if (head_dim == 0 || (head_dim % 4 == 0 && head_stride % 4 == 0)) f |= KF_GEMM_VEC_OK;
  if (head_dim > 0) {
    f &= ~KF_GEMM_TMA_OUT;  // scatter into head-padded slots: direct stores
  } else if (out_split) {
    f = (f & ~KF_GEMM_ROUND_TF32) | KF_GEMM_OUT_SPLIT;
    const uint64_t dims[3] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M), 2};
    const uint64_t strides[2] = {static_cast<uint64_t>(ldc) * 2,
                                 static_cast<uint64_t>(M) * static_cast<uint64_t>(ldc) * 2};
    const uint32_t box[3] = {32, 128, 1};
    rc = encode_tensor_map(&tcm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, C, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_64B);
  } else {
    const uint64_t dims[2] = {static_cast<uint64_t>(N), static_cast<uint64_t>(M)};
    const uint64_t strides[1] = {static_cast<uint64_t>(ldc) * 4};
    const uint32_t box[2] = {32, 128};
    rc = encode_tensor_map(&tcm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, C, dims, strides, box,
                           CU_TENSOR_MAP_SWIZZLE_128B);
  }
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
  float* Cf = static_cast<float*>(C);
  if (sk) {
    if (bn == 64)
      return epilogue == KF_EPI_BIAS
                 ? launch_gemm_sk<64, KF_EPI_BIAS>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f, head_dim,
                                                   head_stride, live_tiles, live_count, *sk, st)
                 : launch_gemm_sk<64, KF_EPI_BIAS_GELU>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f,
                                                        head_dim, head_stride, live_tiles,
                                                        live_count, *sk, st);
    if (bn == 128)
      return epilogue == KF_EPI_BIAS
                 ? launch_gemm_sk<128, KF_EPI_BIAS>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f,
                                                    head_dim, head_stride, live_tiles, live_count,
                                                    *sk, st)
                 : launch_gemm_sk<128, KF_EPI_BIAS_GELU>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f,
                                                         head_dim, head_stride, live_tiles,
                                                         live_count, *sk, st);
    return epilogue == KF_EPI_BIAS
               ? launch_gemm_sk<256, KF_EPI_BIAS>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f, head_dim,
                                                  head_stride, live_tiles, live_count, *sk, st)
               : launch_gemm_sk<256, KF_EPI_BIAS_GELU>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f,
                                                       head_dim, head_stride, live_tiles,
                                                       live_count, *sk, st);
  }
  if (pair) {
    if (bn == 128)
      return epilogue == KF_EPI_BIAS
                 ? launch_gemm_pair<128, KF_EPI_BIAS>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f,
                                                      head_dim, head_stride, live_tiles,
                                                      live_count, st)
                 : launch_gemm_pair<128, KF_EPI_BIAS_GELU>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f,
                                                           head_dim, head_stride, live_tiles,
                                                           live_count, st);
    return epilogue == KF_EPI_BIAS
               ? launch_gemm_pair<256, KF_EPI_BIAS>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f,
                                                    head_dim, head_stride, live_tiles, live_count,
                                                    st)
               : launch_gemm_pair<256, KF_EPI_BIAS_GELU>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f,
                                                         head_dim, head_stride, live_tiles,
                                                         live_count, st);
  }
#define KF_GEMM_PRE_CASE(BNV)                                                                  \
  if (bn == BNV) {                                                                             \
    if (epilogue == KF_EPI_BIAS)                                                               \
      return launch_gemm<BNV, KF_EPI_BIAS, 3>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f,          \
                                              head_dim, head_stride, live_tiles, live_count,   \
                                              st);                                             \
    return launch_gemm<BNV, KF_EPI_BIAS_GELU, 3>(ta, tb, tcm, Cf, ldc, bias, m, n, k, f,       \
                                                 head_dim, head_stride, live_tiles,            \
                                                 live_count, st);                              \
  }
  KF_GEMM_PRE_CASE(64)
  KF_GEMM_PRE_CASE(96)
  KF_GEMM_PRE_CASE(112)
  KF_GEMM_PRE_CASE(128)
  KF_GEMM_PRE_CASE(256)
#undef KF_GEMM_PRE_CASE
  return KF_E_INVALID;
}

extern "C" int kf_gemm_bf16x3(const uint16_t* A2, int64_t lda, const uint16_t* W2, int64_t ldw,
                              const float* bias, void* C, int64_t ldc, int64_t M, int64_t N,
                              int64_t K, int epilogue, int flags, int bn, int head_dim,
                              int head_stride, const int32_t* live_tiles,
                              const int32_t* live_count, void* stream) {
  return gemm_bf16x3_impl(A2, lda, W2, ldw, bias, C, ldc, M, N, K, epilogue, flags, bn, head_dim,
                          head_stride, live_tiles, live_count, nullptr, stream);
}

extern "C" int64_t kf_gemm_sk_workspace_bytes(int64_t M, int64_t N, int bn) {
  if (M <= 0 || N <= 0 || (bn != 64 && bn != 128 && bn != 256)) return 0;
  return sk_workspace_bytes(M, N, bn);
}

extern "C" int kf_gemm_bf16x3_sk(const uint16_t* A2, int64_t lda, const uint16_t* W2, int64_t ldw,
                                 const float* bias, void* C, int64_t ldc, int64_t M, int64_t N,
                                 int64_t K, int epilogue, int flags, int bn, int head_dim,
                                 int head_stride, const int32_t* live_tiles,
                                 const int32_t* live_count, void* workspace,
                                 int64_t workspace_bytes, void* stream) {
  if (bn == 0) bn = 128;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 15u) || bn <= 0 ||
      workspace_bytes < sk_workspace_bytes(M > 0 ? M : 1, N > 0 ? N : 1, bn)) {
    set_last_error("kf_gemm_bf16x3_sk: workspace missing, unaligned or below "
                   "kf_gemm_sk_workspace_bytes");
    return KF_E_INVALID;
  }
  const int64_t tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
  // Partials at the start, counters at the END of the caller's buffer: GEMMs
  // of different shapes can share one workspace sized max(partials) +
  // max(counters) without one's partials landing on another's counters.
  SkArgs sk;
  sk.ws = static_cast<float*>(workspace);
  sk.flags = reinterpret_cast<int*>(static_cast<char*>(workspace) +
                                    ((workspace_bytes - tiles * 2 * 4) & ~static_cast<int64_t>(15)));
  return gemm_bf16x3_impl(A2, lda, W2, ldw, bias, C, ldc, M, N, K, epilogue, flags, bn, head_dim,
                          head_stride, live_tiles, live_count, &sk, stream);
}

