// Fused residual-add + padding-mask + LayerNorm (one pass over HBM).
//
//   s = keep[r] ? x[r] + y[r] : 0
//   h = (s - mean) * rsqrt(var_biased + eps) * w + b      (LN of a zero row = b)
//   h = (MASK_OUT && !keep[r]) ? 0 : h
//
// The row mask is a select, not a multiply, so a padded row is exactly 0 even
// if its inputs hold non-finite values (masked_fill semantics of
// torch_transformer_benchmark.py:120-121, 143-144, 170-171).
//
// x and s_out may alias (the residual stream is updated in place): every
// element is read by the thread that later writes it, so no restrict/ldg on
// those two operands.
//
// Work split: one warp per row, each lane owning every 32nd float4 of the row,
// so a warp's loads are fully coalesced 512-byte transactions and the two
// reductions (mean, then centred variance, as nn.LayerNorm computes them) are
// warp shuffles over values already in registers. The row is read once (x and
// y) and written once (s and h): 16*d bytes per row, the HBM floor.
#include "kf_common.cuh"

namespace kf {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Rows of 768 and 1024 floats (NV 6, 8) keep four 256-thread blocks per SM
// (64 registers a thread, no spills): the norm is a memory-latency-bound
// stream, and more rows in flight per SM is what brings it to the copy
// bandwidth (c4: 165.9 -> 135.2 us per norm, 0.95 of the measured copy
// rate). Other widths keep the compiler's choice (at 64 registers NV 4
// would spill).
//
// MAP (kf_ln_add_mask_rows): bit 0 = y of row r is read from row row_map[r]
// (KF_LN_Y_MAPPED), bit 1 = h is written to it (KF_LN_H_MAPPED); an entry of
// -1 means no y and no h for that row. Separate instantiations, so the plain
// norm carries none of it and an h-mapped norm's loads wait on nothing.
template <int NV, int MAP>
__global__ void __launch_bounds__(256, (NV == 6 || NV == 8) ? 4 : 1) ln_add_mask_vec_kernel(
    const float* x, int64_t ldx, const float* y, int64_t ldy, const uint8_t* __restrict__ keep,
    const float* __restrict__ w, const float* __restrict__ b, float* s_out, int64_t lds,
    float* __restrict__ h_out, int64_t ldh, int64_t M,
    int d, float eps, int flags, const int32_t* __restrict__ row_map) {
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  const int nv4 = d >> 2;
  // The kernel is latency-bound (one short row per warp), so every load it
  // needs -- the row's keep byte, x, y and, for rows of up to 512 floats,
  // gamma and beta -- is issued up front instead of one dependent round trip
  // after another; a padded row's loads are simply not used. With
  // KF_LN_STATIC_PARAMS (keep, gamma and beta were written before the
  // previous kernel in the stream started) those go out before the wait on
  // the previous kernel, and a skipped padded row leaves without waiting.
  // Wider rows read gamma and beta (L1-resident) where they are used, which
  // keeps their register count low enough for four blocks per SM.
  constexpr bool PREFETCH_WB = NV <= 4;  // wider rows load gamma/beta where they are used
  constexpr int NW = PREFETCH_WB ? NV : 1;
  const bool early = (flags & KF_LN_STATIC_PARAMS) != 0;
  float4 gw[NW], gb[NW];
  bool kept = true;
  int64_t y_row = row, h_row = row;
  auto load_params = [&]() {
    kept = keep ? (__ldg(keep + row) != 0) : true;
    if constexpr (MAP != 0) {
      const int64_t mr = __ldg(row_map + row);
      if constexpr (MAP & 1) y_row = mr;
      if constexpr (MAP & 2) h_row = mr;
    }
    if (PREFETCH_WB) {
#pragma unroll
      for (int i = 0; i < NW; ++i) {
        const int c = lane + 32 * i;
        gw[i] = gb[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c < nv4) {
          gw[i] = __ldg(reinterpret_cast<const float4*>(w) + c);
          gb[i] = __ldg(reinterpret_cast<const float4*>(b) + c);
        }
      }
    }
  };
  if (early) {
    load_params();
    if (!kept && (flags & KF_LN_SKIP_PADDED)) return;  // reads and writes nothing
  }
  pdl_wait();
  if (!early) load_params();
  // Long rows add y as it arrives (registers for two copies would spill).
  constexpr int NT = PREFETCH_WB ? NV : 1;
  float4 v[NV], t[NT];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (PREFETCH_WB) t[i] = v[i];
    if (c < nv4) {
      v[i] = reinterpret_cast<const float4*>(x + row * ldx)[c];
      if (y && (!(MAP & 1) || y_row >= 0)) {
        const float4 yy = reinterpret_cast<const float4*>(y + y_row * ldy)[c];
        if (PREFETCH_WB) {
          t[i] = yy;
        } else {
          v[i].x += yy.x;
          v[i].y += yy.y;
          v[i].z += yy.z;
          v[i].w += yy.w;
        }
      }
    }
  }
  if (!kept && (flags & KF_LN_SKIP_PADDED)) return;
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (c < nv4 && kept) {
      if (PREFETCH_WB) {
        v[i].x += t[i < NT ? i : 0].x;
        v[i].y += t[i < NT ? i : 0].y;
        v[i].z += t[i < NT ? i : 0].z;
        v[i].w += t[i < NT ? i : 0].w;
      }
      sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    } else {
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  const float inv_d = 1.f / static_cast<float>(d);
  const float mean = warp_sum(sum) * inv_d;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (c < nv4) {
      const float a = v[i].x - mean, bb = v[i].y - mean, cc = v[i].z - mean, dd = v[i].w - mean;
      sq += (a * a + bb * bb) + (cc * cc + dd * dd);
    }
  }
  const float var = warp_sum(sq) * inv_d;
  const float rstd = 1.f / sqrtf(var + eps);
  const bool zero_h = (flags & KF_LN_MASK_OUT) && !kept;
  const bool rnd = (flags & KF_LN_ROUND_TF32) != 0;
  const bool split = (flags & KF_LN_OUT_BF16X2) != 0;
  uint16_t* h_hi = reinterpret_cast<uint16_t*>(h_out) + h_row * ldh;
  uint16_t* h_lo = h_hi + M * ldh;
  const bool write_h = !(MAP & 2) || h_row >= 0;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int c = lane + 32 * i;
    if (c < nv4) {
      if (s_out) reinterpret_cast<float4*>(s_out + row * lds)[c] = v[i];
      if (!write_h) continue;
      float4 h;
      if (zero_h) {
        h = make_float4(0.f, 0.f, 0.f, 0.f);
      } else {
        const float4 ww = PREFETCH_WB ? gw[i < NW ? i : 0] : __ldg(reinterpret_cast<const float4*>(w) + c);
        const float4 bb = PREFETCH_WB ? gb[i < NW ? i : 0] : __ldg(reinterpret_cast<const float4*>(b) + c);
        h.x = (v[i].x - mean) * rstd * ww.x + bb.x;
        h.y = (v[i].y - mean) * rstd * ww.y + bb.y;
        h.z = (v[i].z - mean) * rstd * ww.z + bb.z;
        h.w = (v[i].w - mean) * rstd * ww.w + bb.w;
        if (rnd) {
          h.x = round_tf32(h.x);
          h.y = round_tf32(h.y);
          h.z = round_tf32(h.z);
          h.w = round_tf32(h.w);
        }
      }
      if (split)
        store_split4(h_hi + 4 * c, h_lo + 4 * c, h);
      else
        reinterpret_cast<float4*>(h_out + h_row * ldh)[c] = h;
    }
  }
}

// Generic path (any d, any alignment): three strided passes over the row.
__global__ void __launch_bounds__(256) ln_add_mask_scalar_kernel(
    const float* x, int64_t ldx, const float* y, int64_t ldy, const uint8_t* __restrict__ keep,
    const float* __restrict__ w, const float* __restrict__ b, float* s_out, int64_t lds,
    float* __restrict__ h_out, int64_t ldh, int64_t M,
    int d, float eps, int flags, const int32_t* __restrict__ row_map) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  const bool kept = keep ? (keep[row] != 0) : true;  // (KF_LN_STATIC_PARAMS unused here)
  if (!kept && (flags & KF_LN_SKIP_PADDED)) return;
  const int64_t mrow = row_map ? row_map[row] : row;
  const int64_t y_row = !y ? -1 : ((flags & KF_LN_Y_MAPPED) ? mrow : row);
  const int64_t h_row = (flags & KF_LN_H_MAPPED) ? mrow : row;
  auto val = [&](int c) -> float {
    if (!kept) return 0.f;
    float a = x[row * ldx + c];
    if (y_row >= 0) a += y[y_row * ldy + c];
    return a;
  };
  float sum = 0.f;
  for (int c = lane; c < d; c += 32) sum += val(c);
  const float inv_d = 1.f / static_cast<float>(d);
  const float mean = warp_sum(sum) * inv_d;
  float sq = 0.f;
  for (int c = lane; c < d; c += 32) {
    const float t = val(c) - mean;
    sq += t * t;
  }
  const float rstd = 1.f / sqrtf(warp_sum(sq) * inv_d + eps);
  const bool zero_h = (flags & KF_LN_MASK_OUT) && !kept;
  const bool rnd = (flags & KF_LN_ROUND_TF32) != 0;
  for (int c = lane; c < d; c += 32) {
    const float s = val(c);
    if (s_out) s_out[row * lds + c] = s;
    if (h_row < 0) continue;
    float h = zero_h ? 0.f : (s - mean) * rstd * w[c] + b[c];
    if (rnd && !zero_h) h = round_tf32(h);
    if (flags & KF_LN_OUT_BF16X2) {
      uint16_t hi, lo;
      split_bf16(h, hi, lo);
      reinterpret_cast<uint16_t*>(h_out)[h_row * ldh + c] = hi;
      reinterpret_cast<uint16_t*>(h_out)[M * ldh + h_row * ldh + c] = lo;
    } else {
      h_out[h_row * ldh + c] = h;
    }
  }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace kf

using namespace kf;

static int ln_add_mask_impl(const float* x, int64_t ldx, const float* y, int64_t ldy,
                            const uint8_t* keep, const float* w, const float* b, float* s_out,
                            int64_t lds, float* h_out, int64_t ldh, int64_t M, int64_t d,
                            float eps, int flags, const int32_t* row_map, void* stream) {
  if (!x || !w || !b || !h_out || M < 0 || d <= 0 || ldx < d || ldh < d ||
      (y && ldy < d) || (s_out && lds < d) || d > (1 << 24)) {
    set_last_error("kf_ln_add_mask: invalid arguments (M=%lld d=%lld)", (long long)M,
                   (long long)d);
    return KF_E_INVALID;
  }
  if (M == 0) return KF_OK;
  const int threads = 256;
  const int rows_per_block = threads / 32;
  const unsigned blocks = static_cast<unsigned>((M + rows_per_block - 1) / rows_per_block);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int di = static_cast<int>(d);

  bool vec = (d % 4 == 0) && aligned16(x) && aligned16(w) && aligned16(b) && aligned16(h_out) &&
             ldx % 4 == 0 && ldh % 4 == 0 && d <= 4096;
  if ((flags & KF_LN_OUT_BF16X2) && (flags & KF_LN_ROUND_TF32)) {
    set_last_error("kf_ln_add_mask: KF_LN_OUT_BF16X2 and KF_LN_ROUND_TF32 are exclusive");
    return KF_E_INVALID;
  }
  if (y) vec = vec && aligned16(y) && ldy % 4 == 0;
  if (s_out) vec = vec && aligned16(s_out) && lds % 4 == 0;

  cudaError_t e;
  if (vec) {
    const int nv = (di / 4 + 31) / 32;
    const int map = !row_map ? 0
                             : ((flags & KF_LN_Y_MAPPED) ? 1 : 0) | ((flags & KF_LN_H_MAPPED) ? 2 : 0);
#define KF_LN_LAUNCH_MAP(NV, MAPV)                                                            \
  launch_chained(ln_add_mask_vec_kernel<NV, MAPV>, dim3(blocks), dim3(threads), 0, st, x, ldx, y, \
                 ldy, keep, w, b, s_out, lds, h_out, ldh, M, di, eps, flags, row_map)
#define KF_LN_LAUNCH(NV)                                                                      \
  e = map == 0 ? KF_LN_LAUNCH_MAP(NV, 0)                                                      \
               : map == 1 ? KF_LN_LAUNCH_MAP(NV, 1)                                           \
                          : map == 2 ? KF_LN_LAUNCH_MAP(NV, 2) : KF_LN_LAUNCH_MAP(NV, 3)
    if (nv <= 1)
      KF_LN_LAUNCH(1);
    else if (nv <= 2)
      KF_LN_LAUNCH(2);
    else if (nv <= 4)
      KF_LN_LAUNCH(4);
    else if (nv <= 6)
      KF_LN_LAUNCH(6);
    else if (nv <= 8)
      KF_LN_LAUNCH(8);
    else if (nv <= 16)
      KF_LN_LAUNCH(16);
    else
      KF_LN_LAUNCH(32);
#undef KF_LN_LAUNCH
#undef KF_LN_LAUNCH_MAP
  } else {
    e = launch_chained(ln_add_mask_scalar_kernel, dim3(blocks), dim3(threads), 0, st, x, ldx, y,
                       ldy, keep, w, b, s_out, lds, h_out, ldh, M, di, eps, flags, row_map);
  }
  return cuda_status(e, "kf_ln_add_mask launch");
}

extern "C" int kf_ln_add_mask(const float* x, int64_t ldx, const float* y, int64_t ldy,
                              const uint8_t* keep, const float* w, const float* b, float* s_out,
                              int64_t lds, float* h_out, int64_t ldh, int64_t M, int64_t d,
                              float eps, int flags, void* stream) {
  if (flags & (KF_LN_Y_MAPPED | KF_LN_H_MAPPED)) {
    set_last_error("kf_ln_add_mask: the row-map flags need kf_ln_add_mask_rows");
    return KF_E_INVALID;
  }
  return ln_add_mask_impl(x, ldx, y, ldy, keep, w, b, s_out, lds, h_out, ldh, M, d, eps, flags,
                          nullptr, stream);
}

extern "C" int kf_ln_add_mask_rows(const float* x, int64_t ldx, const float* y, int64_t ldy,
                                   const uint8_t* keep, const float* w, const float* b,
                                   float* s_out, int64_t lds, float* h_out, int64_t ldh,
                                   int64_t M, int64_t d, float eps, int flags,
                                   const int32_t* row_map, void* stream) {
  if (!row_map || !(flags & (KF_LN_Y_MAPPED | KF_LN_H_MAPPED))) {
    set_last_error("kf_ln_add_mask_rows: needs row_map and KF_LN_Y_MAPPED and/or KF_LN_H_MAPPED");
    return KF_E_INVALID;
  }
  return ln_add_mask_impl(x, ldx, y, ldy, keep, w, b, s_out, lds, h_out, ldh, M, d, eps, flags,
                          row_map, stream);
}
