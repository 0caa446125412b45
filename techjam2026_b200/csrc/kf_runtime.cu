// Host runtime of the C ABI: error reporting, device status word, tensor-map
// encoding through the driver entry point, and two small utility kernels
// (key-padding bit packing, TF32 rounding).
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "kf_common.cuh"

namespace kf {

static thread_local char t_last_error[512] = {0};

void set_last_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
}

int cuda_status(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return KF_OK;
  set_last_error("%s: %s (%s)", where, cudaGetErrorString(e), cudaGetErrorName(e));
  return KF_E_CUDA;
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

int encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, uint32_t rank, const void* base,
                      const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                      CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!g_encode) {
    set_last_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return KF_E_CUDA;
  }
  cuuint64_t gdim[5];
  cuuint64_t gstride[4];
  cuuint32_t bdim[5];
  cuuint32_t estride[5];
  for (uint32_t i = 0; i < rank; ++i) {
    gdim[i] = dims[i];
    bdim[i] = box[i];
    estride[i] = 1;
    if (i + 1 < rank) gstride[i] = strides_bytes[i];
  }
  CUresult r = g_encode(map, dtype, rank, const_cast<void*>(base), gdim, gstride, bdim, estride,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_last_error("cuTensorMapEncodeTiled failed (CUresult %d, rank %u)", static_cast<int>(r),
                   rank);
    return KF_E_CUDA;
  }
  return KF_OK;
}

int sm_count() {
  static std::atomic<int> cached[KF_MAX_DEVICES];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= KF_MAX_DEVICES) return 148;
  int n = cached[dev].load(std::memory_order_relaxed);
  if (!n) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cached[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

// ---------------------------------------------------------------- kernels

// One warp per 32 keys: ballot of keep != 0 (and k < S).
__global__ void keep_bits_kernel(const uint8_t* __restrict__ keep, int64_t ld_keep, int64_t B,
                                 int64_t S, uint32_t* __restrict__ bits) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t words = (S + 31) / 32;
  const int64_t warp_global = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / 32;
  const int lane = threadIdx.x & 31;
  if (warp_global >= B * words) return;
  const int64_t b = warp_global / words;
  const int64_t w = warp_global % words;
  const int64_t k = w * 32 + lane;
  const bool valid = (k < S) && keep[b * ld_keep + k] != 0;
  const uint32_t m = __ballot_sync(0xffffffffu, valid);
  if (lane == 0) bits[warp_global] = m;
}

// Compact list of the 128-row tiles of [M] keep bytes that hold a live row.
// One CTA of 1024 threads: each pass flags 1024 tiles, a block-wide prefix
// sum places the live ones in ascending order.
__global__ void __launch_bounds__(1024) live_row_tiles_kernel(const uint8_t* __restrict__ keep,
                                                              int64_t M, int32_t* __restrict__ tiles,
                                                              int32_t* __restrict__ count) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int warp_sums[32];
  __shared__ int base;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t n_tiles = (M + 127) / 128;
  if (tid == 0) base = 0;
  __syncthreads();
  for (int64_t t0 = 0; t0 < n_tiles; t0 += 1024) {
    const int64_t t = t0 + tid;
    int live = 0;
    if (t < n_tiles) {
      const int64_t r0 = t * 128;
      const int64_t r1 = (r0 + 128 < M) ? r0 + 128 : M;
      if (r1 - r0 == 128 && (reinterpret_cast<uintptr_t>(keep + r0) & 15u) == 0) {
        const uint4* p = reinterpret_cast<const uint4*>(keep + r0);
        uint32_t acc = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 v = p[i];
          acc |= v.x | v.y | v.z | v.w;
        }
        live = acc != 0;
      } else {
        for (int64_t r = r0; r < r1 && !live; ++r) live = keep[r] != 0;
      }
    }
    // block-wide exclusive prefix sum of `live`
    const unsigned ballot = __ballot_sync(0xffffffffu, live);
    const int in_warp = __popc(ballot & ((1u << lane) - 1u));
    if (lane == 0) warp_sums[warp] = __popc(ballot);
    __syncthreads();
    if (warp == 0) {
      const int v = warp_sums[lane];
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      warp_sums[lane] = incl - v;
    }
    __syncthreads();
    if (live) tiles[base + warp_sums[warp] + in_warp] = static_cast<int32_t>(t);
    __syncthreads();
    if (tid == 1023) base += warp_sums[31] + __popc(ballot);
    __syncthreads();
  }
  if (tid == 0) *count = base;
}

// Packed row order of the valid tokens (kf_pack_rows), step 1 of 2: one CTA.
// A warp counts one batch row's valid keys from its key-bit words; warp 0
// turns each group of 32 counts into row offsets (an exclusive prefix sum
// carried from group to group). Then the tile list of the T packed rows.
__global__ void __launch_bounds__(1024) pack_offsets_kernel(const uint32_t* __restrict__ bits,
                                                            int B, int S,
                                                            int32_t* __restrict__ row_off,
                                                            int32_t* __restrict__ tiles,
                                                            int32_t* __restrict__ tile_count) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int cnt[32];
  __shared__ int run;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int words = (S + 31) >> 5;
  if (tid == 0) run = 0;
  __syncthreads();
  for (int b0 = 0; b0 < B; b0 += 32) {
    const int b = b0 + warp;
    int c = 0;
    if (b < B) {
      const uint32_t* rb = bits + static_cast<int64_t>(b) * words;
      for (int w = lane; w < words; w += 32) c += __popc(rb[w]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    }
    if (lane == 0) cnt[warp] = c;
    __syncthreads();
    if (warp == 0) {
      const int v = cnt[lane];
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      const int r = run;
      if (b0 + lane < B) row_off[b0 + lane] = r + incl - v;
      __syncwarp();
      if (lane == 31) run = r + incl;
    }
    __syncthreads();
  }
  const int T = run;
  const int n = (T + 127) / 128;
  for (int i = tid; i < n; i += 1024) tiles[i] = i;
  if (tid == 0) {
    row_off[B] = T;
    *tile_count = n;
  }
}

// Step 2 of 2: one CTA per batch row writes its entries of the map, 1024
// positions (32 key words, a warp each) at a time; a valid token's packed row
// is the row's offset plus its rank among the row's valid tokens.
__global__ void __launch_bounds__(1024) pack_map_kernel(const uint32_t* __restrict__ bits, int S,
                                                        const int32_t* __restrict__ row_off,
                                                        int32_t* __restrict__ row_map) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int cnt[32], excl[32];
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int words = (S + 31) >> 5;
  const uint32_t* rb = bits + static_cast<int64_t>(b) * words;
  int32_t* out = row_map + static_cast<int64_t>(b) * S;
  int base = row_off[b];
  for (int p0 = 0; p0 < S; p0 += 1024) {
    const int w = (p0 >> 5) + warp;
    const uint32_t word = w < words ? rb[w] : 0u;  // bits past S are 0
    if (lane == 0) cnt[warp] = __popc(word);
    __syncthreads();
    if (warp == 0) {
      const int v = cnt[lane];
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      excl[lane] = incl - v;
    }
    __syncthreads();
    const int pos = p0 + tid;
    if (pos < S)
      out[pos] = ((word >> lane) & 1u)
                     ? base + excl[warp] + __popc(word & ((1u << lane) - 1u))
                     : -1;
    base += excl[31] + cnt[31];
    __syncthreads();  // cnt / excl are rewritten by the next chunk
  }
}

// dst = [2][rows][ld_dst] bf16 planes (hi, then lo) of src [rows][ld_src].
__global__ void split_bf16x2_kernel(const float* __restrict__ src, int64_t rows, int64_t cols,
                                    int64_t ld_src, uint16_t* __restrict__ dst, int64_t ld_dst) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t n = rows * cols;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    const int64_t r = i / cols, c = i % cols;
    uint16_t hi, lo;
    split_bf16(src[r * ld_src + c], hi, lo);
    dst[r * ld_dst + c] = hi;
    dst[rows * ld_dst + r * ld_dst + c] = lo;
  }
}

// Batch rows ranked by valid-key count, longest first (ties by index), from
// the packed key bits: order[rank] = b. One CTA of 1024 threads; the counts
// of up to KF_ORDER_MAX_B rows sit in shared memory, a larger batch gets the
// identity order. A scheduling hint only: attention's results do not depend
// on the order its CTAs run in.
constexpr int KF_ORDER_MAX_B = 4096;

__global__ void __launch_bounds__(1024) batch_order_kernel(const uint32_t* __restrict__ bits,
                                                           int B, int words,
                                                           int32_t* __restrict__ order) {
  pdl_launch_dependents();
  pdl_wait();
  __shared__ int len[KF_ORDER_MAX_B];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  if (B > KF_ORDER_MAX_B) {
    for (int b = threadIdx.x; b < B; b += blockDim.x) order[b] = b;
    return;
  }
  for (int b = warp; b < B; b += nwarps) {
    int n = 0;
    for (int w = lane; w < words; w += 32) n += __popc(bits[static_cast<int64_t>(b) * words + w]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
    if (lane == 0) len[b] = n;
  }
  __syncthreads();
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int lb = len[b];
    int rank = 0;
    for (int c = 0; c < B; ++c) {
      const int lc = len[c];
      rank += (lc > lb) || (lc == lb && c < b);
    }
    order[rank] = b;
  }
}

// Work list of the persistent attention forward (kf_attn_schedule).
//
// sched[0] / sched[1]: the attention kernel's fetch and finish counters
// (zeroed here; the kernel's last CTA zeroes them again, so one list serves
// every layer of a forward); sched[2] = live items, sched[3] = all items;
// items from sched[KF_SCHED_HEADER] as {b * H + h, query tile} pairs.
// Order: batch rows longest first (valid-key count, ties by index), within
// a row its heads in order, within a head the query tiles that hold a valid
// query from the last (heaviest under the causal mask) to the first; after
// every live item, the query tiles without a valid query, in the same row
// and head order. One CTA of 1024 threads, one warp per batch row; rows
// beyond KF_ORDER_MAX_B keep the batch order (no ranking).
constexpr int KF_SCHED_HEADER = 8;
constexpr int KF_SCHED_MAX_B = 16384;

// Does query tile t (128 queries = 4 key-bit words) hold a valid token?
__device__ __forceinline__ bool q_tile_live(const uint32_t* rb, int words, int t) {
  if (!rb) return true;
  uint32_t any = 0;
  const int w0 = t * 4;
#pragma unroll
  for (int w = 0; w < 4; ++w)
    if (w0 + w < words) any |= rb[w0 + w];
  return any != 0;
}

__global__ void __launch_bounds__(1024) attn_schedule_kernel(const uint32_t* __restrict__ bits,
                                                             int B, int H, int S,
                                                             int32_t* __restrict__ sched) {
  pdl_launch_dependents();
  pdl_wait();
  // Dynamic shared memory: three int arrays of B entries.
  extern __shared__ int sh[];
  int* len = sh;           // valid keys per row, then live query tiles per row
  int* order = sh + B;     // order[rank] = row
  int* base = sh + 2 * B;  // first list index of each rank's live items
  __shared__ int totals[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int words = (S + 31) >> 5;
  const int n_qt = (S + 127) >> 7;
  const bool ranked = B <= KF_ORDER_MAX_B;
  if (ranked) {
    for (int b = warp; b < B; b += nwarps) {
      int n = S;
      if (bits) {
        n = 0;
        for (int w = lane; w < words; w += 32) n += __popc(bits[static_cast<int64_t>(b) * words + w]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) n += __shfl_xor_sync(0xffffffffu, n, o);
      }
      if (lane == 0) len[b] = n;
    }
    __syncthreads();
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
      const int lb = len[b];
      int rank = 0;
      for (int c = 0; c < B; ++c) {
        const int lc = len[c];
        rank += (lc > lb) || (lc == lb && c < b);
      }
      order[rank] = b;
    }
  } else {
    for (int b = threadIdx.x; b < B; b += blockDim.x) order[b] = b;
  }
  __syncthreads();
  // Live query tiles per row (one warp per row, a ballot per 32 tiles).
  for (int b = warp; b < B; b += nwarps) {
    const uint32_t* rb = bits ? bits + static_cast<int64_t>(b) * words : nullptr;
    int n = 0;
    for (int t0 = 0; t0 < n_qt; t0 += 32)
      n += __popc(__ballot_sync(0xffffffffu, t0 + lane < n_qt && q_tile_live(rb, words, t0 + lane)));
    if (lane == 0) len[b] = n;  // every warp finished reading len[] before the barrier above
  }
  __syncthreads();
  // List offsets in rank order: warp 0 scans H * live tiles over the ranks.
  if (warp == 0) {
    int run = 0;
    for (int r0 = 0; r0 < B; r0 += 32) {
      const int v = r0 + lane < B ? H * len[order[r0 + lane]] : 0;
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (r0 + lane < B) base[r0 + lane] = run + incl - v;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      totals[0] = run;                   // live items
      totals[1] = B * H * n_qt;          // all items
    }
  }
  __syncthreads();
  const int n_live = totals[0];
  int2* items = reinterpret_cast<int2*>(sched + KF_SCHED_HEADER);
  for (int r = warp; r < B; r += nwarps) {
    const int b = order[r];
    const uint32_t* rb = bits ? bits + static_cast<int64_t>(b) * words : nullptr;
    const int nl = len[b], ne = n_qt - nl;
    // Empty items of this rank start after every live item and the empty
    // items of the ranks before it (which hold H * (n_qt - live) each).
    const int live_base = base[r];
    const int empty_base = n_live + (r * H * n_qt - live_base);
    int seen_l = 0, seen_e = 0;
    for (int t0 = 0; t0 < n_qt; t0 += 32) {
      const int t = t0 + lane;
      const bool in = t < n_qt;
      const bool live = in && q_tile_live(rb, words, t);
      const unsigned bl = __ballot_sync(0xffffffffu, live);
      const unsigned be = __ballot_sync(0xffffffffu, in && !live);
      const unsigned below = (1u << lane) - 1u;
      if (live) {
        const int pos = nl - 1 - (seen_l + __popc(bl & below));  // last tile first
        for (int h = 0; h < H; ++h) items[live_base + h * nl + pos] = make_int2(b * H + h, t);
      } else if (in) {
        const int pos = seen_e + __popc(be & below);
        for (int h = 0; h < H; ++h) items[empty_base + h * ne + pos] = make_int2(b * H + h, t);
      }
      seen_l += __popc(bl);
      seen_e += __popc(be);
    }
  }
  if (threadIdx.x == 0) {
    sched[0] = 0;
    sched[1] = 0;
    sched[2] = n_live;
    sched[3] = totals[1];
  }
}

__global__ void round_tf32_kernel(const float* __restrict__ src, float* __restrict__ dst,
                                  int64_t n) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride)
    dst[i] = round_tf32(src[i]);
}

}  // namespace kf

using namespace kf;

extern "C" int kf_version(void) { return 100; }

extern "C" const char* kf_last_error(void) { return t_last_error; }

extern "C" int kf_device_status(int reset) {
  int v = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return -cuda_status(e, "kf_device_status: synchronize");
  e = cudaMemcpyFromSymbol(&v, g_device_status, sizeof(int));
  if (e != cudaSuccess) return -cuda_status(e, "kf_device_status: read");
  if (reset) {
    int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return -cuda_status(e, "kf_device_status: reset");
  }
  return v;
}

extern "C" int kf_device_status_async(int32_t* host_dst, void* stream) {
  if (!host_dst) {
    set_last_error("kf_device_status_async: host_dst is null");
    return KF_E_INVALID;
  }
  return cuda_status(cudaMemcpyFromSymbolAsync(host_dst, g_device_status, sizeof(int), 0,
                                               cudaMemcpyDeviceToHost,
                                               static_cast<cudaStream_t>(stream)),
                     "kf_device_status_async");
}

extern "C" int kf_set_wait_limit(int64_t cycles) {
  const long long v = cycles > 0 ? static_cast<long long>(cycles) : KF_WAIT_CYCLES;
  return cuda_status(cudaMemcpyToSymbol(g_wait_cycles, &v, sizeof(v)), "kf_set_wait_limit");
}

extern "C" size_t kf_keep_bits_words(int64_t B, int64_t S) {
  if (B <= 0 || S <= 0) return 0;
  return static_cast<size_t>(B) * static_cast<size_t>((S + 31) / 32);
}

extern "C" int kf_keep_bits(const uint8_t* keep, int64_t ld_keep, int64_t B, int64_t S,
                            uint32_t* bits, void* stream) {
  if (!keep || !bits || B <= 0 || S <= 0 || ld_keep < S) {
    set_last_error("kf_keep_bits: invalid arguments (B=%lld S=%lld ld=%lld)", (long long)B,
                   (long long)S, (long long)ld_keep);
    return KF_E_INVALID;
  }
  const int64_t warps = B * ((S + 31) / 32);
  const int threads = 256;
  const int64_t blocks = (warps * 32 + threads - 1) / threads;
  return cuda_status(launch_chained(keep_bits_kernel, dim3(static_cast<unsigned>(blocks)),
                                    dim3(threads), 0, static_cast<cudaStream_t>(stream), keep,
                                    ld_keep, B, S, bits),
                     "kf_keep_bits launch");
}

extern "C" int kf_live_row_tiles(const uint8_t* keep, int64_t M, int32_t* tiles, int32_t* count,
                                 void* stream) {
  if (!keep || !tiles || !count || M < 0 || M > (int64_t)INT32_MAX * 128) {
    set_last_error("kf_live_row_tiles: invalid arguments");
    return KF_E_INVALID;
  }
  return cuda_status(launch_chained(live_row_tiles_kernel, dim3(1), dim3(1024), 0,
                                    static_cast<cudaStream_t>(stream), keep, M, tiles, count),
                     "kf_live_row_tiles launch");
}

extern "C" int kf_pack_rows(const uint32_t* bits, int64_t B, int64_t S, int32_t* row_map,
                            int32_t* row_off, int32_t* tiles, int32_t* tile_count, void* stream) {
  if (!bits || !row_map || !row_off || !tiles || !tile_count || B <= 0 || S <= 0 ||
      B > 65535 || B * S > INT32_MAX) {
    set_last_error("kf_pack_rows: invalid arguments (B=%lld S=%lld)", (long long)B, (long long)S);
    return KF_E_INVALID;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int b = static_cast<int>(B), s = static_cast<int>(S);
  int rc = cuda_status(launch_chained(pack_offsets_kernel, dim3(1), dim3(1024), 0, st, bits, b, s,
                                      row_off, tiles, tile_count),
                       "kf_pack_rows launch (offsets)");
  if (rc) return rc;
  return cuda_status(launch_chained(pack_map_kernel, dim3(static_cast<unsigned>(b)), dim3(1024), 0,
                                    st, bits, s, static_cast<const int32_t*>(row_off), row_map),
                     "kf_pack_rows launch (map)");
}

extern "C" int kf_batch_order(const uint32_t* bits, int64_t B, int64_t S, int32_t* order,
                              void* stream) {
  if (!bits || !order || B <= 0 || S <= 0 || B > INT32_MAX || S > INT32_MAX) {
    set_last_error("kf_batch_order: invalid arguments (B=%lld S=%lld)", (long long)B,
                   (long long)S);
    return KF_E_INVALID;
  }
  const int words = static_cast<int>((S + 31) / 32);
  return cuda_status(launch_chained(batch_order_kernel, dim3(1), dim3(1024), 0,
                                    static_cast<cudaStream_t>(stream), bits,
                                    static_cast<int>(B), words, order),
                     "kf_batch_order launch");
}

extern "C" size_t kf_attn_schedule_words(int64_t B, int64_t H, int64_t S) {
  if (B <= 0 || H <= 0 || S <= 0) return 0;
  return static_cast<size_t>(KF_SCHED_HEADER) +
         2 * static_cast<size_t>(B) * static_cast<size_t>(H) * static_cast<size_t>((S + 127) / 128);
}

extern "C" int kf_attn_schedule(const uint32_t* keep_bits, int64_t B, int64_t H, int64_t S,
                                int32_t* sched, void* stream) {
  if (!sched || B <= 0 || H <= 0 || S <= 0) {
    set_last_error("kf_attn_schedule: invalid arguments (B=%lld H=%lld S=%lld)", (long long)B,
                   (long long)H, (long long)S);
    return KF_E_INVALID;
  }
  if (reinterpret_cast<uintptr_t>(sched) & 7u) {
    set_last_error("kf_attn_schedule: sched must be 8-byte aligned");
    return KF_E_INVALID;
  }
  if (B > KF_SCHED_MAX_B || B * H > 65535 || S > INT32_MAX - 127 ||
      2 * B * H * ((S + 127) / 128) > static_cast<int64_t>(INT32_MAX)) {
    set_last_error("kf_attn_schedule: needs B <= %d, B*H <= 65535 and a list of int32 size",
                   KF_SCHED_MAX_B);
    return KF_E_UNSUPPORTED;
  }
  const size_t smem = 3 * static_cast<size_t>(B) * sizeof(int);
  static DeviceOnce once;
  const int rc = once.run("kf_attn_schedule", nullptr, [&](int) {
    return cuda_status(cudaFuncSetAttribute(attn_schedule_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            3 * KF_SCHED_MAX_B * static_cast<int>(sizeof(int))),
                       "kf_attn_schedule: set smem attribute");
  });
  if (rc) return rc;
  return cuda_status(launch_chained(attn_schedule_kernel, dim3(1), dim3(1024), smem,
                                    static_cast<cudaStream_t>(stream), keep_bits,
                                    static_cast<int>(B), static_cast<int>(H), static_cast<int>(S),
                                    sched),
                     "kf_attn_schedule launch");
}

extern "C" int kf_split_bf16x2(const float* src, int64_t rows, int64_t cols, int64_t ld_src,
                               uint16_t* dst2, int64_t ld_dst, void* stream) {
  if (!src || !dst2 || rows < 0 || cols < 0 || ld_src < cols || ld_dst < cols) {
    set_last_error("kf_split_bf16x2: invalid arguments");
    return KF_E_INVALID;
  }
  if (rows == 0 || cols == 0) return KF_OK;
  const int threads = 256;
  int64_t blocks = (rows * cols + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  return cuda_status(launch_chained(split_bf16x2_kernel, dim3(static_cast<unsigned>(blocks)),
                                    dim3(threads), 0, static_cast<cudaStream_t>(stream), src, rows,
                                    cols, ld_src, dst2, ld_dst),
                     "kf_split_bf16x2 launch");
}

extern "C" int kf_round_tf32(const float* src, float* dst, int64_t n, void* stream) {
  if (!src || !dst || n < 0) {
    set_last_error("kf_round_tf32: invalid arguments");
    return KF_E_INVALID;
  }
  if (n == 0) return KF_OK;
  const int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  return cuda_status(launch_chained(round_tf32_kernel, dim3(static_cast<unsigned>(blocks)),
                                    dim3(threads), 0, static_cast<cudaStream_t>(stream), src, dst,
                                    n),
                     "kf_round_tf32 launch");
}
