// Attention forward for callers that cannot allocate device memory.
//
// kf_flash_fwd_tf32 reads the packed key bits from a workspace the caller
// allocates (kf_keep_bits_words(B, S) words). Some callers cannot allocate:
//   * serving processes that hand nearly all of a GPU's memory to a fixed
//     arena or pool at start-up, where one more cudaMalloc fails or splits
//     the arena;
//   * latency-bound paths that cannot take the device-wide synchronisation
//     cudaMalloc and cudaFree may imply;
//   * FFI callers (ctypes, cgo, JNI) that own no device allocator at all.
// kf_flash_fwd_tf32_keep_noalloc takes the uint8 keep mask instead and packs
// the bits into a static device array of this library, then runs the same
// two kernels through the existing entry points (kf_keep_bits,
// kf_flash_fwd_tf32). It allocates nothing.
//
// Limits and sharing:
//   * the array holds KF_NOALLOC_KEEP_WORDS_MAX words (1 MiB) on every device
//     that loads the library, until the process exits; B * ceil(S/32) above
//     that is rejected with KF_E_UNSUPPORTED, and so is every argument the
//     attention entry point refuses, before anything is launched;
//   * the first call on a device resolves the array's device address with
//     cudaGetSymbolAddress (the host-side name is only a stand-in, never a
//     device pointer); make that first call before any stream capture. The
//     address is cached per device ordinal for the life of the process: after
//     a cudaDeviceReset it is stale, so do not reset a device this library
//     has used and then call it again;
//   * every call shares the array and it keeps the last call's contents. The
//     packer writes every word the attention kernel then reads (bits past S
//     as 0), so nothing has to start at zero; but calls whose kernels overlap
//     on the GPU (different streams without ordering) race on the array:
//     order them on one stream or with events.
#include <mutex>

#include "kf_common.cuh"

namespace kf {

static __device__ __align__(256) uint32_t g_noalloc_keep_bits[KF_NOALLOC_KEEP_WORDS_MAX];

static std::mutex g_noalloc_mutex;
static uint32_t* g_noalloc_ptr[64] = {nullptr};

// Device address of g_noalloc_keep_bits on the current device (resolved once).
static int noalloc_scratch(uint32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "kf_flash_fwd_tf32_keep_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= 64) {
    set_last_error("kf_flash_fwd_tf32_keep_noalloc: device ordinal %d out of range", dev);
    return KF_E_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_keep_bits);
    if (e != cudaSuccess)
      return cuda_status(e, "kf_flash_fwd_tf32_keep_noalloc: cudaGetSymbolAddress");
    g_noalloc_ptr[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return KF_OK;
}

}  // namespace kf

using namespace kf;

extern "C" int kf_flash_fwd_tf32_keep_noalloc(
    const float* q, int64_t q_sb, int64_t q_sh, int64_t q_sm, const float* k, int64_t k_sb,
    int64_t k_sh, int64_t k_sm, const float* v, int64_t v_sb, int64_t v_sh, int64_t v_sm, float* o,
    int64_t o_sb, int64_t o_sh, int64_t o_sm, const uint8_t* keep, int64_t ld_keep, int64_t B,
    int64_t H, int64_t S, int dh, int dh_out, float sm_scale, int flags, void* stream) {
  if (!q || !k || !v || !o || !keep || B < 0 || H < 0 || S < 0) {
    set_last_error("kf_flash_fwd_tf32_keep_noalloc: invalid arguments");
    return KF_E_INVALID;
  }
  if (B == 0 || H == 0 || S == 0) return KF_OK;
  // Every check of the attention call runs before the key-bit packer is
  // queued, so a rejected call launches nothing and leaves the scratch as
  // it was.
  int kernel_flags = 0;
  int rc = flash_fwd_validate(q, q_sb, q_sh, q_sm, k, k_sb, k_sh, k_sm, v, v_sb, v_sh, v_sm, o,
                              o_sb, o_sh, o_sm, B, H, S, dh, dh_out, flags, &kernel_flags);
  if (rc) return rc;
  if (ld_keep < S) {
    set_last_error("kf_flash_fwd_tf32_keep_noalloc: ld_keep %lld < S %lld", (long long)ld_keep,
                   (long long)S);
    return KF_E_INVALID;
  }
  const size_t words = kf_keep_bits_words(B, S);
  if (words > static_cast<size_t>(KF_NOALLOC_KEEP_WORDS_MAX)) {
    set_last_error(
        "kf_flash_fwd_tf32_keep_noalloc: B * ceil(S/32) = %zu key-bit words exceeds the "
        "static scratch of %d words (1 MiB); use kf_flash_fwd_tf32 with a caller workspace",
        words, KF_NOALLOC_KEEP_WORDS_MAX);
    return KF_E_UNSUPPORTED;
  }
  uint32_t* bits = nullptr;
  rc = noalloc_scratch(&bits);
  if (rc) return rc;
  rc = kf_keep_bits(keep, ld_keep, B, S, bits, stream);
  if (rc) return rc;
  return kf_flash_fwd_tf32(q, q_sb, q_sh, q_sm, k, k_sb, k_sh, k_sm, v, v_sb, v_sh, v_sm, o, o_sb,
                           o_sh, o_sm, bits, B, H, S, dh, dh_out, sm_scale, flags, stream);
}
