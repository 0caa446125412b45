// tcgen05 FlashAttention forward, TF32 contractions, causal + key-padding
// masks applied in registers.
//
// One CTA = one (batch, head, 128-query tile). Warp roles:
//   warp 0      TMA producer: Q once, then K and V tiles of BN keys through
//               two independent smem rings, each refilled as soon as its slot
//               frees (K once S = QK^T is done, V after O += PV);
//   warp 1      MMA issuer and TMEM owner. TMEM holds two S buffers (BN fp32
//               columns each) and the O accumulator (DH columns). S_j = Q K_j^T
//               is issued as soon as O += P_{j-2} V_{j-2} has been (its buffer
//               is then free), one softmax pass before it is needed; then
//               O += P_{j-1} V_{j-1}, which waits for that softmax. O += P_j V_j
//               reads P straight from TMEM (tcgen05.mma A operand in TMEM), so
//               P never touches shared memory;
//   warps 2-5   softmax: one thread per query row (TMEM lane). Reads its S row,
//               applies scale, causal and key-padding masks, updates the
//               running max, writes P = exp2(S - m) back over S, and rescales
//               its O row only when the max grew by more than 2^8 (the stale
//               max cancels in O / l, so the result is unchanged). At the end
//               it divides by l (0 for a row with no valid key) and stores O.
//
// KV tiles whose keys are all padding are skipped by every role (the three
// roles walk the same list, derived from the packed key bits). With the
// causal mask only tiles up to the diagonal are visited. V is consumed
// MN-major straight from its [S, Dh] layout (no transpose copy), through the
// 32-byte-atom swizzle that MN-major TF32 operands require.
#include <cstring>

#include "kf_common.cuh"

namespace kf {

template <int DH, int BN, int KST, int VST, int MINB = 1>
struct FlashCfg {
  static constexpr int BM = 128;
  static constexpr int RB = (DH * 4 < 128) ? DH * 4 : 128;  // bytes per swizzle row
  static constexpr int CH = RB / 4;                          // fp32 elements per row chunk
  static constexpr int NCH = DH / CH;                        // chunks along Dh
  static constexpr uint32_t LAYOUT =
      RB == 128 ? KF_SWIZZLE_128B : (RB == 64 ? KF_SWIZZLE_64B : KF_SWIZZLE_32B);
  static constexpr int Q_BYTES = BM * DH * 4;
  static constexpr int KV_BYTES = BN * DH * 4;  // one K tile
  // V is read MN-major (Dh contiguous). For 32-bit elements the only MN-major
  // shared-memory layout the tensor core accepts is 128-byte rows with a
  // 32-byte-granule swizzle (descriptor layout SWIZZLE_128B_BASE32B, 4-row
  // atoms), which TMA writes with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B. Rows
  // are 32 elements wide; DH = 16 uses half a row (the rest is zero fill).
  static constexpr int VCH = (DH + 31) / 32;
  static constexpr int V_BYTES = BN * 128 * VCH;  // one V tile
  static constexpr int K_OFF = Q_BYTES;
  static constexpr int V_OFF = K_OFF + KST * KV_BYTES;
  static constexpr int BAR_OFF = V_OFF + VST * V_BYTES;
  // The batch row's packed key bits (one word per 32 keys) are staged in
  // shared memory behind the barriers, as many words as fit beside the tiles
  // with MINB CTAs per SM (each CTA also pays 1 KB of system shared memory);
  // longer rows are read from global memory instead.
  static constexpr int SMEM_CAP = MINB == 1 ? 232448 : 233472 / MINB - 1024;
  static constexpr int BITS_OFF = BAR_OFF + 256;
  static constexpr int BITS_ROOM = (SMEM_CAP - BITS_OFF - 1024) / 4;
  static constexpr int BITS_WORDS = BITS_ROOM >= 2048 ? 2048 : (BITS_ROOM & ~31);
  static constexpr int SMEM_BYTES = BITS_OFF + BITS_WORDS * 4 + 1024;
  // Power-of-two TMEM allocation covering the S buffers and O; with MINB CTAs
  // per SM the allocations must fit the SM's 512 columns together.
  // S buffers in TMEM: with two, S = Q K^T runs one KV tile ahead of the
  // softmax, and a softmax pass is long enough for the next S to be ready
  // when it ends (measured: three buffers were 2-4% slower, their extra TMEM
  // traffic and allocation bought nothing).
  static constexpr int NSB = 2;
  static constexpr int TMEM_NEED = NSB * BN + DH;
  static constexpr int TMEM_COLS = TMEM_NEED <= 32 ? 32 : TMEM_NEED <= 64 ? 64
                                 : TMEM_NEED <= 128 ? 128 : TMEM_NEED <= 256 ? 256 : 512;
  static constexpr int O_COL = NSB * BN;
  static_assert(DH >= 16 && DH <= 256 && (DH & (DH - 1)) == 0, "DH");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 128, "BN");
  static_assert(NSB * BN + DH <= 512, "TMEM");
  // The producer reuses a K slot on the s_full phase of the tile KST back and
  // a V slot on the o_done phase of the tile VST back; those parity tests are
  // exact only with KST <= NSB and VST <= 2.
  static_assert(KST <= NSB && VST <= 2, "ring depths");
  static_assert(BITS_WORDS >= 32, "key-bit staging");
  static_assert(SMEM_BYTES <= SMEM_CAP, "smem");
  static_assert(TMEM_COLS * MINB <= 512, "TMEM");
};

// Does KV tile j (keys [j*BN, j*BN+BN)) hold at least one valid key? `kb`
// is the row's key bits, staged in shared memory or in global memory.
template <int BN>
__device__ __forceinline__ bool kv_tile_live(const uint32_t* kb, int words, int j, int S) {
  const int k0 = j * BN;
  if (k0 >= S) return false;
  if (!kb) return true;
  const int w0 = k0 >> 5;
  uint32_t any = 0;
#pragma unroll
  for (int w = 0; w < BN / 32; ++w)
    if (w0 + w < words) any |= kb[w0 + w];
  return any != 0;
}

// Masks one query row of a key tile: s[c] becomes -inf unless key k0 + c is
// valid (its bit in the tile's words kw) and k0 + c < k0 + limit, where the
// limit is S (or, causal, min(S, query + 1)) minus k0. One 32-bit valid mask
// per word, then one select per score: the cost of a masked tile stays
// close to that of an unmasked one.
template <int BN>
__device__ __forceinline__ void mask_scores(float (&s)[BN], const uint32_t* kw, int limit) {
#pragma unroll
  for (int w = 0; w < BN / 32; ++w) {
    const int lw = limit - 32 * w;
    const uint32_t vb = kw[w] & (lw >= 32 ? 0xffffffffu : (lw <= 0 ? 0u : ((1u << lw) - 1u)));
#pragma unroll
    for (int c = 0; c < 32; ++c) s[32 * w + c] = ((vb >> c) & 1u) ? s[32 * w + c] : -INFINITY;
  }
}

// Internal flag: O is written through the tmO tensor map (TMA stores).
constexpr int KF_ATTN_TMA_OUT = 1 << 9;

template <int DH, int BN, int KST, int VST, int MINB>
__global__ void __launch_bounds__(192, MINB)
    flash_fwd_tf32_kernel(const __grid_constant__ CUtensorMap tmQ,
                          const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV,
                          const __grid_constant__ CUtensorMap tmO, float* __restrict__ O,
                          int64_t o_sb, int64_t o_sh, int64_t o_sm,
                          const uint32_t* __restrict__ keep_bits,
                          const int32_t* __restrict__ batch_order, int H, int S, int dh_out,
                          float scale_log2, int flags) {
  using Cfg = FlashCfg<DH, BN, KST, VST, MINB>;
  constexpr int BM = Cfg::BM;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + Cfg::K_OFF;
  uint8_t* sV = smem + Cfg::V_OFF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::BAR_OFF);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* v_full = k_full + KST;
  uint64_t* s_full = v_full + VST;        // [NSB]
  uint64_t* p_full = s_full + Cfg::NSB;   // [NSB]
  uint64_t* o_done = p_full + Cfg::NSB;   // [2]: P V products of even / odd index
  uint64_t* o_final = o_done + 2;
  uint64_t* drain = o_final + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Grid (query tiles, heads): blocks launch in linear order, so the query
  // tiles of one (b, h) run together and share its K/V in L2 (a long
  // sequence's K/V is 32 MB per head -- streaming every head at once would
  // re-read K/V from HBM for every query tile). Within a head the heaviest
  // causal tiles go first. With a batch order (kf_batch_order: rows by
  // valid length, longest first) grid row y / H runs batch row
  // batch_order[y / H], so the longest rows' heavy tiles start first and the
  // launch ends on short ones; it is read after the wait on the previous
  // kernel.
  const int bh = blockIdx.y;
  const int h = bh % H;
  const int nb = static_cast<int>(gridDim.y) / H;
  const int n_qt = gridDim.x;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);
  const int q0 = qt * BM;
  const bool causal = (flags & KF_ATTN_CAUSAL) != 0;
  const bool split = (flags & KF_ATTN_OUT_BF16X2) != 0;
  const int words = (S + 31) >> 5;

  // Set-up that reads nothing an earlier kernel writes (barriers, TMEM,
  // descriptor prefetch) runs before the wait on the previous kernel, so it
  // overlaps that kernel's tail.
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KST; ++s) {
      mbar_init(&k_full[s], 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(&v_full[s], 1);
    }
    for (int s = 0; s < Cfg::NSB; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 4);
    }
    mbar_init(&o_done[0], 1);
    mbar_init(&o_done[1], 1);
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    if (flags & KF_ATTN_TMA_OUT) tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // The next kernel is released only once every CTA of this one holds its
  // TMEM, so a CTA of the next kernel that allocates TMEM before its own wait
  // can only ever wait for columns that a running CTA will free.
  pdl_launch_dependents();
  pdl_wait();  // Q/K/V, the key bits and the batch order come from earlier kernels
  int b = bh / H;
  if (batch_order) {
    // An entry outside [0, B) (an order array not made by kf_batch_order
    // for this B) is never used as an index: the row keeps its grid
    // position and the device status records the error.
    const int ob = __ldg(batch_order + b);
    if (ob >= 0 && ob < nb) {
      b = ob;
    } else if (threadIdx.x == 0) {
      record_device_status(KF_DEV_BAD_BATCH_ORDER);
    }
  }
  const uint32_t* bits_b = keep_bits ? keep_bits + static_cast<int64_t>(b) * words : nullptr;

  const int n_kv_all = (S + BN - 1) / BN;
  int kv_end = n_kv_all;
  if (causal) {
    const int last_q = (q0 + BM - 1 < S - 1) ? q0 + BM - 1 : S - 1;
    const int lim = last_q / BN + 1;
    kv_end = lim < kv_end ? lim : kv_end;
  }

  // Stage the key bits of keys [0, kv_end * BN) once; every role then tests
  // tiles and masks keys from shared memory. The staged range holds the
  // query tile's own words (kv_end * BN > its last query), so the same loads
  // tell whether the tile has a valid query and the optional skip of a tile
  // without one (rows later masked) costs no second round trip to memory.
  const uint32_t* kb = bits_b;
  int any_q = 0;
  if (bits_b) {
    const int qw0 = q0 >> 5;
    const int qw1 = ((q0 + BM) >> 5) < words ? ((q0 + BM) >> 5) : words;
    const int need = (kv_end * BN + 31) >> 5;
    const int nw = need < words ? need : words;
    if (nw <= Cfg::BITS_WORDS) {
      uint32_t* sbits = reinterpret_cast<uint32_t*>(smem + Cfg::BITS_OFF);
      for (int w = threadIdx.x; w < nw; w += blockDim.x) {
        const uint32_t v = __ldg(bits_b + w);
        sbits[w] = v;
        if (w >= qw0 && w < qw1 && v) any_q = 1;
      }
      kb = sbits;
    } else {
      for (int w = qw0 + threadIdx.x; w < qw1; w += blockDim.x)
        if (__ldg(bits_b + w)) any_q = 1;
    }
  }
  const bool skip = __syncthreads_or(any_q) == 0 && (flags & KF_ATTN_SKIP_EMPTY_Q) && bits_b;

  if (skip) {
    // Zero rows, written coalesced: one 32-row box of zeros in shared memory
    // stored by TMA over every box of the tile, or whole rows by all threads.
    if (flags & KF_ATTN_TMA_OUT) {
      if (warp == 0) {
        float4* z = reinterpret_cast<float4*>(sQ);
        for (int i = lane; i < 32 * 128 / 16; i += 32) z[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int rg = 0; rg < BM / 32 && q0 + rg * 32 < S; ++rg) {
            if (!split) {
              for (int c = 0; c < DH / 32; ++c) tma_store_4d(&tmO, sQ, c * 32, q0 + rg * 32, h, b);
            } else {
              for (int pl = 0; pl < 2; ++pl)
                for (int c = 0; c < DH / 64; ++c)
                  tma_store_4d(&tmO, sQ, c * 64, q0 + rg * 32, h, b + pl * nb);
            }
          }
          bulk_commit_group();
          bulk_wait_group_read<0>();  // the zero box is read; the writes finish with the grid
        }
      }
    } else {
      const int rows = (S - q0 < BM) ? S - q0 : BM;
      const int n = rows * dh_out;
      const int64_t base = static_cast<int64_t>(b) * o_sb + static_cast<int64_t>(h) * o_sh +
                           static_cast<int64_t>(q0) * o_sm;
      for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const int r = i / dh_out;
        const int64_t off = base + static_cast<int64_t>(r) * o_sm + (i - r * dh_out);
        if (split) {
          uint16_t* ohi = reinterpret_cast<uint16_t*>(O);
          ohi[off] = 0;
          ohi[off + static_cast<int64_t>(nb) * o_sb] = 0;
        } else {
          O[off] = 0.f;
        }
      }
    }
  } else if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      mbar_arrive_expect_tx(q_full, Cfg::Q_BYTES);
#pragma unroll
      for (int c = 0; c < Cfg::NCH; ++c)
        tma_load_4d(sQ + c * BM * Cfg::RB, &tmQ, q_full, c * Cfg::CH, q0, h, b);
      // K and V advance independently: the next K tile is loaded as soon as
      // its ring slot is free, without queueing behind the V slot, which
      // frees only after the slower P V product. One thread polls both rings.
      // A K slot is free once S of the tile KST back has completed (its
      // s_full phase), a V slot once P V of the tile VST back has (its o_done
      // phase); no separate release barriers. Loads go out in tile order, so
      // each of those barriers is at most one phase behind the one tested and
      // the parity test is exact.
      int ks = 0, vs = 0;
      long long k_issued = 0, v_issued = 0;
      bool ok = true;
      auto k_slot_free = [&]() -> bool {
        if (k_issued < KST) return true;
        const long long i = k_issued - KST;
        return mbar_test_wait(&s_full[i % Cfg::NSB], static_cast<uint32_t>((i / Cfg::NSB) & 1));
      };
      auto v_slot_free = [&]() -> bool {
        if (v_issued < VST) return true;
        const long long i = v_issued - VST;
        return mbar_test_wait(&o_done[i & 1], static_cast<uint32_t>((i >> 1) & 1));
      };
      auto next_live = [&](int j) {
        while (j < kv_end && !kv_tile_live<BN>(kb, words, j, S)) ++j;
        return j;
      };
      int jk = next_live(0), jv = jk;
      long long t_idle = clock64();
      while (jk < kv_end || jv < kv_end) {
        bool progress = false;
        if (jk < kv_end && k_slot_free()) {
          mbar_arrive_expect_tx(&k_full[ks], Cfg::KV_BYTES);
#pragma unroll
          for (int c = 0; c < Cfg::NCH; ++c)
            tma_load_4d(sK + ks * Cfg::KV_BYTES + c * BN * Cfg::RB, &tmK, &k_full[ks], c * Cfg::CH,
                        jk * BN, h, b);
          ++k_issued;
          if (++ks == KST) ks = 0;
          jk = next_live(jk + 1);
          progress = true;
        }
        if (jv < kv_end && v_slot_free()) {
          mbar_arrive_expect_tx(&v_full[vs], Cfg::V_BYTES);
#pragma unroll
          for (int c = 0; c < Cfg::VCH; ++c)
            tma_load_4d(sV + vs * Cfg::V_BYTES + c * BN * 128, &tmV, &v_full[vs], c * 32, jv * BN, h,
                        b);
          ++v_issued;
          if (++vs == VST) vs = 0;
          jv = next_live(jv + 1);
          progress = true;
        }
        if (progress) {
          t_idle = clock64();
          continue;
        }
        // Nothing to issue: back off briefly so the poll does not take issue
        // slots from the softmax warp that shares this scheduler.
        __nanosleep(64);
        if (*abort_flag) {
          ok = false;
          break;
        } else if (clock64() - t_idle > wait_limit()) {
          *abort_flag = 1;
          record_device_status(KF_DEV_WAIT_TIMEOUT_TMA);
          ok = false;
          break;
        }
      }
      if (!ok) {
        mbar_wait_drain(q_full, 0, KF_DEV_WAIT_TIMEOUT_TMA);
        for (long long i = (k_issued > KST ? k_issued - KST : 0); i < k_issued; ++i)
          mbar_wait_drain(&k_full[i % KST], static_cast<uint32_t>((i / KST) & 1),
                            KF_DEV_WAIT_TIMEOUT_TMA);
        for (long long i = (v_issued > VST ? v_issued - VST : 0); i < v_issued; ++i)
          mbar_wait_drain(&v_full[i % VST], static_cast<uint32_t>((i / VST) & 1),
                            KF_DEV_WAIT_TIMEOUT_TMA);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_s = make_idesc_tf32(BM, BN, 0, 0);
      constexpr uint32_t idesc_o = make_idesc_tf32(BM, DH, 0, 1);
      const uint32_t sQa = smem_u32(sQ);
      const uint32_t sKa = smem_u32(sK);
      const uint32_t sVa = smem_u32(sV);
      int ks = 0, vs = 0;
      uint32_t kph = 0, vph = 0;
      bool ok = mbar_wait(q_full, 0, abort_flag, KF_DEV_WAIT_TIMEOUT_MMA);
      int it = 0;
      auto issue_pv = [&](int i) -> bool {
        const int sb = i % Cfg::NSB;
        if (!mbar_wait(&p_full[sb], static_cast<uint32_t>((i / Cfg::NSB) & 1), abort_flag,
                       KF_DEV_WAIT_TIMEOUT_MMA))
          return false;
        if (!mbar_wait(&v_full[vs], vph, abort_flag, KF_DEV_WAIT_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t vbase = sVa + vs * Cfg::V_BYTES;
#pragma unroll
        for (int kk = 0; kk < BN / 8; ++kk) {
          // 8 keys = 8 rows of 128 bytes; LBO = next 32-wide Dh chunk,
          // SBO = next 4-row swizzle atom.
          const uint64_t bd =
              make_smem_desc(vbase + kk * 8 * 128, BN * 128, 4 * 128, KF_SWIZZLE_128B_BASE32B);
          mma_tf32_ts(tmem_base + Cfg::O_COL, tmem_base + sb * BN + kk * 8, bd, idesc_o,
                      (i > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&o_done[i & 1]);
        if (++vs == VST) {
          vs = 0;
          vph ^= 1u;
        }
        return true;
      };
      for (int j = 0; j < kv_end && ok; ++j) {
        if (!kv_tile_live<BN>(kb, words, j, S)) continue;
        // S_it first: its buffer (it % NSB) last held P of tile it - NSB,
        // whose P V was issued in an earlier iteration, and the pipe runs in
        // issue order, so S_it needs no wait on any softmax. It goes out as
        // soon as P V of tile it - NSB has, i.e. NSB - 1 softmax passes
        // before the softmax needs it.
        if (!mbar_wait(&k_full[ks], kph, abort_flag, KF_DEV_WAIT_TIMEOUT_MMA)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int sb = it % Cfg::NSB;
        const uint32_t kbase = sKa + ks * Cfg::KV_BYTES;
#pragma unroll
        for (int kk = 0; kk < DH / 8; ++kk) {
          const int chunk = kk / (Cfg::CH / 8);
          const int within = kk % (Cfg::CH / 8);
          const uint64_t ad = make_smem_desc(sQa + chunk * BM * Cfg::RB + within * 32, 16,
                                             8 * Cfg::RB, Cfg::LAYOUT);
          const uint64_t bd = make_smem_desc(kbase + chunk * BN * Cfg::RB + within * 32, 16,
                                             8 * Cfg::RB, Cfg::LAYOUT);
          mma_tf32_ss(tmem_base + sb * BN, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[sb]);
        if (++ks == KST) {
          ks = 0;
          kph ^= 1u;
        }
        ++it;
        // Then P V of tile it - NSB (counting the S just issued): it waits
        // for that tile's softmax only.
        if (it >= Cfg::NSB && !issue_pv(it - Cfg::NSB)) {
          ok = false;
          break;
        }
      }
      for (int i = (it >= Cfg::NSB ? it - Cfg::NSB + 1 : 0); ok && i < it; ++i)
        ok = issue_pv(i);
      if (ok && it > 0) mma_commit(o_final);
      mma_commit(drain);
      mbar_wait_drain(drain, 0, KF_DEV_WAIT_TIMEOUT_MMA);
    }
  } else {
    // -------------------------------------------------- softmax (warps 2..5)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int qi = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_row = tmem_base + lane_off;
    float m_run = -INFINITY;
    float l_run = 0.f;
    int it = 0;
    bool ok = true;
    for (int j = 0; j < kv_end; ++j) {
      if (!kv_tile_live<BN>(kb, words, j, S)) continue;
      const int sb = it % Cfg::NSB;
      if (!mbar_wait(&s_full[sb], static_cast<uint32_t>((it / Cfg::NSB) & 1), abort_flag,
                     KF_DEV_WAIT_TIMEOUT_SOFTMAX)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[BN];
      // One TMEM round trip for the row's BN scores (x64 form when BN == 64).
      if constexpr (BN == 64) {
        tmem_ld64(t_row + sb * BN, s);
      } else {
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          tmem_ld32(t_row + sb * BN + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
      }

      const int k0 = j * BN;
      uint32_t kw[BN / 32];
      bool all_keys = (k0 + BN <= S);
#pragma unroll
      for (int w = 0; w < BN / 32; ++w) {
        const int wi = (k0 >> 5) + w;
        kw[w] = kb ? (wi < words ? kb[wi] : 0u) : 0xffffffffu;
        all_keys = all_keys && (kw[w] == 0xffffffffu);
      }
      const bool diag = causal && (k0 + BN - 1 > q0);
      // Row max of the raw scores (the scale is positive, so it commutes
      // with max and rounding is monotonic), then P = 2^(s*scale - m) with
      // the scale folded into one FMA. Masked keys hold -inf and give P = 0.
      // Eight partial maxima / sums keep the dependency chains short.
      if (!(all_keys && !diag))
        mask_scores<BN>(s, kw, (causal && qi + 1 < S ? qi + 1 : S) - k0);
      // Eight partial maxima, two new scores per three-input max.
      float mp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mp[u] = fmaxf(s[u], s[u + 8]);
#pragma unroll
      for (int c = 16; c + 16 <= BN; c += 16) {
#pragma unroll
        for (int u = 0; u < 8; ++u) mp[u] = fmax3(mp[u], s[c + u], s[c + 8 + u]);
      }
      const float mx = fmax3(fmax3(mp[0], mp[1], mp[2]), fmax3(mp[3], mp[4], mp[5]),
                             fmaxf(mp[6], mp[7])) *
                       scale_log2;
      // Running max with lazy rescale: keep the old reference unless the new
      // max exceeds it by more than 8 (P stays <= 256 in fp32).
      float alpha = 1.f;
      bool rescale_o = false;
      if (mx > m_run + 8.f) {
        if (m_run != -INFINITY) {
          alpha = fast_exp2(m_run - mx);
          l_run *= alpha;
          rescale_o = (it > 0);
        }
        m_run = mx;
      }
      const float neg_m = (m_run == -INFINITY) ? 0.f : -m_run;
      // Scores two at a time: one f32x2 FMA for s * scale - m and one f32x2
      // add into four packed partial sums (the same eight sums, indexed by
      // c mod 8, as scalar code would keep).
      const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
      const uint64_t nm2 = f2_pack(neg_m, neg_m);
      uint64_t sp2[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) sp2[u] = f2_pack(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < BN; c += 2) {
        float t0, t1;
        f2_unpack(f2_fma(f2_pack(s[c], s[c + 1]), sc2, nm2), t0, t1);
        // P is truncated to TF32 here (one AND, as the tensor core would
        // truncate it) and l sums exactly the values the product uses, so
        // the common relative shortfall cancels in O / l and the weights stay
        // unbiased, with the error spread of rounding to nearest.
        const float p0 = __uint_as_float(__float_as_uint(fast_exp2(t0)) & 0xffffe000u);
        const float p1 = __uint_as_float(__float_as_uint(fast_exp2(t1)) & 0xffffe000u);
        s[c] = p0;
        s[c + 1] = p1;
        sp2[(c >> 1) & 3] = f2_add(sp2[(c >> 1) & 3], f2_pack(p0, p1));
      }
      float sp[8];
#pragma unroll
      for (int u = 0; u < 4; ++u) f2_unpack(sp2[u], sp[2 * u], sp[2 * u + 1]);
      l_run += ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
      if (__any_sync(0xffffffffu, rescale_o)) {
        // O += P_{it-1} V_{it-1} must have landed before this row is rescaled.
        // The s_full arrival just observed implies PV_{it-NSB}, hence PV_{it-3},
        // is complete (the MMA pipe completes in issue order and S_it was
        // issued after PV_{it-NSB}).
        // o_done[(it-1) & 1] counts the products of that parity (PV_{it-3},
        // PV_{it-1}, ...), so it is at most one phase (PV_{it-1} itself)
        // behind and the parity wait is exact.
        if (!mbar_wait(&o_done[(it - 1) & 1], static_cast<uint32_t>(((it - 1) >> 1) & 1),
                       abort_flag, KF_DEV_WAIT_TIMEOUT_SOFTMAX)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // DH == 16 uses one 32-column access: the 16 columns past O are
        // unused TMEM, so scaling them is harmless.
#pragma unroll
        for (int c = 0; c < (DH + 31) / 32; ++c) {
          float o[32];
          tmem_ld32(t_row + Cfg::O_COL + c * 32, o);
#pragma unroll
          for (int t = 0; t < 32; ++t) o[t] *= alpha;
          tmem_st32(t_row + Cfg::O_COL + c * 32, o);
        }
      }
      if constexpr (BN == 64) {
        tmem_st64(t_row + sb * BN, s);
      } else {
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          tmem_st32(t_row + sb * BN + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
      ++it;
    }
    if (ok) {
      float* orow = O + static_cast<int64_t>(b) * o_sb + static_cast<int64_t>(h) * o_sh +
                    static_cast<int64_t>(qi) * o_sm;
      const bool rnd = (flags & KF_ATTN_ROUND_TF32) != 0;
      // Split output: bf16 hi plane at O (bf16 elements, same strides), lo
      // plane B * o_sb elements further.
      uint16_t* ohi = reinterpret_cast<uint16_t*>(O) + static_cast<int64_t>(b) * o_sb +
                      static_cast<int64_t>(h) * o_sh + static_cast<int64_t>(qi) * o_sm;
      uint16_t* olo = ohi + static_cast<int64_t>(nb) * o_sb;
      if (it > 0) {
        // o_final (one phase) rather than o_done: by now o_done may be two
        // phases behind, where a parity wait cannot tell the phases apart.
        if (mbar_wait(o_final, 0, abort_flag, KF_DEV_WAIT_TIMEOUT_SOFTMAX)) {
          tc_fence_after();
          const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
          if (flags & KF_ATTN_TMA_OUT) {
            // The Q buffer is idle once o_final has fired (every MMA reading
            // it has completed). Each warp stages its 32 rows there in the
            // 128-byte-swizzled layout of the output map, chunk by chunk, and
            // one lane stores them: fp32 chunks of 32 columns, or bf16 hi/lo
            // planes of 64 columns (the lo plane is batch index b + B of the
            // same map).
            const int rows0 = q0 + quarter * 32;
            const uint32_t sw = static_cast<uint32_t>(lane & 7);
#pragma unroll 1
            for (int c = 0; c < DH / 32; ++c) {
              float o[32];
              tmem_ld32(t_row + Cfg::O_COL + c * 32, o);
              if (!split) {
#pragma unroll
                for (int t = 0; t < 32; ++t) o[t] = rnd ? round_tf32(o[t] * inv_l) : o[t] * inv_l;
                uint8_t* rowp = sQ + c * BM * 128 + quarter * 32 * 128 + lane * 128;
#pragma unroll
                for (int u = 0; u < 8; ++u)
                  *reinterpret_cast<float4*>(rowp + ((u ^ sw) << 4)) =
                      make_float4(o[4 * u], o[4 * u + 1], o[4 * u + 2], o[4 * u + 3]);
              } else {
                uint8_t* hrow = sQ + (c >> 1) * BM * 128 + quarter * 32 * 128 + lane * 128;
                uint8_t* lrow = hrow + BM * DH * 2;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                  uint32_t hw[4], lw[4];
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    // O / l and the hi/lo split, two columns per packed op
                    float a, bb;
                    f2_unpack(f2_mul(f2_pack(o[8 * u + 2 * e], o[8 * u + 2 * e + 1]),
                                     f2_pack(inv_l, inv_l)),
                              a, bb);
                    split_bf16x2(a, bb, hw[e], lw[e]);
                  }
                  const uint32_t off = ((static_cast<uint32_t>((c & 1) * 4 + u)) ^ sw) << 4;
                  *reinterpret_cast<uint4*>(hrow + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                  *reinterpret_cast<uint4*>(lrow + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
                }
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && rows0 < S) {
              if (!split) {
                for (int c = 0; c < DH / 32; ++c)
                  tma_store_4d(&tmO, sQ + c * BM * 128 + quarter * 32 * 128, c * 32, rows0, h, b);
              } else {
                for (int pl = 0; pl < 2; ++pl)
                  for (int c = 0; c < DH / 64; ++c)
                    tma_store_4d(&tmO, sQ + pl * BM * DH * 2 + c * BM * 128 + quarter * 32 * 128,
                                 c * 64, rows0, h, b + pl * nb);
              }
              bulk_commit_group();
              bulk_wait_group_read<0>();  // staging read; the writes finish with the grid
            }
          } else {
#pragma unroll 1
          for (int c = 0; c < (DH + 31) / 32; ++c) {
            float o[32];
            tmem_ld32(t_row + Cfg::O_COL + c * 32, o);
            if (qi < S) {
#pragma unroll
              for (int t = 0; t < 32; t += 4) {
                const int col = c * 32 + t;
                if (col < dh_out) {
                  float4 v4 = make_float4(o[t] * inv_l, o[t + 1] * inv_l, o[t + 2] * inv_l,
                                          o[t + 3] * inv_l);
                  if (rnd) {
                    v4.x = round_tf32(v4.x);
                    v4.y = round_tf32(v4.y);
                    v4.z = round_tf32(v4.z);
                    v4.w = round_tf32(v4.w);
                  }
                  if (split) {
                    if (col + 3 < dh_out) {
                      store_split4(ohi + col, olo + col, v4);
                    } else {
                      const float tmp[4] = {v4.x, v4.y, v4.z, v4.w};
                      for (int u = 0; u < 4 && col + u < dh_out; ++u)
                        split_bf16(tmp[u], ohi[col + u], olo[col + u]);
                    }
                  } else if (col + 3 < dh_out && (flags & (1 << 8))) {
                    *reinterpret_cast<float4*>(orow + col) = v4;
                  } else {
                    const float tmp[4] = {v4.x, v4.y, v4.z, v4.w};
                    for (int u = 0; u < 4 && col + u < dh_out; ++u) orow[col + u] = tmp[u];
                  }
                }
              }
            }
          }
          }
        }
      } else if (qi < S) {
        for (int c = 0; c < dh_out; ++c) {
          if (split) {
            ohi[c] = 0;
            olo[c] = 0;
          } else {
            orow[c] = 0.f;
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

template <int DH, int BN, int KST, int VST, int MINB>
static int launch_flash(const float* q, const int64_t* qs, const float* k, const int64_t* ks,
                        const float* v, const int64_t* vs, float* o, const int64_t* os,
                        const uint32_t* bits, const int32_t* order, int B, int H, int S,
                        int dh_stored, int dh_out, float scale_log2, int flags, cudaStream_t st) {
  using Cfg = FlashCfg<DH, BN, KST, VST, MINB>;
  CUtensorMap tq, tk, tv;
  const uint64_t dims[4] = {static_cast<uint64_t>(dh_stored), static_cast<uint64_t>(S),
                            static_cast<uint64_t>(H), static_cast<uint64_t>(B)};
  auto enc = [&](CUtensorMap* m, const float* base, const int64_t* s, uint32_t rows) {
    // strides (in bytes) of dims 1..3 = row, head, batch
    const uint64_t str[3] = {static_cast<uint64_t>(s[2]) * 4, static_cast<uint64_t>(s[1]) * 4,
                             static_cast<uint64_t>(s[0]) * 4};
    const uint32_t box[4] = {static_cast<uint32_t>(Cfg::CH), rows, 1, 1};
    const CUtensorMapSwizzle sw = Cfg::RB == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : Cfg::RB == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_32B;
    return encode_tensor_map(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, str, box, sw);
  };
  int rc = enc(&tq, q, qs, Cfg::BM);
  if (!rc) rc = enc(&tk, k, ks, BN);
  if (!rc) {
    const uint64_t str[3] = {static_cast<uint64_t>(vs[2]) * 4, static_cast<uint64_t>(vs[1]) * 4,
                             static_cast<uint64_t>(vs[0]) * 4};
    const uint32_t box[4] = {32, static_cast<uint32_t>(BN), 1, 1};
    rc = encode_tensor_map(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, v, dims, str, box,
                           CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  }
  if (rc) return rc;
  // O through TMA stores when the output rows are whole 128-byte swizzle
  // rows: fp32 with Dh >= 32, or bf16 planes with Dh >= 64, 16-byte aligned
  // base and strides. Anything else (a zero-padded head, odd strides) keeps
  // the per-thread stores.
  CUtensorMap to;
  memset(&to, 0, sizeof(to));
  {
    const bool split = (flags & KF_ATTN_OUT_BF16X2) != 0;
    const int esz = split ? 2 : 4;
    const int64_t align = 16 / esz;
    const bool ok = dh_out == DH && DH >= (split ? 64 : 32) &&
                    !(reinterpret_cast<uintptr_t>(o) & 15u) && os[0] % align == 0 &&
                    os[1] % align == 0 && os[2] % align == 0;
    if (ok) {
      const uint64_t odims[4] = {static_cast<uint64_t>(DH), static_cast<uint64_t>(S),
                                 static_cast<uint64_t>(H),
                                 static_cast<uint64_t>(split ? 2 * B : B)};
      const uint64_t ostr[3] = {static_cast<uint64_t>(os[2]) * esz,
                                static_cast<uint64_t>(os[1]) * esz,
                                static_cast<uint64_t>(os[0]) * esz};
      const uint32_t obox[4] = {static_cast<uint32_t>(128 / esz), 32, 1, 1};
      if (encode_tensor_map(&to, split ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                            4, o, odims, ostr, obox, CU_TENSOR_MAP_SWIZZLE_128B) == KF_OK)
        flags |= KF_ATTN_TMA_OUT;
    }
  }

  auto kern = flash_fwd_tf32_kernel<DH, BN, KST, VST, MINB>;
  static DeviceOnce once;
  const int rc_attr = once.run("kf_flash_fwd_tf32", nullptr, [&](int) {
    return cuda_status(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES),
        "kf_flash_fwd_tf32: set smem attribute");
  });
  if (rc_attr) return rc_attr;
  const int n_qt = (S + Cfg::BM - 1) / Cfg::BM;
  dim3 grid(static_cast<unsigned>(n_qt), static_cast<unsigned>(B * H));
  return cuda_status(launch_chained(kern, grid, dim3(192), Cfg::SMEM_BYTES, st, tq, tk, tv, to, o,
                                    os[0], os[1], os[2], bits, order, H, S, dh_out, scale_log2,
                                    flags),
                     "kf_flash_fwd_tf32 launch");
}

}  // namespace kf

using namespace kf;

// Host-side checks of an attention call; launches nothing and touches no
// device state, so a caller can run them before any launch of its own.
// Returns KF_OK and the kernel flags in *kernel_flags, or an error code.
static int flash_fwd_validate(const float* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                              const float* k, int64_t k_sb, int64_t k_sh, int64_t k_sm,
                              const float* v, int64_t v_sb, int64_t v_sh, int64_t v_sm,
                              const float* o, int64_t o_sb, int64_t o_sh, int64_t o_sm,
                              int64_t B, int64_t H, int64_t S, int dh, int dh_out, int flags,
                              int* kernel_flags) {
  if (!q || !k || !v || !o || B < 0 || H < 0 || S < 0) {
    set_last_error("kf_flash_fwd_tf32: invalid arguments");
    return KF_E_INVALID;
  }
  *kernel_flags = 0;
  if (B == 0 || H == 0 || S == 0) return KF_OK;  // nothing to compute, nothing to check
  if (dh != 16 && dh != 32 && dh != 64 && dh != 128 && dh != 256) {
    set_last_error("kf_flash_fwd_tf32: stored head_dim %d not in {16,32,64,128,256}", dh);
    return KF_E_UNSUPPORTED;
  }
  if (dh_out <= 0 || dh_out > dh) {
    set_last_error("kf_flash_fwd_tf32: dh_out %d must be in [1, %d]", dh_out, dh);
    return KF_E_INVALID;
  }
  const int64_t strides[9] = {q_sb, q_sh, q_sm, k_sb, k_sh, k_sm, v_sb, v_sh, v_sm};
  for (int i = 0; i < 9; ++i) {
    if (strides[i] <= 0 || strides[i] % 4) {
      set_last_error("kf_flash_fwd_tf32: Q/K/V strides must be positive multiples of 4");
      return KF_E_UNSUPPORTED;
    }
  }
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v)) &
      15u) {
    set_last_error("kf_flash_fwd_tf32: Q/K/V must be 16-byte aligned");
    return KF_E_UNSUPPORTED;
  }
  if (B * H > 65535 || S > INT32_MAX) {
    set_last_error("kf_flash_fwd_tf32: B*H must be <= 65535 (grid y) and S < 2^31");
    return KF_E_UNSUPPORTED;
  }
  int f = flags & (KF_ATTN_CAUSAL | KF_ATTN_SKIP_EMPTY_Q | KF_ATTN_ROUND_TF32 | KF_ATTN_OUT_BF16X2);
  if ((f & KF_ATTN_OUT_BF16X2) && ((f & KF_ATTN_ROUND_TF32) || o_sm % 4 || o_sb % 4 || o_sh % 4 ||
                                   (reinterpret_cast<uintptr_t>(o) & 7u))) {
    set_last_error("kf_flash_fwd_tf32: split output needs strides %% 4 == 0, 8-byte alignment "
                   "and no TF32 rounding");
    return KF_E_INVALID;
  }
  if ((o_sm % 4 == 0) && !(reinterpret_cast<uintptr_t>(o) & 15u) && o_sb % 4 == 0 &&
      o_sh % 4 == 0)
    f |= (1 << 8);
  *kernel_flags = f;
  return KF_OK;
}

static int flash_fwd_impl(const float* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                          const float* k, int64_t k_sb, int64_t k_sh, int64_t k_sm,
                          const float* v, int64_t v_sb, int64_t v_sh, int64_t v_sm, float* o,
                          int64_t o_sb, int64_t o_sh, int64_t o_sm, const uint32_t* keep_bits,
                          const int32_t* order, int64_t B, int64_t H, int64_t S, int dh,
                          int dh_out, float sm_scale, int flags, void* stream) {
  int f = 0;
  const int rc = flash_fwd_validate(q, q_sb, q_sh, q_sm, k, k_sb, k_sh, k_sm, v, v_sb, v_sh, v_sm,
                                    o, o_sb, o_sh, o_sm, B, H, S, dh, dh_out, flags, &f);
  if (rc) return rc;
  if (B == 0 || H == 0 || S == 0) return KF_OK;
  const float scale_log2 = sm_scale * 1.4426950408889634f;
  const int64_t qs[3] = {q_sb, q_sh, q_sm}, ks[3] = {k_sb, k_sh, k_sm},
                vs[3] = {v_sb, v_sh, v_sm}, os[3] = {o_sb, o_sh, o_sm};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int Bi = static_cast<int>(B), Hi = static_cast<int>(H), Si = static_cast<int>(S);
  switch (dh) {
    case 16:
      return launch_flash<16, 64, 2, 2, 2>(q, qs, k, ks, v, vs, o, os, keep_bits, order, Bi, Hi,
                                           Si, dh, dh_out, scale_log2, f, st);
    case 32:
      return launch_flash<32, 64, 2, 2, 2>(q, qs, k, ks, v, vs, o, os, keep_bits, order, Bi, Hi,
                                           Si, dh, dh_out, scale_log2, f, st);
    case 64:
      return launch_flash<64, 64, 2, 2, 2>(q, qs, k, ks, v, vs, o, os, keep_bits, order, Bi, Hi,
                                           Si, dh, dh_out, scale_log2, f, st);
    case 128:
      return launch_flash<128, 64, 2, 2, 1>(q, qs, k, ks, v, vs, o, os, keep_bits, order, Bi, Hi,
                                            Si, dh, dh_out, scale_log2, f, st);
    default:
      return launch_flash<256, 32, 2, 1, 1>(q, qs, k, ks, v, vs, o, os, keep_bits, order, Bi, Hi,
                                            Si, dh, dh_out, scale_log2, f, st);
  }
}

extern "C" int kf_flash_fwd_tf32(const float* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                                 const float* k, int64_t k_sb, int64_t k_sh, int64_t k_sm,
                                 const float* v, int64_t v_sb, int64_t v_sh, int64_t v_sm,
                                 float* o, int64_t o_sb, int64_t o_sh, int64_t o_sm,
                                 const uint32_t* keep_bits, int64_t B, int64_t H, int64_t S,
                                 int dh, int dh_out, float sm_scale, int flags, void* stream) {
  return flash_fwd_impl(q, q_sb, q_sh, q_sm, k, k_sb, k_sh, k_sm, v, v_sb, v_sh, v_sm, o, o_sb,
                        o_sh, o_sm, keep_bits, nullptr, B, H, S, dh, dh_out, sm_scale, flags,
                        stream);
}

extern "C" int kf_flash_fwd_tf32_ordered(const float* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                                         const float* k, int64_t k_sb, int64_t k_sh, int64_t k_sm,
                                         const float* v, int64_t v_sb, int64_t v_sh, int64_t v_sm,
                                         float* o, int64_t o_sb, int64_t o_sh, int64_t o_sm,
                                         const uint32_t* keep_bits, const int32_t* batch_order,
                                         int64_t B, int64_t H, int64_t S, int dh, int dh_out,
                                         float sm_scale, int flags, void* stream) {
  if (!batch_order) {
    set_last_error("kf_flash_fwd_tf32_ordered: batch_order is null");
    return KF_E_INVALID;
  }
  return flash_fwd_impl(q, q_sb, q_sh, q_sm, k, k_sb, k_sh, k_sm, v, v_sb, v_sh, v_sm, o, o_sb,
                        o_sh, o_sm, keep_bits, batch_order, B, H, S, dh, dh_out, sm_scale, flags,
                        stream);
}
