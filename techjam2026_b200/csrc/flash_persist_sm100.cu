// Persistent tcgen05 FlashAttention forward over a device-built work list.
//
// The grid is as many CTAs as fit on the GPU at once (two per SM for
// head_dim <= 64). Each CTA takes work items -- one (batch row, head,
// 128-query tile) -- from the list that kf_attn_schedule wrote, with one
// atomic fetch per item, until the list is exhausted. The list runs the
// batch rows longest first and, within a head, the heaviest causal query
// tiles first, so concurrently running items share a head's K/V in L2 and
// the launch ends on the lightest items. Per item the arithmetic is exactly
// that of flash_fwd_tf32_kernel (same products, same softmax, same lazy
// rescale), so the output is bit-identical; what changes is that a CTA
// keeps its barriers, TMEM and pipeline state across items:
//
//   warp 0      TMA producer: fetches items, publishes them to the other
//               roles through a 4-slot ring in shared memory, loads Q of
//               the next item as soon as the softmax warps release the
//               single Q buffer, and streams K and V tiles of all its items
//               through two rings;
//   warp 1      MMA issuer: S_j into two TMEM buffers, O += P V from P in
//               TMEM; after an item's last P V it commits o_final;
//   warps 2-5   softmax (one thread per query row), then the item's O:
//               TMEM -> registers -> O / l, staged in the Q buffer (idle once
//               every S of the item has completed) and written by TMA stores;
//               then they release the buffer for the next item's Q. While a
//               CTA is between items, the other CTA on the SM keeps the
//               tensor pipe busy.
//
// The next item's first P V overwrites O in TMEM; it waits for that item's
// first softmax pass, which the softmax warps reach only after reading the
// previous O out, so no separate release of O is needed.
//
// The fetch counter and a finish counter live in the list's header: the
// CTA that finishes last zeroes both, so the list built once per forward
// serves every layer. Every wait is bounded (wait_limit()); on a timeout
// the CTA raises its abort flag, drains in-flight copies and products,
// frees TMEM and records the device status word.

#include "kf_common.cuh"

namespace kf {

constexpr int KF_PERSIST_RING = 4;  // item slots between the producer and the consumers

template <int DH, int BN, int KST, int VST, int MINB>
struct PersistCfg {
  using F = FlashCfg<DH, BN, KST, VST, MINB>;
  static constexpr int IR = KF_PERSIST_RING;
  static constexpr int RING_OFF = F::BAR_OFF + 256;
  static constexpr int SMEM_BYTES = RING_OFF + IR * 16 + 1024;
  static_assert(SMEM_BYTES <= F::SMEM_CAP, "smem");
};

// Walks the key tiles [0, end) of a batch row that hold a valid key, with the
// row's key-bit words of the NEXT tile loaded one tile ahead, so the
// global-memory latency of the mask overlaps the current tile's work. A
// tile is live exactly when kv_tile_live says so (one of its words is
// nonzero; every tile is live without key bits). `w` holds the current
// tile's words (all ones without key bits).
template <int BN>
struct LiveWalk {
  static constexpr int NW = BN / 32;
  const uint32_t* kb;
  int words, end, j;
  uint32_t w[NW], wn[NW];

  __device__ __forceinline__ void load(int t, uint32_t (&d)[NW]) const {
#pragma unroll
    for (int x = 0; x < NW; ++x) {
      const int wi = t * NW + x;
      d[x] = kb ? (wi < words ? __ldg(kb + wi) : 0u) : 0xffffffffu;
    }
  }
  __device__ __forceinline__ static bool any(const uint32_t (&d)[NW]) {
    uint32_t a = 0;
#pragma unroll
    for (int x = 0; x < NW; ++x) a |= d[x];
    return a != 0;
  }
  __device__ __forceinline__ void settle_and_prefetch() {
    while (j < end && !any(w)) {
      ++j;
      if (j < end) load(j, w);
    }
    if (j + 1 < end) load(j + 1, wn);
  }
  __device__ __forceinline__ void begin(const uint32_t* kb_, int words_, int end_) {
    kb = kb_;
    words = words_;
    end = end_;
    j = 0;
    if (end > 0) load(0, w);
    settle_and_prefetch();
  }
  __device__ __forceinline__ bool done() const { return j >= end; }
  __device__ __forceinline__ void next() {
    ++j;
    if (j < end) {
#pragma unroll
      for (int x = 0; x < NW; ++x) w[x] = wn[x];
    }
    settle_and_prefetch();
  }
};

template <int DH, int BN, int KST, int VST, int MINB>
__global__ void __launch_bounds__(192, MINB)
    flash_fwd_persist_kernel(const __grid_constant__ CUtensorMap tmQ,
                             const __grid_constant__ CUtensorMap tmK,
                             const __grid_constant__ CUtensorMap tmV,
                             const __grid_constant__ CUtensorMap tmO, float* __restrict__ O,
                             int64_t o_sb, int64_t o_sh, int64_t o_sm,
                             const uint32_t* __restrict__ keep_bits, int32_t* __restrict__ sched,
                             int nb, int H, int S, int dh_out, float scale_log2, int flags) {
  using Cfg = FlashCfg<DH, BN, KST, VST, MINB>;
  using PC = PersistCfg<DH, BN, KST, VST, MINB>;
  constexpr int BM = Cfg::BM;
  constexpr int NSB = Cfg::NSB;
  constexpr int IR = PC::IR;
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
  uint64_t* p_full = s_full + NSB;        // [NSB]
  uint64_t* o_done = p_full + NSB;        // [2]: P V products of even / odd tile index
  uint64_t* o_final = o_done + 2;
  uint64_t* item_full = o_final + 1;      // [IR]
  uint64_t* item_empty = item_full + IR;  // [IR]
  uint64_t* drain = item_empty + IR;
  uint64_t* q_free = drain + 1;           // the softmax warps are done with sQ
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(q_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int4* ring = reinterpret_cast<int4*>(smem + PC::RING_OFF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const bool causal = (flags & KF_ATTN_CAUSAL) != 0;
  const bool split = (flags & KF_ATTN_OUT_BF16X2) != 0;
  const bool zero_empty = (flags & KF_ATTN_SKIP_EMPTY_Q) != 0;
  const bool tma_out = (flags & KF_ATTN_TMA_OUT) != 0;
  const int words = (S + 31) >> 5;
  const int n_kv_all = (S + BN - 1) / BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KST; ++s) mbar_init(&k_full[s], 1);
    for (int s = 0; s < VST; ++s) mbar_init(&v_full[s], 1);
    for (int s = 0; s < NSB; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 4);
    }
    mbar_init(&o_done[0], 1);
    mbar_init(&o_done[1], 1);
    mbar_init(o_final, 1);
    for (int s = 0; s < IR; ++s) {
      mbar_init(&item_full[s], 1);
      mbar_init(&item_empty[s], 5);  // the MMA thread and the four softmax warps
    }
    mbar_init(drain, 1);
    mbar_init(q_free, 4);
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
  pdl_launch_dependents();
  pdl_wait();  // Q/K/V, the key bits and the work list come from earlier kernels

  // Item geometry, the same for every role: the keys to visit end at the
  // causal diagonal; an empty query tile (list index >= live count) is a
  // zero-writer when the caller asked for zeros there.
  auto kv_end_of = [&](int qt, bool empty) -> int {
    if (empty && zero_empty) return 0;
    int e = n_kv_all;
    if (causal) {
      const int q0 = qt * BM;
      const int last_q = (q0 + BM - 1 < S - 1) ? q0 + BM - 1 : S - 1;
      const int lim = last_q / BN + 1;
      e = lim < e ? lim : e;
    }
    return e;
  };
  auto row_bits = [&](int b) -> const uint32_t* {
    return keep_bits ? keep_bits + static_cast<int64_t>(b) * words : nullptr;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------ TMA producer
      const int n_live = sched[2];
      const int n_items = (flags & KF_ATTN_EMPTY_Q_UNTOUCHED) ? n_live : sched[3];
      const int2* items = reinterpret_cast<const int2*>(sched + KF_SCHED_HEADER);
      // Fetched items (local copies, IR deep) for the K and V cursors. Item,
      // tile and load counters are per CTA and per launch: 32 bits suffice
      // (a launch has fewer than 2^31 tiles) and keep the ring arithmetic
      // (% NSB, / NSB) cheap.
      int lb[IR], lh[IR], lend[IR];
      int kseq = 0, vseq = 0;  // items fetched; item the V cursor is on
      bool fetch_done = false, k_need_item = true, q_pending = false;
      bool v_active = false, v_done = false;
      int jk = 0, kend = 0, kb_ = 0, kh = 0, kq = 0;  // K cursor
      int jv = 0, vend = 0, vb = 0, vh = 0;           // V cursor
      const uint32_t* kbits = nullptr;
      const uint32_t* vbits = nullptr;
      int ks = 0, vs = 0;
      int k_issued = 0, v_issued = 0, q_loads = 0;
      bool ok = true;
      auto next_live = [&](const uint32_t* rb, int j, int end) {
        while (j < end && !kv_tile_live<BN>(rb, words, j, S)) ++j;
        return j;
      };
      auto k_slot_free = [&]() -> bool {
        if (k_issued < KST) return true;
        const int i = k_issued - KST;
        return mbar_test_wait(&s_full[i % NSB], static_cast<uint32_t>((i / NSB) & 1));
      };
      auto v_slot_free = [&]() -> bool {
        if (v_issued < VST) return true;
        const int i = v_issued - VST;
        return mbar_test_wait(&o_done[i & 1], static_cast<uint32_t>((i >> 1) & 1));
      };
      long long t_idle = clock64();
      while (!v_done) {
        bool progress = false;
        // (1) the K cursor needs its next item: fetch one into a free slot
        // (q_pending: the Q load still to issue uses the current item's
        // coordinates, so no new item is taken before it has gone out)
        if (k_need_item && !fetch_done && !q_pending && kseq - vseq < IR &&
            (kseq < IR || mbar_test_wait(&item_empty[kseq % IR],
                                         static_cast<uint32_t>(((kseq / IR) - 1) & 1)))) {
          const int idx = atomicAdd(&sched[0], 1);
          int bh = -1, qt = 0, empty = 0;
          if (idx < n_items) {
            const int2 it = items[idx];
            bh = it.x;
            qt = it.y;
            empty = idx >= n_live;
          }
          const int slot = static_cast<int>(kseq % IR);
          ring[slot] = make_int4(bh, qt, empty, 0);
          mbar_arrive(&item_full[slot]);  // release: the ring entry is visible with the phase
          if (bh < 0) {
            fetch_done = true;
            lb[slot] = -1;
          } else {
            const int b = bh / H, h = bh - (bh / H) * H;
            const int e = kv_end_of(qt, empty != 0);
            lb[slot] = b;
            lh[slot] = h;
            lend[slot] = e;
            const uint32_t* rb = row_bits(b);
            const int first = next_live(rb, 0, e);
            if (first < e) {
              // The Q tile goes to L2 now; its load into the Q buffer waits
              // until the previous item has left the buffer.
#pragma unroll
              for (int c = 0; c < Cfg::NCH; ++c)
                tma_prefetch_l2_4d(&tmQ, c * Cfg::CH, qt * BM, h, b);
              kb_ = b;
              kh = h;
              kq = qt;
              kend = e;
              kbits = rb;
              jk = first;
              k_need_item = false;
              q_pending = true;
            }
          }
          ++kseq;
          progress = true;
        }
        // (2) Q of the K cursor's item, once the softmax warps are done with
        // the Q buffer (every S of the previous item has completed and its
        // output has been staged out of the buffer)
        if (q_pending) {
          const bool free =
              q_loads == 0 || mbar_test_wait(q_free, static_cast<uint32_t>((q_loads - 1) & 1));
          if (free) {
            mbar_arrive_expect_tx(q_full, Cfg::Q_BYTES);
#pragma unroll
            for (int c = 0; c < Cfg::NCH; ++c)
              tma_load_4d(sQ + c * BM * Cfg::RB, &tmQ, q_full, c * Cfg::CH, kq * BM, kh, kb_);
            ++q_loads;
            q_pending = false;
            progress = true;
          }
        }
        // (3) the next K tile of that item: K slots free as the previous
        // item's products complete, independently of the Q buffer
        if (!k_need_item && k_slot_free()) {
          mbar_arrive_expect_tx(&k_full[ks], Cfg::KV_BYTES);
#pragma unroll
          for (int c = 0; c < Cfg::NCH; ++c)
            tma_load_4d(sK + ks * Cfg::KV_BYTES + c * BN * Cfg::RB, &tmK, &k_full[ks], c * Cfg::CH,
                        jk * BN, kh, kb_);
          ++k_issued;
          if (++ks == KST) ks = 0;
          jk = next_live(kbits, jk + 1, kend);
          if (jk >= kend) k_need_item = true;
          progress = true;
        }
        // (4) V follows the same tile sequence, never ahead of K
        if (!v_active && vseq < kseq) {
          const int slot = static_cast<int>(vseq % IR);
          if (lb[slot] < 0) {
            v_done = true;  // the end of the list: every K and V tile is out
          } else {
            const uint32_t* rb = row_bits(lb[slot]);
            const int first = next_live(rb, 0, lend[slot]);
            if (first < lend[slot]) {
              v_active = true;
              vb = lb[slot];
              vh = lh[slot];
              vend = lend[slot];
              vbits = rb;
              jv = first;
            } else {
              ++vseq;  // an item without key tiles
            }
          }
          progress = true;
        }
        if (v_active && v_issued < k_issued && v_slot_free()) {
          mbar_arrive_expect_tx(&v_full[vs], Cfg::V_BYTES);
#pragma unroll
          for (int c = 0; c < Cfg::VCH; ++c)
            tma_load_4d(sV + vs * Cfg::V_BYTES + c * BN * 128, &tmV, &v_full[vs], c * 32, jv * BN,
                        vh, vb);
          ++v_issued;
          if (++vs == VST) vs = 0;
          jv = next_live(vbits, jv + 1, vend);
          if (jv >= vend) {
            v_active = false;
            ++vseq;
          }
          progress = true;
        }
        if (progress) {
          t_idle = clock64();
          continue;
        }
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
        // Unwinding: let every copy already issued land before the CTA
        // leaves. Only the last Q load can be in flight (a Q load waits for
        // every product of the previous Q), and at most KST / VST K / V.
        if (q_loads > 0)
          mbar_wait_drain(q_full, static_cast<uint32_t>((q_loads - 1) & 1),
                          KF_DEV_WAIT_TIMEOUT_TMA);
        for (int i = (k_issued > KST ? k_issued - KST : 0); i < k_issued; ++i)
          mbar_wait_drain(&k_full[i % KST], static_cast<uint32_t>((i / KST) & 1),
                          KF_DEV_WAIT_TIMEOUT_TMA);
        for (int i = (v_issued > VST ? v_issued - VST : 0); i < v_issued; ++i)
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
      int it = 0, q_used = 0, seq = 0;
      bool ok = true;
      int item_first = 0;
      auto issue_pv = [&](int i) -> bool {
        const int sb = static_cast<int>(i % NSB);
        if (!mbar_wait(&p_full[sb], static_cast<uint32_t>((i / NSB) & 1), abort_flag,
                       KF_DEV_WAIT_TIMEOUT_MMA))
          return false;
        if (!mbar_wait(&v_full[vs], vph, abort_flag, KF_DEV_WAIT_TIMEOUT_MMA)) return false;
        tc_fence_after();
        const uint32_t vbase = sVa + vs * Cfg::V_BYTES;
#pragma unroll
        for (int kk = 0; kk < BN / 8; ++kk) {
          const uint64_t bd =
              make_smem_desc(vbase + kk * 8 * 128, BN * 128, 4 * 128, KF_SWIZZLE_128B_BASE32B);
          mma_tf32_ts(tmem_base + Cfg::O_COL, tmem_base + sb * BN + kk * 8, bd, idesc_o,
                      (i > item_first || kk > 0) ? 1u : 0u);
        }
        mma_commit(&o_done[i & 1]);
        if (++vs == VST) {
          vs = 0;
          vph ^= 1u;
        }
        return true;
      };
      while (ok) {
        const int slot = static_cast<int>(seq % IR);
        if (!mbar_wait(&item_full[slot], static_cast<uint32_t>((seq / IR) & 1), abort_flag,
                       KF_DEV_WAIT_TIMEOUT_MMA))
          break;
        const int4 itm = ring[slot];
        mbar_arrive(&item_empty[slot]);
        ++seq;
        if (itm.x < 0) break;
        const int b = itm.x / H;
        const int kend = kv_end_of(itm.y, itm.z != 0);
        const uint32_t* kb = row_bits(b);
        item_first = it;
        bool have_q = false;
        LiveWalk<BN> walk;
        for (walk.begin(kb, words, kend); !walk.done() && ok; walk.next()) {
          if (!have_q) {
            if (!mbar_wait(q_full, static_cast<uint32_t>(q_used & 1), abort_flag,
                           KF_DEV_WAIT_TIMEOUT_MMA)) {
              ok = false;
              break;
            }
            ++q_used;
            have_q = true;
          }
          if (!mbar_wait(&k_full[ks], kph, abort_flag, KF_DEV_WAIT_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int sb = static_cast<int>(it % NSB);
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
          if (it - item_first >= NSB && !issue_pv(it - NSB)) {
            ok = false;
            break;
          }
        }
        // The item's remaining P V products, then its O is final.
        for (int i = (it - NSB + 1 > item_first ? it - NSB + 1 : item_first); ok && i < it; ++i)
          ok = issue_pv(i);
        if (ok && it > item_first) mma_commit(o_final);
      }
      mma_commit(drain);
      mbar_wait_drain(drain, 0, KF_DEV_WAIT_TIMEOUT_MMA);
    }
  } else {
    // -------------------------------------------------- softmax (warps 2..5)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_row = tmem_base + lane_off;
    const bool rnd = (flags & KF_ATTN_ROUND_TF32) != 0;
    int it = 0, seq = 0, n_final = 0;
    bool ok = true;
    while (ok) {
      const int slot = static_cast<int>(seq % IR);
      if (!mbar_wait(&item_full[slot], static_cast<uint32_t>((seq / IR) & 1), abort_flag,
                     KF_DEV_WAIT_TIMEOUT_SOFTMAX))
        break;
      const int4 itm = ring[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&item_empty[slot]);
      ++seq;
      if (itm.x < 0) break;
      const int b = itm.x / H, h = itm.x - (itm.x / H) * H;
      const int q0 = itm.y * BM;
      const int qi = q0 + r;
      const int kend = kv_end_of(itm.y, itm.z != 0);
      const uint32_t* kb = row_bits(b);
      const int item_first = it;
      float m_run = -INFINITY;
      float l_run = 0.f;
      LiveWalk<BN> walk;
      for (walk.begin(kb, words, kend); !walk.done(); walk.next()) {
        const int j = walk.j;
        const int sb = static_cast<int>(it % NSB);
        if (!mbar_wait(&s_full[sb], static_cast<uint32_t>((it / NSB) & 1), abort_flag,
                       KF_DEV_WAIT_TIMEOUT_SOFTMAX)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[BN];
        if constexpr (BN == 64) {
          tmem_ld64(t_row + sb * BN, s);
        } else {
#pragma unroll
          for (int c = 0; c < BN / 32; ++c)
            tmem_ld32(t_row + sb * BN + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
        }
        const int k0 = j * BN;
        // this tile's mask words, loaded while the previous tile was processed
        const uint32_t* kw = walk.w;
        bool all_keys = (k0 + BN <= S);
#pragma unroll
        for (int w = 0; w < BN / 32; ++w) all_keys = all_keys && (kw[w] == 0xffffffffu);
        const bool diag = causal && (k0 + BN - 1 > q0);
        if (!(all_keys && !diag))
          mask_scores<BN>(s, kw, (causal && qi + 1 < S ? qi + 1 : S) - k0);
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
        float alpha = 1.f;
        bool rescale_o = false;
        if (mx > m_run + 8.f) {
          if (m_run != -INFINITY) {
            alpha = fast_exp2(m_run - mx);
            l_run *= alpha;
            rescale_o = (it > item_first);
          }
          m_run = mx;
        }
        const float neg_m = (m_run == -INFINITY) ? 0.f : -m_run;
        const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
        const uint64_t nm2 = f2_pack(neg_m, neg_m);
        uint64_t sp2[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) sp2[u] = f2_pack(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < BN; c += 2) {
          float t0, t1;
          f2_unpack(f2_fma(f2_pack(s[c], s[c + 1]), sc2, nm2), t0, t1);
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
          // P V of the item's previous tile must have landed before O is
          // rescaled; o_done[(it-1) & 1] is at most one phase behind it
          // (the s_full arrival just observed implies P V of tile it - NSB,
          // hence of tile it - 3).
          if (!mbar_wait(&o_done[(it - 1) & 1], static_cast<uint32_t>(((it - 1) >> 1) & 1),
                         abort_flag, KF_DEV_WAIT_TIMEOUT_SOFTMAX)) {
            ok = false;
            break;
          }
          tc_fence_after();
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
      if (!ok) break;
      // The item's output row: O / l from TMEM, or zeros for a row of a
      // query tile without key tiles.
      float* orow = O + static_cast<int64_t>(b) * o_sb + static_cast<int64_t>(h) * o_sh +
                    static_cast<int64_t>(qi) * o_sm;
      uint16_t* ohi = reinterpret_cast<uint16_t*>(O) + static_cast<int64_t>(b) * o_sb +
                      static_cast<int64_t>(h) * o_sh + static_cast<int64_t>(qi) * o_sm;
      uint16_t* olo = ohi + static_cast<int64_t>(nb) * o_sb;
      if (it > item_first) {
        // o_final completes once per item with key tiles, in item order.
        if (!mbar_wait(o_final, static_cast<uint32_t>(n_final & 1), abort_flag,
                       KF_DEV_WAIT_TIMEOUT_SOFTMAX)) {
          ok = false;
          break;
        }
        ++n_final;
        tc_fence_after();
        const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
        if (tma_out) {
          // Every S of the item has completed (o_final), so the Q buffer is
          // idle: each warp stages its 32 rows there in the 128-byte-swizzled
          // layout of the output map, chunk by chunk, and one lane stores
          // them with TMA (fp32 chunks of 32 columns, or bf16 hi/lo planes of
          // 64 columns, the lo plane as batch index b + B of the same map).
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
            bulk_wait_group_read<0>();  // staging read; the writes finish on their own
          }
          __syncwarp();
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
        // The next item's first P V overwrites O: it waits for that item's
        // first P, which this warp arrives only after these loads completed
        // (tmem_ld waits for them), behind a tcgen05 fence.
        tc_fence_before();
        // The Q buffer may take the next item's Q (its staging has been read).
        if (lane == 0) mbar_arrive(q_free);
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
  if (threadIdx.x == 0) {
    // The last CTA to finish resets the list's counters for the next launch
    // (every CTA has fetched past the end of the list before it gets here).
    __threadfence();
    if (atomicAdd(&sched[1], 1) == static_cast<int>(gridDim.x) - 1) {
      sched[0] = 0;
      sched[1] = 0;
      __threadfence();
    }
  }
}

template <int DH, int BN, int KST, int VST, int MINB>
static int launch_flash_persist(const float* q, const int64_t* qs, const float* k,
                                const int64_t* ks, const float* v, const int64_t* vs, float* o,
                                const int64_t* os, const uint32_t* bits, int32_t* sched, int B,
                                int H, int S, int dh_stored, int dh_out, float scale_log2,
                                int flags, cudaStream_t st) {
  using Cfg = FlashCfg<DH, BN, KST, VST, MINB>;
  using PC = PersistCfg<DH, BN, KST, VST, MINB>;
  CUtensorMap tq, tk, tv;
  const uint64_t dims[4] = {static_cast<uint64_t>(dh_stored), static_cast<uint64_t>(S),
                            static_cast<uint64_t>(H), static_cast<uint64_t>(B)};
  auto enc = [&](CUtensorMap* m, const float* base, const int64_t* s, uint32_t rows) {
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
  // O through TMA stores (staged in the idle Q buffer) when the output rows
  // are whole 128-byte swizzle rows: the same rule as kf_flash_fwd_tf32.
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
  auto kern = flash_fwd_persist_kernel<DH, BN, KST, VST, MINB>;
  static DeviceOnce once;
  static int resident[KF_MAX_DEVICES] = {0};
  int dev = 0;
  rc = once.run("kf_flash_fwd_tf32_sched", &dev, [&](int d) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, PC::SMEM_BYTES);
    // All of the SM's unified memory as shared memory: MINB CTAs of this
    // size need it (the default carve-out may leave room for fewer).
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                               cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess) return cuda_status(e, "kf_flash_fwd_tf32_sched: set attributes");
    // MINB CTAs per SM by construction: shared memory and TMEM are sized
    // for it (static_asserts of FlashCfg / PersistCfg) and __launch_bounds__
    // caps the registers. CTAs never wait for one another, so a grid that
    // could not be resident at once would only run in more than one wave.
    resident[d] = MINB * sm_count();
    return static_cast<int>(KF_OK);
  });
  if (rc) return rc;
  const int64_t upper = static_cast<int64_t>(B) * H * ((S + Cfg::BM - 1) / Cfg::BM);
  const int grid = static_cast<int>(upper < resident[dev] ? upper : resident[dev]);
  return cuda_status(launch_chained(kern, dim3(static_cast<unsigned>(grid)), dim3(192),
                                    PC::SMEM_BYTES, st, tq, tk, tv, to, o, os[0], os[1], os[2], bits,
                                    sched, B, H, S, dh_out, scale_log2, flags),
                     "kf_flash_fwd_tf32_sched launch");
}

}  // namespace kf

using namespace kf;

extern "C" int kf_flash_fwd_tf32_sched(const float* q, int64_t q_sb, int64_t q_sh, int64_t q_sm,
                                       const float* k, int64_t k_sb, int64_t k_sh, int64_t k_sm,
                                       const float* v, int64_t v_sb, int64_t v_sh, int64_t v_sm,
                                       float* o, int64_t o_sb, int64_t o_sh, int64_t o_sm,
                                       const uint32_t* keep_bits, int32_t* sched, int64_t B,
                                       int64_t H, int64_t S, int dh, int dh_out, float sm_scale,
                                       int flags, void* stream) {
  if (!sched || (reinterpret_cast<uintptr_t>(sched) & 7u)) {
    set_last_error("kf_flash_fwd_tf32_sched: sched is null or not 8-byte aligned");
    return KF_E_INVALID;
  }
  int f = 0;
  const int rc = flash_fwd_validate(q, q_sb, q_sh, q_sm, k, k_sb, k_sh, k_sm, v, v_sb, v_sh, v_sm,
                                    o, o_sb, o_sh, o_sm, B, H, S, dh, dh_out, flags, &f);
  if (rc) return rc;
  if (B == 0 || H == 0 || S == 0) return KF_OK;
  f |= flags & KF_ATTN_EMPTY_Q_UNTOUCHED;
  const float scale_log2 = sm_scale * 1.4426950408889634f;
  const int64_t qs[3] = {q_sb, q_sh, q_sm}, ks[3] = {k_sb, k_sh, k_sm},
                vs[3] = {v_sb, v_sh, v_sm}, os[3] = {o_sb, o_sh, o_sm};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int Bi = static_cast<int>(B), Hi = static_cast<int>(H), Si = static_cast<int>(S);
  switch (dh) {
    case 16:
      return launch_flash_persist<16, 64, 2, 2, 2>(q, qs, k, ks, v, vs, o, os, keep_bits, sched,
                                                   Bi, Hi, Si, dh, dh_out, scale_log2, f, st);
    case 32:
      return launch_flash_persist<32, 64, 2, 2, 2>(q, qs, k, ks, v, vs, o, os, keep_bits, sched,
                                                   Bi, Hi, Si, dh, dh_out, scale_log2, f, st);
    case 64:
      return launch_flash_persist<64, 64, 2, 2, 2>(q, qs, k, ks, v, vs, o, os, keep_bits, sched,
                                                   Bi, Hi, Si, dh, dh_out, scale_log2, f, st);
    case 128:
      return launch_flash_persist<128, 64, 2, 2, 1>(q, qs, k, ks, v, vs, o, os, keep_bits, sched,
                                                    Bi, Hi, Si, dh, dh_out, scale_log2, f, st);
    default:
      return launch_flash_persist<256, 32, 2, 1, 1>(q, qs, k, ks, v, vs, o, os, keep_bits, sched,
                                                    Bi, Hi, Si, dh, dh_out, scale_log2, f, st);
  }
}
