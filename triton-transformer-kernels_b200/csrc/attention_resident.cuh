// attention_resident.cuh - row-resident softmax schedule of the 16-bit
// tcgen05 attention for short sequences (seq_len <= 512, head_dim 64).
//
// A work item is one 128-row query tile of one (batch, head). All of its
// score tiles (up to four 128-key tiles = the 512 TMEM columns) stay in TMEM,
// so the softmax runs over whole rows, like the explicit reference
// (transformer_opt/dispatch.py:69-96: scores rounded to the input dtype T,
// fp32 softmax over the row, probabilities rounded to T, then P@V):
//   pass A  row maximum of the raw Q K^T values. Rounding to T and scaling by
//           scale > 0 are monotone, so T(T(max) * scale) is the maximum of the
//           scores s = T(T(qk) * scale).
//   pass B  e = exp(s - max) for every key, written back over the raw scores
//           (fp32), and the row sum of the e.
//   pass C  P = T(e / sum), packed into the first half of each key tile's
//           columns; the P@V of that tile is issued at once.
// Every exponential is evaluated once and Q K^T is computed once (the
// streaming two-pass schedule evaluates both twice), and the row sum is the
// plain sum of the e values. The rounding boundaries (s in T, e in fp32, P in
// T, fp32 accumulation of P@V) are the two-pass schedule's.
//
// Warps: 0-15 softmax, 16 producer (TMA), 17 MMA. Softmax warp w reads TMEM
// lane quadrant w % 4 (rows 32 (w % 4) + 16 blk .. + 15, blk = (w / 4) % 2)
// with the 16x256b shape, columns [64 half, 64 half + 64) of every key tile
// (half = w / 8): lane i holds rows i / 4 and i / 4 + 8 of its 16-row block
// and columns 8g + 2(i % 4), + 1 of every 8-column group g, so a row's four
// threads in one warp combine with shuffles and the two warps of a row (w and
// w + 8) exchange their row maximum and sum through shared memory behind a
// bounded mbarrier. Sixteen warps (four per SM sub-partition) keep the
// MUFU / ALU / TMEM latencies covered; eight left the issue slots idle.
//
// TMEM columns: key tile j at [128 j, 128 j + 128). Pass C packs each half's
// probabilities into the first 32 columns of its own 64 (column c holds keys
// 2c, 2c + 1 of the half): P_j at [128 j, + 32) and [128 j + 96, + 32), so no
// warp overwrites columns the other half still has to read, and the P@V MMA
// takes its K steps from those two places. O lives at [416, 480), the middle
// 64 columns of key tile 3; pass C finishes the tiles in descending order, so
// those columns are free before the first P@V writes O.
//
// Ordering across items. One thread issues every MMA and tcgen05.mma
// executes in issue order, so the next item's score MMA into tile j follows
// this item's P@V of tile j, which read P_j. The next item's score MMA into
// tile 3 and its first P@V (whichever writes O's columns first) wait until
// the epilogue has read O (o_empty). Only the parity of each key tile's
// mbarrier phase count is needed: bit j of `tile_par` (items whose key range
// reached tile j, mod 2), kept identically in every role.
//
// Every wait is bounded (mbar_wait): on timeout the CTA raises its abort
// flag and a device status bit, drains its copies and MMAs with bounded
// waits, frees TMEM and returns.
#pragma once

#include "attention_tc.cuh"

namespace b200tk {
namespace tc {

struct RrLayout {
  static constexpr int D = 64;
  static constexpr int BN = 128;
  static constexpr int kTiles = 4;  // key tiles of a row: seq_len <= 512
  static constexpr int kQStages = 2;
  static constexpr int KST = 4, VST = 4;
  static constexpr int kQBytes = BM * D * 2;
  static constexpr int kKVBytes = BN * D * 2;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQStages * kQBytes;
  static constexpr int kV = kK + KST * kKVBytes;
  static constexpr int kBar = kV + VST * kKVBytes;
  static constexpr int kPairs = 8;  // softmax warp pairs (w, w + 8) sharing rows
  static constexpr int kNumBars = 2 * kQStages + 2 * KST + 2 * VST + 2 * kTiles + 3 + kPairs;
  // row statistics exchanged between the two warps of a row: [max | sum][half][row]
  static constexpr int kStats = kBar + kNumBars * 8;
  static constexpr int kMisc = kStats + 2 * 2 * BM * 4;
  static constexpr int kBytes = kMisc + 64 + 1024;  // + alignment slack
  static constexpr int kSoftmaxWarps = 16;
  static constexpr int kProducerWarp = 16;
  static constexpr int kMmaWarp = 17;
  static constexpr int kThreads = 32 * 18;
  static constexpr int kSoftmaxThreads = 32 * kSoftmaxWarps;
  static constexpr int kPCol1 = 96;  // P of a tile's second key half
  static constexpr int kOCol = (kTiles - 1) * BN + 32;
  static constexpr int kMaxSeq = kTiles * BN;
  static_assert(kBytes <= 232448, "shared memory budget");
  static_assert(kOCol + D == (kTiles - 1) * BN + kPCol1, "O between tile 3's two P halves");
};

template <typename T, bool CAUSAL, bool HAS_MASK>
__global__ void __launch_bounds__(RrLayout::kThreads, 1)
    attention_resident_kernel(const __grid_constant__ AttnTcParams p) {
  using L = RrLayout;
  constexpr int D = L::D;
  constexpr int BN = L::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);

  const uint32_t bar0 = sbase + L::kBar;
  auto bar_q_full = [&](int s) { return bar0 + 8 * s; };
  auto bar_q_empty = [&](int s) { return bar0 + 8 * (L::kQStages + s); };
  const uint32_t kb = bar0 + 8 * 2 * L::kQStages;
  auto bar_k_full = [&](int s) { return kb + 8 * s; };
  auto bar_k_empty = [&](int s) { return kb + 8 * (L::KST + s); };
  const uint32_t vb = kb + 8 * 2 * L::KST;
  auto bar_v_full = [&](int s) { return vb + 8 * s; };
  auto bar_v_empty = [&](int s) { return vb + 8 * (L::VST + s); };
  const uint32_t sb = vb + 8 * 2 * L::VST;
  auto bar_s_full = [&](int j) { return sb + 8 * j; };
  auto bar_p_full = [&](int j) { return sb + 8 * (L::kTiles + j); };
  const uint32_t bar_pv_done = sb + 8 * 2 * L::kTiles;
  const uint32_t bar_o_empty = bar_pv_done + 8;
  const uint32_t bar_drain = bar_o_empty + 8;
  auto bar_pair = [&](int pr) { return bar_drain + 8 + 8 * pr; };
  float* stats = reinterpret_cast<float*>(smem + L::kStats);  // [2][2][BM]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 8);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  if (tid == 0) {
    for (int s = 0; s < L::kQStages; ++s) {
      mbar_init(bar_q_full(s), 1);
      mbar_init(bar_q_empty(s), 1);
    }
    for (int s = 0; s < L::KST; ++s) {
      mbar_init(bar_k_full(s), 1);
      mbar_init(bar_k_empty(s), 1);
    }
    for (int s = 0; s < L::VST; ++s) {
      mbar_init(bar_v_full(s), 1);
      mbar_init(bar_v_empty(s), 1);
    }
    for (int j = 0; j < L::kTiles; ++j) {
      mbar_init(bar_s_full(j), 1);
      mbar_init(bar_p_full(j), L::kSoftmaxThreads);
    }
    mbar_init(bar_pv_done, 1);
    mbar_init(bar_o_empty, L::kSoftmaxThreads);
    mbar_init(bar_drain, 1);
    for (int pr = 0; pr < L::kPairs; ++pr) mbar_init(bar_pair(pr), 64);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == L::kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  __shared__ int s_kv_end[HAS_MASK ? kMaxMaskBatches : 1];
  const bool kv_bounds = HAS_MASK && p.batch <= kMaxMaskBatches;
  if (kv_bounds) mask_key_bounds(p, s_kv_end);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Persistent schedule: CTA c takes items c, c + grid, ... Items of one
  // (batch, head) are adjacent, so the CTAs in flight share its K / V in L2;
  // causal items are taken longest first.
  const int n_qt = p.n_qtiles;
  const int total_items = n_qt * p.batch * p.heads;
  struct Item {
    int b, h, q0, n_kv;
  };
  auto item_at = [&](int it) {
    Item w;
    const int bh = it / n_qt;
    int qt = it - bh * n_qt;
    if (CAUSAL) qt = n_qt - 1 - qt;
    w.b = bh / p.heads;
    w.h = bh - w.b * p.heads;
    w.q0 = qt * BM;
    int kv_end = CAUSAL ? min(p.seq, w.q0 + BM) : p.seq;
    if (HAS_MASK && kv_bounds) kv_end = max(1, min(kv_end, s_kv_end[w.b]));
    w.n_kv = (kv_end + BN - 1) / BN;
    return w;
  };
  auto wait = [&](uint32_t bar, uint32_t parity) {
    return mbar_wait(bar, parity, abort_flag, p.status, B200TK_STATUS_PIPELINE_TIMEOUT,
                     kWaitLimitNs);
  };

  if (warp == L::kProducerWarp) {
    // ------------------------------------------------------------ producer
    // Q into a two-stage buffer; the item's K tiles in key order and its V
    // tiles in the order the P@V MMAs consume them (descending), each into a
    // four-slot ring. Both rings are polled, so neither holds the other back.
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_q);
      tma_prefetch_desc(&p.tm_k);
      tma_prefetch_desc(&p.tm_v);
      int issued_q[L::kQStages] = {};
      int issued_k[L::KST] = {};
      int issued_v[L::VST] = {};
      bool ok = true;
      int kc = 0, vc = 0;
      for (int it = blockIdx.x, k = 0; it < total_items && ok; it += gridDim.x, ++k) {
        const Item w = item_at(it);
        const int qs = k & 1;
        if (k >= L::kQStages && !wait(bar_q_empty(qs), ((k >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(bar_q_full(qs), L::kQBytes);
        tma_load_4d(sbase + L::kQ + qs * L::kQBytes, &p.tm_q, bar_q_full(qs), 0, w.h, w.q0, w.b);
        ++issued_q[qs];
        int gk = 0, iv = 0;
        uint64_t t_last = globaltimer_ns();
        while ((gk < w.n_kv || iv < w.n_kv) && ok) {
          bool progress = false;
          if (gk < w.n_kv) {
            const int kg = kc + gk;
            const int s = kg % L::KST;
            if (kg < L::KST || mbar_try_wait(bar_k_empty(s), ((kg / L::KST) - 1) & 1)) {
              mbar_arrive_expect_tx(bar_k_full(s), L::kKVBytes);
              tma_load_4d(sbase + L::kK + s * L::kKVBytes, &p.tm_k, bar_k_full(s), 0, w.h, gk * BN,
                          w.b);
              ++issued_k[s];
              ++gk;
              progress = true;
            }
          }
          if (iv < w.n_kv) {
            const int vg = vc + iv;
            const int s = vg % L::VST;
            if (vg < L::VST || mbar_try_wait(bar_v_empty(s), ((vg / L::VST) - 1) & 1)) {
              mbar_arrive_expect_tx(bar_v_full(s), L::kKVBytes);
              tma_load_4d(sbase + L::kV + s * L::kKVBytes, &p.tm_v, bar_v_full(s), 0, w.h,
                          (w.n_kv - 1 - iv) * BN, w.b);
              ++issued_v[s];
              ++iv;
              progress = true;
            }
          }
          if (progress) {
            t_last = globaltimer_ns();
          } else if (*abort_flag) {
            ok = false;
          } else if (globaltimer_ns() - t_last > kWaitLimitNs) {
            *abort_flag = 1;
            atomicOr(p.status, B200TK_STATUS_PIPELINE_TIMEOUT);
            ok = false;
          }
        }
        kc += w.n_kv;
        vc += w.n_kv;
      }
      if (*abort_flag) {
        // drain: every copy this thread started lands before the CTA exits
        auto drain = [&](uint32_t bar, int issued) {
          if (issued == 0) return;
          const uint32_t par = (issued - 1) & 1;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(bar, par) && globaltimer_ns() - t0 < kWaitLimitNs) {
          }
        };
        for (int s = 0; s < L::kQStages; ++s) drain(bar_q_full(s), issued_q[s]);
        for (int s = 0; s < L::KST; ++s) drain(bar_k_full(s), issued_k[s]);
        for (int s = 0; s < L::VST; ++s) drain(bar_v_full(s), issued_v[s]);
      }
    }
  } else if (warp == L::kMmaWarp) {
    // ----------------------------------------------------------- MMA issuer
    // Warp-uniform loop; one elected lane issues every tcgen05.mma and
    // tcgen05.commit.
    const bool leader = elect_one_sync();
    constexpr uint32_t kFmt = ElemTraits<T>::kFmt;
    constexpr uint32_t idesc_qk = make_idesc(kFmt, 0, 0, BN, BM);  // Q K-major, K K-major
    constexpr uint32_t idesc_qk2 = make_idesc(kFmt, 0, 0, 2 * BN, BM);  // two key tiles
    constexpr uint32_t idesc_pv = make_idesc(kFmt, 0, 1, D, BM);   // P (tmem), V MN-major
    const uint64_t q_desc0 = make_sdesc(sbase + L::kQ, 16, 1024, kLayoutSw128);
    const uint64_t k_desc0 = make_sdesc(sbase + L::kK, 16, 1024, kLayoutSw128);
    const uint64_t v_desc0 = make_sdesc(sbase + L::kV, BN * 128, 1024, kLayoutSw128);
    auto wait_all = [&](uint32_t bar, uint32_t parity) {
      return __all_sync(0xFFFFFFFFu, wait(bar, parity));
    };
    bool ok = true;
    int kc = 0, vc = 0;
    uint32_t tile_par = 0;
    for (int it = blockIdx.x, k = 0; it < total_items && ok; it += gridDim.x, ++k) {
      const Item w = item_at(it);
      const int qs = k & 1;
      ok = wait_all(bar_q_full(qs), (k >> 1) & 1);
      if (!ok) break;
      bool o_free = k == 0;
      // S_j = Q K_j^T into key tile j's columns. Two key tiles in adjacent
      // ring slots (slot of tile j even) take one N = 256 MMA per K step:
      // their K rows are contiguous in shared memory and their score columns
      // in TMEM.
      for (int j = 0; j < w.n_kv && ok;) {
        const int kg = kc + j;
        const int s = kg % L::KST;
        const bool wide = (s % 2 == 0) && j + 1 < w.n_kv;
        const int last = wide ? j + 1 : j;
        for (int jj = j; jj <= last && ok; ++jj) {
          const int g = kc + jj;
          ok = wait_all(bar_k_full(g % L::KST), (g / L::KST) & 1);
        }
        if (ok && last == L::kTiles - 1 && !o_free) {
          ok = wait_all(bar_o_empty, (k - 1) & 1);
          o_free = true;
        }
        if (!ok) break;
        tc_fence_after();
        if (leader) {
          const uint64_t qd = q_desc0 + static_cast<uint32_t>((qs * L::kQBytes) >> 4);
          const uint64_t kd = k_desc0 + static_cast<uint32_t>((s * L::kKVBytes) >> 4);
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks)  // 32 bytes of K per step, one swizzle atom
            mma_ss_f16(tmem + j * BN, qd + static_cast<uint32_t>(ks * 2),
                       kd + static_cast<uint32_t>(ks * 2), wide ? idesc_qk2 : idesc_qk,
                       ks > 0 ? 1u : 0u);
          for (int jj = j; jj <= last; ++jj) tc_commit(bar_k_empty((kc + jj) % L::KST));
          if (last == w.n_kv - 1) tc_commit(bar_q_empty(qs));
          for (int jj = j; jj <= last; ++jj) tc_commit(bar_s_full(jj));
        }
        __syncwarp();
        j = last + 1;
      }
      // O += P_j V_j, tiles in descending order as pass C releases them. The
      // V tiles and O's columns are waited for first (while the softmax is
      // still in passes A / B), so each P@V step only waits for its P.
      for (int i = 0; i < w.n_kv && ok; ++i) {
        const int vg = vc + i;
        ok = wait_all(bar_v_full(vg % L::VST), (vg / L::VST) & 1);
      }
      if (ok && !o_free) {
        ok = wait_all(bar_o_empty, (k - 1) & 1);
        o_free = true;
      }
      for (int i = 0; i < w.n_kv && ok; ++i) {
        const int j = w.n_kv - 1 - i;
        const int s = (vc + i) % L::VST;
        ok = wait_all(bar_p_full(j), (tile_par >> j) & 1u);
        if (!ok) break;
        tc_fence_after();
        if (leader) {
          const uint64_t vd = v_desc0 + static_cast<uint32_t>((s * L::kKVBytes) >> 4);
#pragma unroll
          for (int ks = 0; ks < BN / 16; ++ks) {  // 16 keys (8 packed columns, 16 V rows) per step
            const uint32_t a_tmem = tmem + j * BN + (ks < 4 ? ks * 8 : L::kPCol1 + (ks - 4) * 8);
            mma_ts_f16(tmem + L::kOCol, a_tmem, vd + static_cast<uint32_t>((ks * 16 * 128) >> 4),
                       idesc_pv, (i > 0 || ks > 0) ? 1u : 0u);
          }
          tc_commit(bar_v_empty(s));
          if (i == w.n_kv - 1) tc_commit(bar_pv_done);
        }
        __syncwarp();
      }
      tile_par ^= (1u << w.n_kv) - 1u;
      kc += w.n_kv;
      vc += w.n_kv;
    }
    // no MMA may still be writing TMEM when the CTA tears down
    if (leader) {
      tc_commit(bar_drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(bar_drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else {
    // -------------------------------------------------------------- softmax
    constexpr int NE = 32;  // values per thread and key tile: 2 rows x 16 keys
    const int sw = warp;
    const int quad = sw & 3;              // the TMEM lane quadrant this warp may access
    const int blk = (sw >> 2) & 1;
    const int half = sw >> 3;             // key columns [64 half, 64 half + 64) of each tile
    const int pair = sw & 7;              // softmax warps sw and sw + 8 hold the same rows
    const int rb = quad * 32 + blk * 16;  // first row of this warp's block
    const int ra = rb + (lane >> 2);      // this thread's rows: ra and ra + 8
    const int cq = 2 * (lane & 3);
    const uint32_t lane_off = static_cast<uint32_t>(rb) << 16;
    const int c0 = 64 * half;
    auto e_row = [&](int e) { return ra + 8 * ((e >> 1) & 1); };
    auto e_col = [&](int e) { return c0 + 8 * (e >> 2) + cq + (e & 1); };  // column in the tile
    const float scale = p.scale;
    const bool pow2 = std::is_same_v<T, __nv_bfloat16> && p.scale_pow2 != 0;
    // T(qk) * scale * log2e in one rounding when scale is a power of two
    // (T(qk) * scale is then exact)
    const float scale_log2e = scale * kLog2e;
    float* st_max = stats;           // [half][row]
    float* st_sum = stats + 2 * BM;  // [half][row]
    bool ok = true;
    uint32_t tile_par = 0;

    auto issue_tile = [&](int j, uint32_t (&r)[NE]) {
      tmem_ld16x256b<8>(tmem + lane_off + j * BN + c0, r);
    };
    // Completes issue_tile(j) for raw Q K^T: keys outside the sequence,
    // padding keys and (causal) keys after the row become -inf.
    auto finish_scores = [&](const Item& w, int j, uint32_t (&raw)[NE]) {
      const int n0 = j * BN + c0;
      uint32_t kbits[2];
      if constexpr (HAS_MASK) {
#pragma unroll
        for (int wd = 0; wd < 2; ++wd) {
          const int n = n0 + wd * 32 + lane;
          bool valid = false;
          if (n < p.seq) valid = p.mask[w.b * p.mask_sb + n * p.mask_ss] != 0;
          kbits[wd] = __ballot_sync(0xFFFFFFFFu, valid);
        }
      }
      tc_wait_ld_regs(raw);
      bool pad = false;
      if constexpr (HAS_MASK) pad = (kbits[0] & kbits[1]) != 0xFFFFFFFFu;
      const bool masked = pad || (n0 + 64 > p.seq) || (CAUSAL && n0 + 63 > w.q0 + rb);
      if (masked) {
#pragma unroll
        for (int e = 0; e < NE; ++e) {
          const int c = e_col(e) - c0;
          const int n = n0 + c;
          bool allowed;
          if constexpr (HAS_MASK)
            allowed = (kbits[c / 32] >> (c % 32)) & 1u;
          else
            allowed = n < p.seq;
          if (CAUSAL) allowed = allowed && (n <= w.q0 + e_row(e));
          raw[e] = allowed ? raw[e] : __float_as_uint(-INFINITY);
        }
      }
    };
    // Publishes this half's per-row values v[2] (rows ra, ra + 8) and returns
    // the other half's, through shared memory and the pair's mbarrier (two
    // phases per item: maximum, then sum).
    auto exchange = [&](float* base, const float (&v)[2], float (&other)[2], uint32_t parity) {
      if ((lane & 3) == 0) {
        base[half * BM + ra] = v[0];
        base[half * BM + ra + 8] = v[1];
      }
      mbar_arrive(bar_pair(pair));
      if (!__all_sync(0xFFFFFFFFu, wait(bar_pair(pair), parity))) return false;
      other[0] = base[(half ^ 1) * BM + ra];
      other[1] = base[(half ^ 1) * BM + ra + 8];
      return true;
    };

    for (int it = blockIdx.x, k = 0; it < total_items && ok; it += gridDim.x, ++k) {
      const Item w = item_at(it);

      // pass A: row maxima of the raw scores. TMEM reads run one key tile
      // ahead (the next tile's load is issued before this tile's arithmetic;
      // tcgen05.wait::ld waits for all of a thread's loads, so at most one
      // tile is in flight when a wait is reached).
      uint32_t buf[2][NE];
      float mraw[2][2] = {{-INFINITY, -INFINITY}, {-INFINITY, -INFINITY}};
      ok = __all_sync(0xFFFFFFFFu, wait(bar_s_full(0), tile_par & 1u));
      if (!ok) break;
      tc_fence_after();
      issue_tile(0, buf[0]);
#pragma unroll
      for (int j = 0; j < L::kTiles; ++j) {
        if (j >= w.n_kv) break;
        finish_scores(w, j, buf[j & 1]);
        if (j + 1 < w.n_kv) {
          ok = __all_sync(0xFFFFFFFFu, wait(bar_s_full(j + 1), (tile_par >> (j + 1)) & 1u));
          if (!ok) break;
          tc_fence_after();
          issue_tile(j + 1, buf[(j + 1) & 1]);
        }
#pragma unroll
        for (int e = 0; e < NE; e += 2) {
          const int h = (e >> 1) & 1;
          const int q = (e >> 2) & 1;
          mraw[h][q] = fmaxf(mraw[h][q], fmaxf(__uint_as_float(buf[j & 1][e]),
                                               __uint_as_float(buf[j & 1][e + 1])));
        }
      }
      if (!ok) break;
      float mx[2], mo[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float m = fmaxf(mraw[h][0], mraw[h][1]);
        m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
        mx[h] = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
      }
      ok = exchange(st_max, mx, mo, 0);
      if (!ok) break;
      // the scores' row maximum with the reference's dtype boundaries, in
      // log2 units (the two-pass schedule's m_fin)
      float m_use[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float m = fmaxf(mx[h], mo[h]);
        float z = m;
        round_pair<T>(m, z);  // T(max qk)
        m *= scale;
        if (!pow2) round_pair<T>(m, z);  // T(T(max qk) * scale)
        const float ml = m * kLog2e;
        m_use[h] = ml == -INFINITY ? 0.f : ml;
      }

      // pass B: e = exp(s - max) over the scores, written back in place
      // (MUFU-bound: its loads are not pipelined, which would spill at the
      // 96 registers a thread has with 18 warps)
      float part[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
      for (int j = 0; j < w.n_kv; ++j) {
        uint32_t (&raw)[NE] = buf[0];
        issue_tile(j, raw);
        finish_scores(w, j, raw);
#pragma unroll
        for (int i = 0; i < NE / 2; ++i) {
          const int h = i & 1;
          float a, c;
          unpack2<T>(cvt_pack2<T>(__uint_as_float(raw[2 * i]), __uint_as_float(raw[2 * i + 1])),
                     a, c);
          if (pow2) {
            fma2(a, c, scale_log2e, scale_log2e, -m_use[h], -m_use[h]);
          } else {
            mul2(a, c, scale, scale);
            round_pair<T>(a, c);
            fma2(a, c, kLog2e, kLog2e, -m_use[h], -m_use[h]);
          }
          a = ex2_approx(a);
          c = ex2_approx(c);
          add2(part[h][0], part[h][1], a, c);
          raw[2 * i] = __float_as_uint(a);
          raw[2 * i + 1] = __float_as_uint(c);
        }
        tmem_st16x256b<8>(tmem + lane_off + j * BN + c0, raw);
      }
      // row sums: this half over the row's four threads (each thread adds the
      // same values in the same order, so all four agree bitwise), then the
      // two halves in the order (half 0) + (half 1) on both warps
      float ls[2], lo[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float l = part[h][0] + part[h][1];
        l = l + __shfl_xor_sync(0xFFFFFFFFu, l, 1);
        ls[h] = l + __shfl_xor_sync(0xFFFFFFFFu, l, 2);
      }
      ok = exchange(st_sum, ls, lo, 1);
      if (!ok) break;
      float inv_l[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float l = half == 0 ? ls[h] + lo[h] : lo[h] + ls[h];
        inv_l[h] = l > 0.f ? 1.f / l : 0.f;
      }
      tc_wait_st();

      // pass C: P = T(e / sum), last tile first (O lives in tile 3), packed
      // in place in the registers and stored into the first 32 columns of
      // this half (16x128b shape: column 4g + i % 4 of repetition g holds
      // the key pair 8g + 2(i % 4), + 1 a thread holds)
      issue_tile(w.n_kv - 1, buf[0]);
#pragma unroll
      for (int i = 0; i < L::kTiles; ++i) {
        if (i >= w.n_kv) break;
        const int j = w.n_kv - 1 - i;
        uint32_t (&ev)[NE] = buf[i & 1];
        tc_wait_ld_regs(ev);
        if (j > 0) issue_tile(j - 1, buf[(i + 1) & 1]);
#pragma unroll
        for (int q = 0; q < NE / 2; ++q) {
          const int h = q & 1;
          float a = __uint_as_float(ev[2 * q]), c = __uint_as_float(ev[2 * q + 1]);
          mul2(a, c, inv_l[h], inv_l[h]);
          ev[q] = cvt_pack2<T>(a, c);
        }
        tmem_st16x128b_x8(tmem + lane_off + j * BN + (half ? L::kPCol1 : 0), ev);
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(bar_p_full(j));
      }

      // epilogue: this half's 32 head-dim columns of O (already normalised),
      // rounded to T
      ok = __all_sync(0xFFFFFFFFu, wait(bar_pv_done, k & 1));
      if (!ok) break;
      tc_fence_after();
      uint32_t o[16];
      tmem_ld16x256b<4>(tmem + lane_off + L::kOCol + 32 * half, o);
      tc_wait_ld();
      tc_fence_before();
      mbar_arrive(bar_o_empty);
#pragma unroll
      for (int e = 0; e < 16; e += 2) {
        const int m = w.q0 + e_row(e);
        if (m < p.seq) {
          T* dst = reinterpret_cast<T*>(p.out) +
                   ((static_cast<int64_t>(w.b) * p.seq + m) * p.heads + w.h) * D + 32 * half +
                   8 * (e >> 2) + cq;
          *reinterpret_cast<uint32_t*>(dst) =
              cvt_pack2<T>(__uint_as_float(o[e]), __uint_as_float(o[e + 1]));
        }
      }
      tile_par ^= (1u << w.n_kv) - 1u;
    }
  }

  // ------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == L::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// Launches the row-resident schedule (16-bit T, head_dim 64, seq_len <= 512):
// one persistent CTA per SM (at most one per item).
template <typename T>
cudaError_t launch_resident(AttnTcParams prm, int num_sms, bool causal, bool has_mask,
                            cudaStream_t stream);

extern template cudaError_t launch_resident<__half>(AttnTcParams, int, bool, bool, cudaStream_t);
extern template cudaError_t launch_resident<__nv_bfloat16>(AttnTcParams, int, bool, bool,
                                                           cudaStream_t);

}  // namespace tc
}  // namespace b200tk
