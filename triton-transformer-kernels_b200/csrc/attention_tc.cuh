// attention_tc.cuh - fused attention forward on sm_100a tensor cores.
//
// One CTA owns a 128-row query tile of one (batch, head) and walks the key /
// value tiles of that head with an online softmax (the algorithm of the
// reference kernel transformer_opt/kernels/attention.py:103-265):
//   * warp 4 (producer)  : TMA loads of Q once and of K/V tiles into
//                          KST/VST-deep smem rings (128-byte swizzle).
//   * warp 5 (MMA issuer): one elected thread issues tcgen05.mma:
//                          S_j = Q K_j^T into a double-buffered TMEM score
//                          tile, then O += P_j V_j with P read from TMEM.
//   * warps 0-3 (softmax): thread r owns query row r (TMEM lane r). It reads
//                          S_j with tcgen05.ld, reproduces the reference's
//                          dtype boundaries, masks (causal diagonal, sequence
//                          end, key padding), keeps the running max / sum in
//                          fp32, writes P_j back into TMEM, rescales O only
//                          when its running max grew by more than 2^8, and
//                          finally normalises O and stores the output row.
//   * warps 6-9 (fp32 only): split every fp32 tile in smem into a tf32 "hi"
//                          part (in place) and the residual "lo" part, so
//                          that each product runs as hi*hi + hi*lo + lo*hi
//                          (3xTF32) on the tf32 tensor-core path.
// Causal tiles beyond the diagonal are never loaded (the key loop ends at
// min(S, q0 + 128)), matching the reference's end bound (:163-166).
//
// Every mbarrier wait is bounded (ptx_sm100.cuh mbar_wait): on timeout the
// CTA raises an abort flag and a device status bit, drains its own copies and
// MMAs with further bounded waits, frees TMEM and returns.

#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "attention.h"
#include "ptx_sm100.cuh"

namespace b200tk {
namespace tc {

constexpr int BM = 128;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per wait
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

struct __align__(64) AttnTcParams {
  CUtensorMap tm_q;
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  void* out;
  const uint8_t* mask;
  int64_t mask_sb, mask_ss;
  int batch, seq, heads, n_qtiles;
  float scale;
  int causal_reverse;  // schedule longest causal tiles first
  unsigned int* status;
};

template <typename T>
struct ElemTraits;
template <>
struct ElemTraits<float> {
  static constexpr uint32_t kFmt = 2;  // tf32
  static constexpr bool kSplit = true;
};
template <>
struct ElemTraits<__half> {
  static constexpr uint32_t kFmt = 0;
  static constexpr bool kSplit = false;
};
template <>
struct ElemTraits<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;
  static constexpr bool kSplit = false;
};

// Round a pair of fp32 scores to T and back (the reference rounds the GEMM
// output and the scaled scores to the input dtype, dispatch.py:81-82 and
// attention.py:215-216).
template <typename T>
__device__ __forceinline__ void round_pair(float& a, float& b) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    uint32_t u = *reinterpret_cast<uint32_t*>(&h);
    a = __uint_as_float(u << 16);
    b = __uint_as_float(u & 0xFFFF0000u);
  } else if constexpr (std::is_same_v<T, __half>) {
    __half2 h = __floats2half2_rn(a, b);
    float2 f = __half22float2(h);
    a = f.x;
    b = f.y;
  }
}

template <typename T>
__device__ __forceinline__ uint32_t pack_pair(float a, float b) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <typename T, int D, int BN, int KST, int VST>
struct TcLayout {
  static constexpr bool kSplit = ElemTraits<T>::kSplit;
  static constexpr int kElem = sizeof(T);
  static constexpr int kAtomElems = 128 / kElem;  // elements per 128-byte row
  static constexpr int kAtoms = D / kAtomElems;   // swizzle atoms along head_dim
  static constexpr int kUmmaK = 32 / kElem;       // K per MMA instruction
  static constexpr int kQBytes = BM * D * kElem;
  static constexpr int kKVBytes = BN * D * kElem;
  static constexpr int kCopies = kSplit ? 2 : 1;  // hi (+ lo) buffers
  // smem offsets (all multiples of 1024)
  static constexpr int kQ = 0;
  static constexpr int kQlo = kQ + kQBytes;
  static constexpr int kK = kQ + kCopies * kQBytes;
  static constexpr int kKStage = kCopies * kKVBytes;  // hi then lo
  static constexpr int kV = kK + KST * kKStage;
  static constexpr int kVStage = kCopies * kKVBytes;
  static constexpr int kBar = kV + VST * kVStage;
  static constexpr int kNumBars = 1 + 1 + 3 * KST + 3 * VST + 2 + 1 + 1 + 1;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 64 + 1024;  // + alignment slack
  // TMEM columns
  // 16-bit: P (packed pairs) overwrites the first BN/2 columns of its S
  // buffer. fp32: P hi and P lo get buffers of their own, so no score MMA
  // ever writes columns a P@V MMA may still be reading.
  static constexpr int kTS = 0;                          // S buffers: 2 x BN
  static constexpr int kTPhi = kSplit ? 2 * BN : 0;      // fp32: P hi, 2 x BN
  static constexpr int kTPlo = 4 * BN;                   // fp32: P lo, 2 x BN
  static constexpr int kTO = kSplit ? 6 * BN : 2 * BN;   // O: D columns
  static constexpr int kTCols = kTO + D;
  static constexpr uint32_t kTAlloc = kTCols <= 32    ? 32
                                      : kTCols <= 64  ? 64
                                      : kTCols <= 128 ? 128
                                      : kTCols <= 256 ? 256
                                                      : 512;
  static constexpr int kThreads = kSplit ? 320 : 192;
  // V (MN-major B operand of P@V): 16-bit types use the 128-byte swizzle
  // (8-row groups, SBO 1024 B); tf32 requires the 128B_BASE32B swizzle
  // (32-byte chunks, 4-row groups, SBO 512 B), loaded by TMA with
  // SWIZZLE_128B_ATOM_32B.
  static constexpr uint32_t kVLayout = kSplit ? kLayoutSw128Base32b : kLayoutSw128;
  static constexpr uint32_t kVSbo = kSplit ? 512 : 1024;
  static_assert(kTCols <= 512, "TMEM budget");
  static_assert(D % kAtomElems == 0, "head_dim must fill whole swizzle atoms");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
};

template <typename T, int D, int BN, int KST, int VST, bool CAUSAL, bool HAS_MASK>
__global__ void __launch_bounds__(TcLayout<T, D, BN, KST, VST>::kThreads, 1)
    attention_fwd_tc_kernel(const __grid_constant__ AttnTcParams p) {
  using L = TcLayout<T, D, BN, KST, VST>;
  constexpr bool kSplit = L::kSplit;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_u32(smem);

  // barrier addresses
  const uint32_t bar0 = sbase + L::kBar;
  const uint32_t bar_q_full = bar0 + 0;
  const uint32_t bar_q_ready = bar0 + 8;
  auto bar_k_full = [&](int s) { return bar0 + 16 + 8 * s; };
  auto bar_k_ready = [&](int s) { return bar0 + 16 + 8 * (KST + s); };
  auto bar_k_empty = [&](int s) { return bar0 + 16 + 8 * (2 * KST + s); };
  const uint32_t vb = bar0 + 16 + 8 * 3 * KST;
  auto bar_v_full = [&](int s) { return vb + 8 * s; };
  auto bar_v_ready = [&](int s) { return vb + 8 * (VST + s); };
  auto bar_v_empty = [&](int s) { return vb + 8 * (2 * VST + s); };
  const uint32_t bar_s_full0 = vb + 8 * 3 * VST;
  const uint32_t bar_p_full = bar_s_full0 + 16;
  const uint32_t bar_pv_done = bar_p_full + 8;
  const uint32_t bar_drain = bar_pv_done + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 8);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  // tile scheduling: consecutive CTAs share one (batch, head) so its K/V
  // stay hot in L2; causal tiles run longest first.
  const int linear = blockIdx.x;
  const int bh = linear / p.n_qtiles;
  int qt = linear - bh * p.n_qtiles;
  if (CAUSAL && p.causal_reverse) qt = p.n_qtiles - 1 - qt;
  const int b = bh / p.heads;
  const int h = bh - b * p.heads;
  const int q0 = qt * BM;
  const int kv_end = CAUSAL ? min(p.seq, q0 + BM) : p.seq;
  const int n_kv = (kv_end + BN - 1) / BN;

  if (tid == 0) {
    mbar_init(bar_q_full, 1);
    mbar_init(bar_q_ready, 128);
    for (int s = 0; s < KST; ++s) {
      mbar_init(bar_k_full(s), 1);
      mbar_init(bar_k_ready(s), 128);
      mbar_init(bar_k_empty(s), 1);
    }
    for (int s = 0; s < VST; ++s) {
      mbar_init(bar_v_full(s), 1);
      mbar_init(bar_v_ready(s), 128);
      mbar_init(bar_v_empty(s), 1);
    }
    mbar_init(bar_s_full0, 1);
    mbar_init(bar_s_full0 + 8, 1);
    mbar_init(bar_p_full, 128);
    mbar_init(bar_pv_done, 1);
    mbar_init(bar_drain, 1);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), L::kTAlloc);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Tile schedule. 16-bit inputs take two passes over the key tiles: pass 1
  // only accumulates the row max and row sum, pass 2 forms probabilities
  // that are already normalised, rounds them to T and multiplies by V -- the
  // explicit reference's rounding boundary (softmax in fp32, then cast, then
  // P@V). fp32 inputs take one online pass (P keeps ~fp32 precision through
  // the 3xTF32 split, so normalising at the end is equivalent).
  constexpr bool kTwoPass = !kSplit;
  const int n_s = kTwoPass ? 2 * n_kv : n_kv;  // score tiles the CTA computes
  auto in_pass2 = [&](int g) { return !kTwoPass || g >= n_kv; };
  auto tile_of = [&](int g) { return (kTwoPass && g >= n_kv) ? g - n_kv : g; };

  if (warp == 4) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_q);
      tma_prefetch_desc(&p.tm_k);
      tma_prefetch_desc(&p.tm_v);
      int issued_k[KST] = {};
      int issued_v[VST] = {};
      bool ok = true;
      mbar_arrive_expect_tx(bar_q_full, L::kQBytes);
#pragma unroll
      for (int a = 0; a < L::kAtoms; ++a)
        tma_load_4d(sbase + L::kQ + a * BM * 128, &p.tm_q, bar_q_full, a * L::kAtomElems, h, q0, b);
      for (int g = 0; g < n_s && ok; ++g) {
        const int j = tile_of(g);
        const int s = g % KST;
        if (g >= KST)
          ok = mbar_wait(bar_k_empty(s), ((g / KST) - 1) & 1, abort_flag, p.status,
                         B200TK_STATUS_PIPELINE_TIMEOUT, kWaitLimitNs);
        if (!ok) break;
        mbar_arrive_expect_tx(bar_k_full(s), L::kKVBytes);
        const uint32_t kdst = sbase + L::kK + s * L::kKStage;
#pragma unroll
        for (int a = 0; a < L::kAtoms; ++a)
          tma_load_4d(kdst + a * BN * 128, &p.tm_k, bar_k_full(s), a * L::kAtomElems, h, j * BN, b);
        ++issued_k[s];
        if (!in_pass2(g)) continue;
        const int sv = j % VST;
        if (j >= VST)
          ok = mbar_wait(bar_v_empty(sv), ((j / VST) - 1) & 1, abort_flag, p.status,
                         B200TK_STATUS_PIPELINE_TIMEOUT, kWaitLimitNs);
        if (!ok) break;
        mbar_arrive_expect_tx(bar_v_full(sv), L::kKVBytes);
        const uint32_t vdst = sbase + L::kV + sv * L::kVStage;
#pragma unroll
        for (int a = 0; a < L::kAtoms; ++a)
          tma_load_4d(vdst + a * BN * 128, &p.tm_v, bar_v_full(sv), a * L::kAtomElems, h, j * BN, b);
        ++issued_v[sv];
      }
      if (*abort_flag) {
        // drain: every copy this thread started lands before the CTA exits
        mbar_wait(bar_q_full, 0, abort_flag, nullptr, 0, kWaitLimitNs);
        for (int s = 0; s < KST; ++s)
          if (issued_k[s] > 0) {
            const uint32_t par = (issued_k[s] - 1) & 1;
            uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(bar_k_full(s), par) && globaltimer_ns() - t0 < kWaitLimitNs) {
            }
          }
        for (int s = 0; s < VST; ++s)
          if (issued_v[s] > 0) {
            const uint32_t par = (issued_v[s] - 1) & 1;
            uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(bar_v_full(s), par) && globaltimer_ns() - t0 < kWaitLimitNs) {
            }
          }
      }
    }
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kFmt = ElemTraits<T>::kFmt;
      constexpr uint32_t idesc_qk = make_idesc(kFmt, 0, 0, BN, BM);  // Q K-major, K K-major
      constexpr uint32_t idesc_pv = make_idesc(kFmt, 0, 1, D, BM);   // P (tmem), V MN-major
      const uint32_t bar_q = kSplit ? bar_q_ready : bar_q_full;
      bool ok = mbar_wait(bar_q, 0, abort_flag, p.status, B200TK_STATUS_PIPELINE_TIMEOUT,
                          kWaitLimitNs);
      tc_fence_after();

      auto issue_s = [&](int g) -> bool {
        const int s = g % KST;
        const uint32_t bar_k = kSplit ? bar_k_ready(s) : bar_k_full(s);
        if (!mbar_wait(bar_k, (g / KST) & 1, abort_flag, p.status, B200TK_STATUS_PIPELINE_TIMEOUT,
                       kWaitLimitNs))
          return false;
        tc_fence_after();
        const uint32_t d_tmem = tmem + L::kTS + (g & 1) * BN;
        const uint32_t qa = sbase + L::kQ;
        const uint32_t kb = sbase + L::kK + s * L::kKStage;
        constexpr int kSteps = D / L::kUmmaK;
        constexpr int kPasses = kSplit ? 3 : 1;
#pragma unroll
        for (int pass = 0; pass < kPasses; ++pass) {
          // 3xTF32 order: lo*hi, hi*lo, hi*hi (small terms first)
          const uint32_t a_off = (kSplit && pass == 0) ? L::kQlo - L::kQ : 0;
          const uint32_t b_off = (kSplit && pass == 1) ? L::kKVBytes : 0;
#pragma unroll
          for (int ks = 0; ks < kSteps; ++ks) {
            const int byte = ks * 32;
            const int atom = byte / 128;
            const int within = byte % 128;
            const uint64_t adesc =
                make_sdesc(qa + a_off + atom * BM * 128 + within, 16, 1024, kLayoutSw128);
            const uint64_t bdesc =
                make_sdesc(kb + b_off + atom * BN * 128 + within, 16, 1024, kLayoutSw128);
            if constexpr (kSplit)
              mma_ss_tf32(d_tmem, adesc, bdesc, idesc_qk, (pass > 0 || ks > 0) ? 1u : 0u);
            else
              mma_ss_f16(d_tmem, adesc, bdesc, idesc_qk, ks > 0 ? 1u : 0u);
          }
        }
        tc_commit(bar_k_empty(s));
        tc_commit(bar_s_full0 + 8 * (g & 1));
        return true;
      };

      if (ok) ok = issue_s(0);
      if (ok && n_s > 1) ok = issue_s(1);
      for (int g = 0; g < n_s && ok; ++g) {
        // the softmax warps are done with S_g (and wrote P_g in pass 2)
        ok = mbar_wait(bar_p_full, g & 1, abort_flag, p.status, B200TK_STATUS_PIPELINE_TIMEOUT,
                       kWaitLimitNs);
        if (!ok) break;
        if (in_pass2(g)) {
          const int j = tile_of(g);
          const int sv = j % VST;
          const uint32_t bar_v = kSplit ? bar_v_ready(sv) : bar_v_full(sv);
          ok = mbar_wait(bar_v, (j / VST) & 1, abort_flag, p.status,
                         B200TK_STATUS_PIPELINE_TIMEOUT, kWaitLimitNs);
          if (!ok) break;
          tc_fence_after();
          const uint32_t o_tmem = tmem + L::kTO;
          const uint32_t vbuf = sbase + L::kV + sv * L::kVStage;
          constexpr int kSteps = BN / L::kUmmaK;
          constexpr int kPasses = kSplit ? 3 : 1;
#pragma unroll
          for (int pass = 0; pass < kPasses; ++pass) {
            const uint32_t p_tmem = !kSplit    ? tmem + L::kTS + (g & 1) * BN
                                    : pass == 0 ? tmem + L::kTPlo + (g & 1) * BN
                                                : tmem + L::kTPhi + (g & 1) * BN;
            const uint32_t v_off = (kSplit && pass == 1) ? L::kKVBytes : 0;
#pragma unroll
            for (int ks = 0; ks < kSteps; ++ks) {
              // V is MN-major: K advances over 128-byte rows; LBO steps across
              // head_dim atoms, SBO across the swizzle's row groups.
              const uint64_t bdesc = make_sdesc(vbuf + v_off + ks * L::kUmmaK * 128, BN * 128,
                                                L::kVSbo, L::kVLayout);
              const uint32_t a_tmem = p_tmem + ks * 8;  // 8 columns per K step
              const uint32_t acc = (j > 0 || pass > 0 || ks > 0) ? 1u : 0u;
              if constexpr (kSplit)
                mma_ts_tf32(o_tmem, a_tmem, bdesc, idesc_pv, acc);
              else
                mma_ts_f16(o_tmem, a_tmem, bdesc, idesc_pv, acc);
            }
          }
          tc_commit(bar_v_empty(sv));
          tc_commit(bar_pv_done);
        }
        if (g + 2 < n_s) ok = issue_s(g + 2);
      }
      // make sure no MMA is still writing TMEM when the CTA tears down
      tc_commit(bar_drain);
      uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(bar_drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
  } else if (kSplit && warp >= 6) {
    // ------------------------------------------- fp32 hi/lo split workers
    const int t = tid - 192;  // 0..127
    auto split_tile = [&](uint32_t off, int bytes) {
      float4* hi = reinterpret_cast<float4*>(smem + off);
      float4* lo = reinterpret_cast<float4*>(smem + off + bytes);
      for (int i = t; i < bytes / 16; i += 128) {
        float4 x = hi[i];
        float4 xh, xl;
        xh.x = __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
        xh.y = __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
        xh.z = __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
        xh.w = __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
        xl.x = x.x - xh.x;
        xl.y = x.y - xh.y;
        xl.z = x.z - xh.z;
        xl.w = x.w - xh.w;
        hi[i] = xh;
        lo[i] = xl;
      }
      fence_proxy_async_smem();
    };
    bool ok = mbar_wait(bar_q_full, 0, abort_flag, p.status, B200TK_STATUS_PIPELINE_TIMEOUT,
                        kWaitLimitNs);
    if (ok) {
      split_tile(L::kQ, L::kQBytes);
      mbar_arrive(bar_q_ready);
    }
    for (int j = 0; j < n_kv && ok; ++j) {
      const int s = j % KST;
      ok = mbar_wait(bar_k_full(s), (j / KST) & 1, abort_flag, p.status,
                     B200TK_STATUS_PIPELINE_TIMEOUT, kWaitLimitNs);
      if (!ok) break;
      split_tile(L::kK + s * L::kKStage, L::kKVBytes);
      mbar_arrive(bar_k_ready(s));
      const int sv = j % VST;
      ok = mbar_wait(bar_v_full(sv), (j / VST) & 1, abort_flag, p.status,
                     B200TK_STATUS_PIPELINE_TIMEOUT, kWaitLimitNs);
      if (!ok) break;
      split_tile(L::kV + sv * L::kVStage, L::kKVBytes);
      mbar_arrive(bar_v_ready(sv));
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------- softmax
    const int r = tid;  // query row within the tile == TMEM lane
    const int m = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const int warp_row0 = q0 + warp * 32;
    float m_ref = -INFINITY;  // running max, log2 units
    float l_sum = 0.f;
    float m_fin = 0.f, inv_l = 0.f;  // two-pass: final max and 1/sum
    bool ok = true;
    const float scale = p.scale;

    for (int g = 0; g < n_s && ok; ++g) {
      const int buf = g & 1;
      const int j = tile_of(g);
      const bool pass2 = in_pass2(g);
      // warp-uniform outcome: the tcgen05.ld/st below are warp-collective
      ok = __all_sync(0xFFFFFFFFu, mbar_wait(bar_s_full0 + 8 * buf, (g >> 1) & 1, abort_flag,
                                             p.status, B200TK_STATUS_PIPELINE_TIMEOUT,
                                             kWaitLimitNs));
      if (!ok) break;
      tc_fence_after();
      const int n0 = j * BN;
      // key-padding bits for this tile: warp-cooperative load + ballot
      uint32_t kbits[BN / 32];
      if constexpr (HAS_MASK) {
#pragma unroll
        for (int w = 0; w < BN / 32; ++w) {
          const int n = n0 + w * 32 + lane;
          bool valid = false;
          if (n < p.seq) valid = p.mask[b * p.mask_sb + n * p.mask_ss] != 0;
          kbits[w] = __ballot_sync(0xFFFFFFFFu, valid);
        }
      }
      float s[BN];
      {
        uint32_t raw[BN / 32][32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          tmem_ld32(tmem + lane_off + L::kTS + buf * BN + c * 32, raw[c]);
        tc_wait_ld();
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(raw[c][i]);
      }
      // dtype boundaries of the explicit reference: (round(round(qk) * scale))
      if constexpr (std::is_same_v<T, float>) {
#pragma unroll
        for (int i = 0; i < BN; ++i) s[i] *= scale;
      } else {
#pragma unroll
        for (int i = 0; i < BN; i += 2) {
          round_pair<T>(s[i], s[i + 1]);
          s[i] *= scale;
          s[i + 1] *= scale;
          round_pair<T>(s[i], s[i + 1]);
        }
      }
      const bool tail = n0 + BN > p.seq;
      const bool diag = CAUSAL && (n0 + BN - 1 > warp_row0);
      if (HAS_MASK || tail || diag) {
#pragma unroll
        for (int i = 0; i < BN; ++i) {
          const int n = n0 + i;
          bool allowed;
          if constexpr (HAS_MASK)
            allowed = (kbits[i / 32] >> (i % 32)) & 1u;
          else
            allowed = n < p.seq;
          if (CAUSAL) allowed = allowed && (n <= m);
          s[i] = allowed ? s[i] : -INFINITY;
        }
      }

      // pv_done is a parity barrier: it only tells the current phase from the
      // previous one. The softmax warps therefore wait for every P@V phase in
      // order (PV_{j-1} before storing P_j), which keeps the barrier at most one
      // phase ahead and also orders any O rescale after the MMA that wrote O.
      auto wait_prev_pv = [&]() -> bool {
        if (j == 0) return true;
        const bool done = mbar_wait(bar_pv_done, (j - 1) & 1, abort_flag, p.status,
                                    B200TK_STATUS_PIPELINE_TIMEOUT, kWaitLimitNs);
        return __all_sync(0xFFFFFFFFu, done);
      };

      if constexpr (kTwoPass) {
        if (!pass2) {
          // pass 1: running max and sum only
          float mx = -INFINITY;
#pragma unroll
          for (int i = 0; i < BN; ++i) mx = fmaxf(mx, s[i]);
          const float m_new = fmaxf(m_ref, mx * kLog2e);
          const float m_use = m_new == -INFINITY ? 0.f : m_new;
          const float alpha = m_ref == -INFINITY ? 0.f : ex2_approx(m_ref - m_use);
          float part = 0.f;
#pragma unroll
          for (int i = 0; i < BN; ++i) part += ex2_approx(fmaf(s[i], kLog2e, -m_use));
          l_sum = l_sum * alpha + part;
          m_ref = m_new;
          if (j == n_kv - 1) {
            m_fin = m_ref == -INFINITY ? 0.f : m_ref;
            inv_l = l_sum > 0.f ? 1.f / l_sum : 0.f;
          }
          tc_fence_before();
          mbar_arrive(bar_p_full);
          continue;
        }
        // pass 2: normalised probabilities, rounded to T, into TMEM
        uint32_t pk[BN / 2];
#pragma unroll
        for (int i = 0; i < BN / 2; ++i) {
          const float p0 = ex2_approx(fmaf(s[2 * i], kLog2e, -m_fin)) * inv_l;
          const float p1 = ex2_approx(fmaf(s[2 * i + 1], kLog2e, -m_fin)) * inv_l;
          pk[i] = pack_pair<T>(p0, p1);
        }
        if (!wait_prev_pv()) {
          ok = false;
          break;
        }
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          tmem_st16(tmem + lane_off + L::kTS + buf * BN + c * 16, &pk[c * 16]);
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(bar_p_full);
      } else {
        // one online pass (fp32 / 3xTF32)
        float mx = -INFINITY;
#pragma unroll
        for (int i = 0; i < BN; ++i) mx = fmaxf(mx, s[i]);
        const float m_new = fmaxf(m_ref, mx * kLog2e);  // -inf stays -inf
        bool rescale = false;
        float alpha = 1.f;
        if (j == 0) {
          m_ref = m_new;
        } else if (__any_sync(0xFFFFFFFFu, m_new > m_ref + kRescaleThreshold)) {
          // the running max grew by more than 2^8: move every row of this
          // warp to its new max (rows whose max did not grow keep alpha = 1)
          rescale = true;
          if (m_new > m_ref) {
            alpha = ex2_approx(m_ref - m_new);
            m_ref = m_new;
          }
          l_sum *= alpha;
        }
        const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
        uint32_t ph[BN], pl[BN];
#pragma unroll
        for (int i = 0; i < BN; ++i) {
          const float pv = ex2_approx(fmaf(s[i], kLog2e, -m_use));
          l_sum += pv;
          const uint32_t hb = __float_as_uint(pv) & 0xFFFFE000u;
          ph[i] = hb;
          pl[i] = __float_as_uint(pv - __uint_as_float(hb));
        }
        if (!wait_prev_pv()) {
          ok = false;
          break;
        }
        if (rescale) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            const uint32_t addr = tmem + lane_off + L::kTO + c * 32;
            tmem_ld32(addr, o);
            tc_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(addr, o);
          }
        }
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          tmem_st32(tmem + lane_off + L::kTPhi + buf * BN + c * 32,
                    *reinterpret_cast<const uint32_t(*)[32]>(&ph[c * 32]));
          tmem_st32(tmem + lane_off + L::kTPlo + buf * BN + c * 32,
                    *reinterpret_cast<const uint32_t(*)[32]>(&pl[c * 32]));
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(bar_p_full);
      }
    }

    // ------------------------------------------------------------ epilogue
    if (ok) {
      ok = mbar_wait(bar_pv_done, (n_kv - 1) & 1, abort_flag, p.status,
                     B200TK_STATUS_PIPELINE_TIMEOUT, kWaitLimitNs);
      ok = __all_sync(0xFFFFFFFFu, ok);
    }
    if (ok) {
      tc_fence_after();
      // two-pass: O is already normalised; one pass: divide by the row sum
      const float out_scale = kTwoPass ? 1.f : (l_sum > 0.f ? 1.f / l_sum : 0.f);
      T* out_row = reinterpret_cast<T*>(p.out) +
                   ((static_cast<int64_t>(b) * p.seq + m) * p.heads + h) * D;
      const bool row_ok = m < p.seq;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tmem + lane_off + L::kTO + c * 32, o);
        tc_wait_ld();
        if (row_ok) {
          if constexpr (std::is_same_v<T, float>) {
            float4* dst = reinterpret_cast<float4*>(out_row + c * 32);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float4 v;
              v.x = __uint_as_float(o[4 * i + 0]) * out_scale;
              v.y = __uint_as_float(o[4 * i + 1]) * out_scale;
              v.z = __uint_as_float(o[4 * i + 2]) * out_scale;
              v.w = __uint_as_float(o[4 * i + 3]) * out_scale;
              dst[i] = v;
            }
          } else {
            uint4* dst = reinterpret_cast<uint4*>(out_row + c * 32);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              uint4 v;
              uint32_t* vv = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
              for (int e = 0; e < 4; ++e)
                vv[e] = pack_pair<T>(__uint_as_float(o[8 * i + 2 * e]) * out_scale,
                                     __uint_as_float(o[8 * i + 2 * e + 1]) * out_scale);
              dst[i] = v;
            }
          }
        }
      }
    }
  }

  // ------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTAlloc);
  }
}

template <typename T, int D, int BN, int KST, int VST, bool CAUSAL, bool HAS_MASK>
cudaError_t launch_tc(const AttnTcParams& prm, int grid, cudaStream_t stream) {
  using L = TcLayout<T, D, BN, KST, VST>;
  auto kernel = attention_fwd_tc_kernel<T, D, BN, KST, VST, CAUSAL, HAS_MASK>;
  // at least ~116 KB so that one CTA (and one TMEM allocation) owns each SM
  const int smem = L::kBytes > 118 * 1024 ? L::kBytes : 118 * 1024;
  cudaError_t err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (err != cudaSuccess) return err;
  kernel<<<grid, L::kThreads, smem, stream>>>(prm);
  return cudaGetLastError();
}

template <typename T, int D, int BN, int KST, int VST>
cudaError_t dispatch_flags(const AttnTcParams& prm, int grid, bool causal, bool has_mask,
                           cudaStream_t stream) {
  if (causal)
    return has_mask ? launch_tc<T, D, BN, KST, VST, true, true>(prm, grid, stream)
                    : launch_tc<T, D, BN, KST, VST, true, false>(prm, grid, stream);
  return has_mask ? launch_tc<T, D, BN, KST, VST, false, true>(prm, grid, stream)
                  : launch_tc<T, D, BN, KST, VST, false, false>(prm, grid, stream);
}

// Tile configuration per (dtype, head_dim): keys per tile (BN) and the K / V
// ring depths, chosen so that shared memory stays under the 227 KB opt-in
// limit (fp32 tiles carry both the tf32 hi and lo copies).
template <typename T, int D>
struct TcTile {
  static constexpr int kBN = 128, kKST = D == 64 ? 3 : 2, kVST = D == 64 ? 3 : 2;
};
template <>
struct TcTile<float, 64> {
  static constexpr int kBN = 64, kKST = 2, kVST = 2;
};
template <>
struct TcTile<float, 128> {
  static constexpr int kBN = 32, kKST = 2, kVST = 1;
};

template <typename T, int D>
cudaError_t launch_dtype_hd(const AttnTcParams& prm, int grid, bool causal, bool has_mask,
                            cudaStream_t stream) {
  using C = TcTile<T, D>;
  return dispatch_flags<T, D, C::kBN, C::kKST, C::kVST>(prm, grid, causal, has_mask, stream);
}

// Explicit instantiations live in attention_tc_inst.cu, compiled once per
// (dtype, head_dim) so the six variants build in parallel.
#define B200TK_TC_DECLARE(T, D)                                                              \
  extern template cudaError_t launch_dtype_hd<T, D>(const AttnTcParams&, int, bool, bool, \
                                                    cudaStream_t);
B200TK_TC_DECLARE(__nv_bfloat16, 64)
B200TK_TC_DECLARE(__nv_bfloat16, 128)
B200TK_TC_DECLARE(__half, 64)
B200TK_TC_DECLARE(__half, 128)
B200TK_TC_DECLARE(float, 64)
B200TK_TC_DECLARE(float, 128)
#undef B200TK_TC_DECLARE

}  // namespace tc
}  // namespace b200tk
