// attention_tc.cuh - fused attention forward on sm_100a tensor cores.
//
// A CTA owns work items of NQ (1 or 2) 128-row query tiles of one (batch,
// head) and walks the key / value tiles of that head (the algorithm of the
// reference kernel transformer_opt/kernels/attention.py:103-265):
//   * producer warp : TMA loads of the Q tiles and of K/V tiles into KST/VST
//                     deep smem rings (128-byte swizzle), shared by all query
//                     tiles of the CTA; the K and V rings are refilled
//                     independently.
//   * MMA warp(s)   : one elected lane issues tcgen05.mma: S_t = Q_t K_j^T
//                     into TMEM score buffers, then O_t += P_t V_j with P read
//                     from TMEM. 16-bit: one warp for both query tiles (each
//                     tile has one score buffer, so tile 0's softmax overlaps
//                     tile 1's MMAs and vice versa). fp32: one warp issues the
//                     score MMAs and another the P@V MMAs.
//   * softmax warps : eight per query tile, two threads per score row (TMEM
//                     lane r), each owning half of the key columns. They read
//                     S with tcgen05.ld, reproduce the reference's dtype
//                     boundaries, mask (causal diagonal, sequence end, key
//                     padding), keep the row max / sum in fp32, write P back
//                     into TMEM and finally store the normalised output row.
//                     16-bit inputs take two passes over the keys (row max
//                     and sum, then normalised P rounded to T); fp32 takes one
//                     online pass on 3xTF32.
//   * split warps   : (fp32 only) write the residual lo = x - tf32(x) of
//                     every K/V tile (the tf32 MMA truncates the raw tile to
//                     its hi part) and move Q hi / lo into TMEM once per item,
//                     so each product runs as lo*hi + hi*lo + hi*hi.
// Causal key tiles beyond the item's last query row are never loaded (the key
// loop ends at min(S, last row + 1)), the reference's end bound (:163-166).
// Launches are persistent (at most one CTA per SM walking the items; causal
// items are taken in (long, short) query-tile pairs of equal cost).
//
// Every mbarrier wait is bounded (ptx_sm100.cuh mbar_wait): on timeout the
// CTA raises an abort flag and a device status bit, drains its own copies and
// MMAs with further bounded waits, frees TMEM and returns. Parity barriers
// only tell the current phase from the previous one, so every waiter observes
// every phase of the barriers it waits on, in order.

#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
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
  int causal_pairs;    // persistent causal schedule over (long, short) tile pairs
  int scale_pow2;      // bf16 only: scale is an exact power of two
  int one_pass;        // 16-bit only: online softmax (see TcLayout::kTwoPass)
  unsigned int* status;
};

// Key-padding bound of every batch row of the mask: one past its last valid
// key (0 for a row without valid keys), computed by the whole CTA at set-up
// into shared memory (launches of at most kMaxMaskBatches rows; larger ones
// keep every key tile). Key tiles from that bound on hold only padding keys,
// whose probabilities are exactly zero, so no role loads or multiplies them;
// an item keeps at least one key tile, so a row without valid keys still
// takes the all-masked path and yields zeros.
constexpr int kMaxMaskBatches = 1024;
__device__ __forceinline__ void mask_key_bounds(const AttnTcParams& p, int* end) {
  const int warps = static_cast<int>(blockDim.x >> 5);
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  for (int b = warp; b < p.batch; b += warps) {
    const uint8_t* row = p.mask + static_cast<int64_t>(b) * p.mask_sb;
    int last = -1;
    int n0 = 0;
    if (p.mask_ss == 1 && (reinterpret_cast<uintptr_t>(row) & 15u) == 0) {
      // 16 bytes per lane and load; the highest nonzero byte of a word is
      // (31 - clz(word)) / 8 (little-endian)
      const int nv = p.seq >> 4;
      for (int i = lane; i < nv; i += 32) {
        const uint4 v = reinterpret_cast<const uint4*>(row)[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (w[q] != 0u) last = max(last, 16 * i + 4 * q + (31 - __clz(w[q])) / 8);
      }
      n0 = nv << 4;
    }
    for (int n = n0 + lane; n < p.seq; n += 32)
      if (row[static_cast<int64_t>(n) * p.mask_ss] != 0) last = max(last, n);
    last = __reduce_max_sync(0xFFFFFFFFu, last);
    if (lane == 0) end[b] = last + 1;
  }
}

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

// Row max / row sum over one score row in registers with 8 independent
// partial results: a single accumulator would make a dependency chain as
// long as the tile.
template <int N>
__device__ __forceinline__ float row_max(const float (&v)[N]) {
  float m[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) m[k] = v[k];
#pragma unroll
  for (int i = 8; i < N; ++i) m[i % 8] = fmaxf(m[i % 8], v[i]);
  return fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])),
               fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
}

// ---- packed pair arithmetic (sm_100 f32x2 and 16-bit x2 instructions)
// Two fp32 lanes per instruction: c = a * b, a * b + c, a + b, element-wise,
// each with one round-to-nearest-even rounding like the scalar forms.
__device__ __forceinline__ void mul2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "mul.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}
__device__ __forceinline__ void fma2(float& a0, float& a1, float b0, float b1, float c0, float c1) {
  asm("{\n\t.reg .b64 x, y, z;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "mov.b64 z, {%4, %5};\n\tfma.rn.f32x2 x, x, y, z;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void add2(float& a0, float& a1, float b0, float b1) {
  asm("{\n\t.reg .b64 x, y;\n\tmov.b64 x, {%0, %1};\n\tmov.b64 y, {%2, %3};\n\t"
      "add.rn.f32x2 x, x, y;\n\tmov.b64 {%0, %1}, x;\n\t}"
      : "+f"(a0), "+f"(a1)
      : "f"(b0), "f"(b1));
}

// Round two fp32 values to T and pack them (a in the low half).
template <typename T>
__device__ __forceinline__ uint32_t cvt_pack2(float a, float b) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}
template <typename T>
__device__ __forceinline__ void unpack2(uint32_t u, float& a, float& b) {
  if constexpr (std::is_same_v<T, __nv_bfloat16>) {
    a = __uint_as_float(u << 16);
    b = __uint_as_float(u & 0xFFFF0000u);
  } else {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&u));
    a = f.x;
    b = f.y;
  }
}
// Element-wise max of two packed T pairs (exact).
template <typename T>
__device__ __forceinline__ uint32_t max_pack2(uint32_t a, uint32_t b) {
  uint32_t d;
  if constexpr (std::is_same_v<T, __nv_bfloat16>)
    asm("max.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  else
    asm("max.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// OP (16-bit types only) selects the one-pass schedule: online softmax, P
// rounded to T before normalisation. Without it 16-bit types take two passes
// (row statistics first, then normalised P rounded to T: the explicit
// reference's rounding boundary). fp32 always takes one pass (3xTF32 keeps P
// at ~fp32 precision, so normalising at the end is equivalent).
template <typename T, int D, int BN, int KST, int VST, int NQ, bool OP = false>
struct TcLayout {
  static constexpr bool kSplit = ElemTraits<T>::kSplit;
  // Score buffers per query tile: two whenever TMEM holds them (the next
  // score MMA then overlaps the softmax of the current tile), else one.
  static constexpr int kNSB =
      (NQ * (ElemTraits<T>::kSplit ? 2 * BN + 2 * BN + 3 * D : 2 * BN + D)) <= 512 ? 2 : 1;
  static constexpr int kElem = sizeof(T);
  static constexpr int kAtomElems = 128 / kElem;  // elements per 128-byte row
  static constexpr int kAtoms = D / kAtomElems;   // swizzle atoms along head_dim
  static constexpr int kUmmaK = 32 / kElem;       // K per MMA instruction
  static constexpr int kQBytes = BM * D * kElem;
  static constexpr int kKVBytes = BN * D * kElem;
  static constexpr int kCopies = kSplit ? 2 : 1;  // K/V: hi (+ lo) buffers
  // smem offsets (all multiples of 1024). K/V tiles are stored hi then lo;
  // Q is stored once (fp32 Q hi / lo are moved into TMEM by the split warps).
  static constexpr int kQStage = kQBytes;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + NQ * kQStage;
  static constexpr int kKStage = kCopies * kKVBytes;
  static constexpr int kV = kK + KST * kKStage;
  static constexpr int kVStage = kCopies * kKVBytes;
  static constexpr bool kTwoPass = !kSplit && !OP;
  static constexpr bool kOnePass16 = !kSplit && OP;
  // Softmax threads per score row: 16-bit two-pass: two, each owning BN/2
  // keys (32x32b TMEM shape); one-pass and fp32: a warp covers 16 rows with
  // four threads per row (16x256b shape), two warps per 32-lane quadrant --
  // also 256 threads per query tile.
  static constexpr int kThreadsPerRow = 2;
  static constexpr int kSoftmaxWarpsPerTile = 4 * kThreadsPerRow;
  static constexpr int kSoftmaxWarps = NQ * kSoftmaxWarpsPerTile;
  // 16-bit (max, sum) exchange at the end of pass 1, float2 per thread (fp32
  // combines its row statistics with shuffles and needs none)
  static constexpr int kStats = kV + VST * kVStage;
  static constexpr int kBar = kStats + (kTwoPass ? NQ * kThreadsPerRow * BM * 8 : 0);
  // fp32 P layout. kPAlias: P hi is written back into the score buffer it
  // came from and every score buffer has a P-lo buffer of its own, so the
  // softmax stores P_j while P@V_{j-1} still runs (one pv_done barrier per
  // P-lo buffer); a score buffer is then reused after the P@V that read it.
  // Otherwise one P hi and one P lo buffer, and a score buffer is reused
  // once the softmax has read it. Measured: aliasing pays with 64-key tiles
  // (head_dim 64) and costs with 32-key tiles (head_dim 128).
  static constexpr bool kPAlias = kSplit && BN >= 64;
  static constexpr int kPvBufs = kPAlias ? kNSB : 1;
  static constexpr int kNumBars =
      2 + 3 * KST + 3 * VST + 2 * NQ * kNSB + NQ * kPvBufs + 2 * NQ + 2;
  static constexpr int kMisc = kBar + kNumBars * 8;
  static constexpr int kBytes = kMisc + 64 + 1024;  // + alignment slack
  // TMEM columns per query tile: S buffers, O, and for fp32 the P buffers
  // (kPAlias: a P lo buffer per score buffer, P hi written back into the
  // score buffer it came from; else one P hi and one P lo buffer) plus the
  // Q hi / Q lo operands of the score MMA. 16-bit P
  // (packed pairs) goes back into the score buffer it came from: each
  // half-row thread packs its BN/2 keys into the first BN/4 columns of its
  // own half, so no thread overwrites scores another thread has yet to read.
  static constexpr int kTileCols = !kSplit   ? kNSB * BN + D
                                   : kPAlias ? 2 * kNSB * BN + 3 * D
                                             : kNSB * BN + 2 * BN + 3 * D;
  static constexpr int kTCols = NQ * kTileCols;
  static constexpr uint32_t kTAlloc = kTCols <= 32    ? 32
                                      : kTCols <= 64  ? 64
                                      : kTCols <= 128 ? 128
                                      : kTCols <= 256 ? 256
                                                      : 512;
  __host__ __device__ static constexpr int t_s(int t, int b) { return t * kTileCols + b * BN; }
  __host__ __device__ static constexpr int t_phi(int t, int b) {
    return kPAlias ? t_s(t, b) : t * kTileCols + kNSB * BN;
  }
  __host__ __device__ static constexpr int t_plo(int t, int b) {
    return t * kTileCols + (kNSB + (kPAlias ? b : 1)) * BN;
  }
  __host__ __device__ static constexpr int t_o(int t) {
    return t * kTileCols + (!kSplit ? kNSB * BN : kPAlias ? 2 * kNSB * BN : (kNSB + 2) * BN);
  }
  __host__ __device__ static constexpr int t_qhi(int t) { return t_o(t) + D; }
  __host__ __device__ static constexpr int t_qlo(int t) { return t_o(t) + 2 * D; }
  // warps: [softmax][producer][MMA issuers][fp32: split x 4]. 16-bit: one
  // MMA warp for all query tiles; fp32: one for the score MMAs, one for P@V.
  static constexpr int kMmaWarps = kSplit ? 2 : 1;
  static constexpr int kProducerWarp = kSoftmaxWarps;
  static constexpr int kMmaWarp = kSoftmaxWarps + 1;
  static constexpr int kSplitWarp0 = kMmaWarp + kMmaWarps;
  static constexpr int kThreads = 32 * (kSplitWarp0 + (kSplit ? 4 : 0));
  // V (MN-major B operand of P@V): 16-bit types use the 128-byte swizzle
  // (8-row groups, SBO 1024 B); tf32 requires the 128B_BASE32B swizzle
  // (32-byte chunks, 4-row groups, SBO 512 B), loaded by TMA with
  // SWIZZLE_128B_ATOM_32B.
  static constexpr uint32_t kVLayout = kSplit ? kLayoutSw128Base32b : kLayoutSw128;
  static constexpr uint32_t kVSbo = kSplit ? 512 : 1024;
  static_assert(kTCols <= 512, "TMEM budget");
  static_assert(kBytes <= 232448, "shared memory budget");
  static_assert(D % kAtomElems == 0, "head_dim must fill whole swizzle atoms");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert(NQ == 1 || NQ == 2, "one or two query tiles per CTA");
  static_assert(!kSplit || NQ == 1, "fp32 keeps one query tile per CTA");
};

template <typename T, int D, int BN, int KST, int VST, int NQ, bool OP, bool CAUSAL,
          bool HAS_MASK>
__global__ void __launch_bounds__(TcLayout<T, D, BN, KST, VST, NQ, OP>::kThreads, 1)
    attention_fwd_tc_kernel(const __grid_constant__ AttnTcParams p) {
  using L = TcLayout<T, D, BN, KST, VST, NQ, OP>;
  constexpr bool kSplit = L::kSplit;
  constexpr int NSB = L::kNSB;
  constexpr bool kTwoPass = L::kTwoPass;
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
  const uint32_t tb = vb + 8 * 3 * VST;
  // One s_full and one p_full barrier per score buffer: the softmax warps
  // arrive on a buffer's p_full again only after the MMA warp has consumed
  // its previous phase (the next score tile of that buffer is issued after
  // it), so no parity phase can be skipped.
  auto bar_s_full = [&](int t, int buf) { return tb + 8 * (t * NSB + buf); };
  auto bar_p_full = [&](int t, int buf) { return tb + 8 * (NQ * NSB + t * NSB + buf); };
  const uint32_t tb2 = tb + 8 * (2 * NQ * NSB);
  constexpr int PVB = L::kPvBufs;
  auto bar_pv_done = [&](int t, int b) { return tb2 + 8 * (t * PVB + b); };
  const uint32_t tb3 = tb2 + 8 * (NQ * PVB);
  auto bar_stats = [&](int t) { return tb3 + 8 * t; };
  auto bar_o_empty = [&](int t) { return tb3 + 8 * (NQ + t); };
  const uint32_t bar_q_empty = tb3 + 8 * (2 * NQ);
  const uint32_t bar_drain = bar_q_empty + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMisc + 8);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

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
    for (int t = 0; t < NQ; ++t) {
      for (int bf = 0; bf < NSB; ++bf) {
        mbar_init(bar_s_full(t, bf), 1);
        mbar_init(bar_p_full(t, bf), 128 * L::kThreadsPerRow);
      }
      for (int bf = 0; bf < PVB; ++bf) mbar_init(bar_pv_done(t, bf), 1);
      mbar_init(bar_stats(t), 128 * L::kThreadsPerRow);
      mbar_init(bar_o_empty(t), 128 * L::kThreadsPerRow);
    }
    mbar_init(bar_q_empty, 1);
    mbar_init(bar_drain, L::kMmaWarps);
    *abort_flag = 0;
    fence_mbarrier_init();
  }
  if (warp == L::kMmaWarp) {
    tmem_alloc(smem_u32(tmem_slot), L::kTAlloc);
    tmem_relinquish();
  }
  __shared__ int s_kv_end[HAS_MASK ? kMaxMaskBatches : 1];
  const bool kv_bounds = HAS_MASK && p.batch <= kMaxMaskBatches;
  if (kv_bounds) mask_key_bounds(p, s_kv_end);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // Persistent schedule: CTA c processes work items c, c + gridDim.x, ...
  // An item is NQ query tiles of one (batch, head). Items of one batch-head
  // are adjacent (its K/V stay hot in L2) and, causally, longest first. Every
  // role walks the same item sequence, so mbarrier phases simply continue
  // from item to item: each role keeps running counts of the K tiles, V tiles
  // and items it has seen.
  //
  // 16-bit inputs take two passes over the key tiles: pass 1 only
  // accumulates the row max and row sum, pass 2 forms probabilities that are
  // already normalised, rounds them to T and multiplies by V -- the explicit
  // reference's rounding boundary (softmax in fp32, then cast, then P@V).
  // fp32 inputs take one online pass (P keeps ~fp32 precision through the
  // 3xTF32 split, so normalising at the end is equivalent).
  //
  // Causal items get longer with the query tile. With causal_pairs the
  // launch is persistent too: item index 2 * pair + member, where pair
  // (bh, pos) holds query tiles n - 1 - pos (member 0) and pos (member 1),
  // whose costs add up to the same for every pair; CTA c takes pairs c,
  // c + grid, ... (pairs of one batch-head are adjacent, so the CTAs in
  // flight share a few heads' K/V in L2). With an odd tile count the middle
  // tile's pair has one member.
  const int pair_half = (p.n_qtiles + 1) / 2;  // pairs per batch-head
  const int total_items = (CAUSAL && p.causal_pairs)
                              ? 2 * pair_half * p.batch * p.heads
                              : p.n_qtiles * p.batch * p.heads;
  auto item_valid = [&](int it) {
    if (!(CAUSAL && p.causal_pairs) || !(it & 1)) return true;
    const int pos = (it >> 1) % pair_half;
    return pos != p.n_qtiles - 1 - pos;
  };
  // first item of this CTA / the one after `it` (same sequence in every role)
  auto first_item = [&]() {
    int it = (CAUSAL && p.causal_pairs) ? 2 * static_cast<int>(blockIdx.x)
                                        : static_cast<int>(blockIdx.x);
    return it;
  };
  auto next_item = [&](int it) {
    if (CAUSAL && p.causal_pairs) {
      do {
        it = (it & 1) ? it + 2 * static_cast<int>(gridDim.x) - 1 : it + 1;
      } while (it < total_items && !item_valid(it));
      return it;
    }
    return it + static_cast<int>(gridDim.x);
  };
  struct Item {
    int b, h, q0, n_kv, n_s;
  };
  auto item_at = [&](int it) {
    Item w;
    int bh, qt;
    if (CAUSAL && p.causal_pairs) {
      const int pair = it >> 1;
      bh = pair / pair_half;
      const int pos = pair - bh * pair_half;
      qt = (it & 1) ? pos : p.n_qtiles - 1 - pos;
    } else {
      bh = it / p.n_qtiles;
      qt = it - bh * p.n_qtiles;
      if (CAUSAL && p.causal_reverse) qt = p.n_qtiles - 1 - qt;
    }
    w.b = bh / p.heads;
    w.h = bh - w.b * p.heads;
    w.q0 = qt * NQ * BM;
    int kv_end = CAUSAL ? min(p.seq, w.q0 + NQ * BM) : p.seq;
    if (HAS_MASK && kv_bounds) kv_end = max(1, min(kv_end, s_kv_end[w.b]));
    w.n_kv = (kv_end + BN - 1) / BN;
    w.n_s = kTwoPass ? 2 * w.n_kv : w.n_kv;
    return w;
  };
  auto wait = [&](uint32_t bar, uint32_t parity) {
    return mbar_wait(bar, parity, abort_flag, p.status, B200TK_STATUS_PIPELINE_TIMEOUT,
                     kWaitLimitNs);
  };

  if (warp == L::kProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&p.tm_q);
      tma_prefetch_desc(&p.tm_k);
      tma_prefetch_desc(&p.tm_v);
      int issued_k[KST] = {};
      int issued_v[VST] = {};
      bool ok = true;
      int kc = 0, vc = 0, items_loaded = 0;
      for (int it = first_item(), k = 0; it < total_items && ok; it = next_item(it), ++k) {
        const Item w = item_at(it);
        auto tile_of = [&](int g) { return (kTwoPass && g >= w.n_kv) ? g - w.n_kv : g; };
        // Q smem (and, for fp32, the Q operand in TMEM) is free once every
        // score MMA of the previous item has completed.
        if (k > 0 && !wait(bar_q_empty, (k - 1) & 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(bar_q_full, NQ * L::kQBytes);
#pragma unroll
        for (int t = 0; t < NQ; ++t)
#pragma unroll
          for (int a = 0; a < L::kAtoms; ++a)
            tma_load_4d(sbase + L::kQ + t * L::kQStage + a * BM * 128, &p.tm_q, bar_q_full,
                        a * L::kAtomElems, w.h, w.q0 + t * BM, w.b);
        ++items_loaded;
        // K and V rings are filled independently: the thread polls whichever
        // slot frees first, so a full V ring never holds back K prefetch. V_j
        // is consumed after K of its P@V tile, so V never runs ahead of it.
        int gk = 0, jv = 0;
        uint64_t t_last = globaltimer_ns();
        while ((gk < w.n_s || jv < w.n_kv) && ok) {
          bool progress = false;
          if (gk < w.n_s) {
            const int kg = kc + gk;
            const int s = kg % KST;
            if (kg < KST || mbar_try_wait(bar_k_empty(s), ((kg / KST) - 1) & 1)) {
              mbar_arrive_expect_tx(bar_k_full(s), L::kKVBytes);
              const uint32_t kdst = sbase + L::kK + s * L::kKStage;
              const int j = tile_of(gk);
#pragma unroll
              for (int a = 0; a < L::kAtoms; ++a)
                tma_load_4d(kdst + a * BN * 128, &p.tm_k, bar_k_full(s), a * L::kAtomElems, w.h,
                            j * BN, w.b);
              ++issued_k[s];
              ++gk;
              progress = true;
            }
          }
          const int k_needed = kTwoPass ? w.n_kv + jv : jv;  // score tile preceding PV_jv
          if (jv < w.n_kv && gk > k_needed) {
            const int vg = vc + jv;
            const int sv = vg % VST;
            if (vg < VST || mbar_try_wait(bar_v_empty(sv), ((vg / VST) - 1) & 1)) {
              mbar_arrive_expect_tx(bar_v_full(sv), L::kKVBytes);
              const uint32_t vdst = sbase + L::kV + sv * L::kVStage;
#pragma unroll
              for (int a = 0; a < L::kAtoms; ++a)
                tma_load_4d(vdst + a * BN * 128, &p.tm_v, bar_v_full(sv), a * L::kAtomElems, w.h,
                            jv * BN, w.b);
              ++issued_v[sv];
              ++jv;
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
        kc += w.n_s;
        vc += w.n_kv;
      }
      if (*abort_flag) {
        // drain: every copy this thread started lands before the CTA exits
        if (items_loaded > 0) {
          const uint32_t par = (items_loaded - 1) & 1;
          uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(bar_q_full, par) && globaltimer_ns() - t0 < kWaitLimitNs) {
          }
        }
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
  } else if (warp >= L::kMmaWarp && warp < L::kMmaWarp + L::kMmaWarps) {
    // --------------------------------------------------------- MMA issuers
    // 16-bit: one warp issues the score and P@V MMAs of all query tiles (P
    // aliases the score buffer, so a tile's P@V and its next score MMA keep
    // one issue order; interleaving the tiles in one warp also measured
    // faster than a warp per tile). fp32 (one query tile): warp 0 issues the
    // score MMAs, warp 1 the P@V MMAs; P has TMEM buffers of its own, so the
    // two streams only meet through the softmax barriers.
    //
    // Each warp walks its schedule warp-uniformly (loop control and
    // descriptor arithmetic stay uniform); one elected lane issues every
    // tcgen05.mma and tcgen05.commit (a commit tracks the MMAs of the thread
    // that issues it). Shared-memory descriptors are built once and advanced
    // by adding byte offsets >> 4 to their address field (compile-time
    // constants per K step).
    const bool do_s = !kSplit || warp == L::kMmaWarp;
    const bool leader = elect_one_sync();
    constexpr uint32_t kFmt = ElemTraits<T>::kFmt;
    constexpr uint32_t idesc_qk = make_idesc(kFmt, 0, 0, BN, BM);  // Q K-major, K K-major
    constexpr uint32_t idesc_pv = make_idesc(kFmt, 0, 1, D, BM);   // P (tmem), V MN-major
    const uint64_t q_desc0 = make_sdesc(sbase + L::kQ, 16, 1024, kLayoutSw128);
    const uint64_t k_desc0 = make_sdesc(sbase + L::kK, 16, 1024, kLayoutSw128);
    const uint64_t v_desc0 = make_sdesc(sbase + L::kV, BN * 128, L::kVSbo, L::kVLayout);
    auto wait_all = [&](uint32_t bar, uint32_t parity) {
      return __all_sync(0xFFFFFFFFu, wait(bar, parity));
    };
    bool ok = true;
    int kc = 0, vc = 0;
    for (int it = first_item(), k = 0; it < total_items && ok; it = next_item(it), ++k) {
      const Item w = item_at(it);
      auto tile_of = [&](int g) { return (kTwoPass && g >= w.n_kv) ? g - w.n_kv : g; };
      if (do_s) {
        ok = wait_all(kSplit ? bar_q_ready : bar_q_full, k & 1);
        if (!ok) break;
        tc_fence_after();
      }

      // S_t(g) = Q_t K_g^T into score buffer (kc + g) % NSB of tile t. The K
      // tile is waited for by the first query tile and released after the
      // last; after the item's last score MMA, Q is released.
      auto issue_s = [&](int t, int g) -> bool {
        const int kg = kc + g;
        const int s = kg % KST;
        if (t == 0) {
          if (!wait_all(kSplit ? bar_k_ready(s) : bar_k_full(s), (kg / KST) & 1)) return false;
          tc_fence_after();
        }
        if (leader) {
          const uint32_t d_tmem = tmem + L::t_s(t, kg % NSB);
          const uint64_t qd = q_desc0 + static_cast<uint32_t>((t * L::kQStage) >> 4);
          const uint64_t kd = k_desc0 + static_cast<uint32_t>((s * L::kKStage) >> 4);
          constexpr int kSteps = D / L::kUmmaK;
          constexpr int kPasses = kSplit ? 3 : 1;
#pragma unroll
          for (int pass = 0; pass < kPasses; ++pass) {
            // 3xTF32 order: lo*hi, hi*lo, hi*hi (small terms first). fp32 Q
            // comes from TMEM (hi / lo columns written by the split warps),
            // so the only smem operand of the score MMA is K.
            const uint32_t q_tmem = tmem + (pass == 0 ? L::t_qlo(t) : L::t_qhi(t));
            const int b_off = (kSplit && pass == 1) ? L::kKVBytes : 0;
#pragma unroll
            for (int ks = 0; ks < kSteps; ++ks) {
              constexpr int kAtomStep = 128 / 32;  // K steps per 128-byte swizzle row
              const int atom = ks / kAtomStep;
              const int within = (ks % kAtomStep) * 32;
              const uint64_t bdesc =
                  kd + static_cast<uint32_t>((b_off + atom * BN * 128 + within) >> 4);
              if constexpr (kSplit) {
                mma_ts_tf32(d_tmem, q_tmem + ks * 8, bdesc, idesc_qk,
                            (pass > 0 || ks > 0) ? 1u : 0u);
              } else {
                const uint64_t adesc = qd + static_cast<uint32_t>((atom * BM * 128 + within) >> 4);
                mma_ss_f16(d_tmem, adesc, bdesc, idesc_qk, ks > 0 ? 1u : 0u);
              }
            }
          }
          if (t == NQ - 1) {
            tc_commit(bar_k_empty(s));
            if (g == w.n_s - 1) tc_commit(bar_q_empty);
          }
          tc_commit(bar_s_full(t, kg % NSB));
        }
        __syncwarp();
        return true;
      };

      // O_t += P_t(g) V_j for pass-2 step g (key tile j). The V tile is
      // waited for by the first query tile and released after the last.
      auto issue_pv = [&](int t, int g) -> bool {
        const int j = tile_of(g);
        const int vg = vc + j;
        const int sv = vg % VST;
        if (t == 0 &&
            !wait_all(kSplit ? bar_v_ready(sv) : bar_v_full(sv), (vg / VST) & 1))
          return false;
        // the first P@V of an item overwrites O: the previous item's
        // epilogue must have read it
        if (j == 0 && k > 0 && !wait_all(bar_o_empty(t), (k - 1) & 1)) return false;
        tc_fence_after();
        if (leader) {
          const uint32_t o_tmem = tmem + L::t_o(t);
          const uint64_t vd = v_desc0 + static_cast<uint32_t>((sv * L::kVStage) >> 4);
          constexpr int kSteps = BN / L::kUmmaK;
          constexpr int kPasses = kSplit ? 3 : 1;
#pragma unroll
          for (int pass = 0; pass < kPasses; ++pass) {
            const int pb = (kc + g) % NSB;
            const uint32_t p_tmem = !kSplit    ? tmem + L::t_s(t, pb)
                                    : pass == 0 ? tmem + L::t_plo(t, pb)
                                                : tmem + L::t_phi(t, pb);
            const int v_off = (kSplit && pass == 1) ? L::kKVBytes : 0;
#pragma unroll
            for (int ks = 0; ks < kSteps; ++ks) {
              // V is MN-major: K advances over 128-byte rows; LBO steps
              // across head_dim atoms, SBO across the swizzle's row groups.
              const uint64_t bdesc =
                  vd + static_cast<uint32_t>((v_off + ks * L::kUmmaK * 128) >> 4);
              // 8 columns per K step. 16-bit P: each half-row thread packs
              // its BN/2 keys into the first BN/4 columns of its own half of
              // the score buffer.
              constexpr int kStepsPerHalf = BN / 2 / L::kUmmaK;
              // One-pass 16-bit P is packed contiguously (column c holds keys
              // 2c, 2c + 1).
              const uint32_t a_tmem =
                  (kSplit || L::kOnePass16)
                      ? p_tmem + ks * 8
                      : p_tmem + (ks / kStepsPerHalf) * (BN / 2) + (ks % kStepsPerHalf) * 8;
              const uint32_t acc = (j > 0 || pass > 0 || ks > 0) ? 1u : 0u;
              if constexpr (kSplit)
                mma_ts_tf32(o_tmem, a_tmem, bdesc, idesc_pv, acc);
              else
                mma_ts_f16(o_tmem, a_tmem, bdesc, idesc_pv, acc);
            }
          }
          tc_commit(bar_pv_done(t, L::kPAlias ? (kc + g) % NSB : 0));
          if (t == NQ - 1) tc_commit(bar_v_empty(sv));
        }
        __syncwarp();
        return true;
      };
      // the softmax warps of tile t are done with S_t(g) (and wrote P_t(g))
      auto wait_p = [&](int t, int g) {
        return wait_all(bar_p_full(t, (kc + g) % NSB), ((kc + g) / NSB) & 1);
      };

      if constexpr (kSplit) {
        if (do_s) {
          // A score buffer is reused once the softmax has read it, or (P hi
          // aliased into it) once the P@V that read P hi has completed.
          // Steps count across items, so every phase of the awaited barrier
          // is waited for in order (the first tiles of an item reuse the
          // buffers of the previous item's last tiles).
          for (int g = 0; g < w.n_s && ok; ++g) {
            const int G = kc + g;
            if (G >= NSB) {
              ok = L::kPAlias ? wait_all(bar_pv_done(0, G % NSB), ((G - NSB) / NSB) & 1)
                              : wait_p(0, g - NSB);
            }
            if (ok) ok = issue_s(0, g);
          }
        } else {
          for (int g = 0; g < w.n_s && ok; ++g) {
            ok = wait_p(0, g);
            if (ok) ok = issue_pv(0, g);
          }
        }
      } else {
        for (int g = 0; g < NSB && g < w.n_s && ok; ++g)
          for (int t = 0; t < NQ && ok; ++t) ok = issue_s(t, g);
        for (int g = 0; g < w.n_s && ok; ++g) {
          for (int t = 0; t < NQ && ok; ++t) {
            ok = wait_p(t, g);
            if (ok && (!kTwoPass || g >= w.n_kv)) ok = issue_pv(t, g);
            if (ok && g + NSB < w.n_s) ok = issue_s(t, g + NSB);
          }
        }
      }
      kc += w.n_s;
      vc += w.n_kv;
    }
    // make sure no MMA is still writing TMEM when the CTA tears down
    if (leader) {
      tc_commit(bar_drain);
      uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(bar_drain, 0) && globaltimer_ns() - t0 < kWaitLimitNs) {
      }
    }
    __syncwarp();
  } else if (kSplit && warp >= L::kSplitWarp0) {
    // ------------------------------------------- fp32 hi/lo split workers
    // The tf32 MMA reads the top 19 bits of each fp32 operand and ignores the
    // low 13 mantissa bits (it truncates), so an unmodified fp32 tile is its
    // own "hi" part; only the residual lo = x - trunc_tf32(x) is written.
    const int t = tid - 32 * L::kSplitWarp0;  // 0..127
    auto split_tile = [&](uint32_t off, int bytes) {
      const float4* hi = reinterpret_cast<const float4*>(smem + off);
      float4* lo = reinterpret_cast<float4*>(smem + off + bytes);
      for (int i = t; i < bytes / 16; i += 128) {
        const float4 x = hi[i];
        float4 xl;
        xl.x = x.x - __uint_as_float(__float_as_uint(x.x) & 0xFFFFE000u);
        xl.y = x.y - __uint_as_float(__float_as_uint(x.y) & 0xFFFFE000u);
        xl.z = x.z - __uint_as_float(__float_as_uint(x.z) & 0xFFFFE000u);
        xl.w = x.w - __uint_as_float(__float_as_uint(x.w) & 0xFFFFE000u);
        lo[i] = xl;
      }
      fence_proxy_async_smem();
    };
    bool ok = true;
    int kc = 0, vc = 0;
    for (int it = first_item(), k = 0; it < total_items && ok; it = next_item(it), ++k) {
      const Item w = item_at(it);
      ok = wait(bar_q_full, k & 1);
      // the previous item's score MMAs read the Q operand in TMEM
      if (ok && k > 0) ok = wait(bar_q_empty, (k - 1) & 1);
      if (!ok) break;
      {
        // Q row r (TMEM lane r) -> hi / lo columns of the score MMA's A
        // operand. Warp w may only touch TMEM lanes 32*(w%4)..+31, so each
        // split warp moves the rows of its own lane quadrant.
        tc_fence_after();
        const int quad = warp & 3;
        const int r = quad * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
#pragma unroll 1
        for (int a = 0; a < L::kAtoms; ++a) {
          uint32_t qh[32], ql[32];
          const uint8_t* row = smem + L::kQ + a * BM * 128 + r * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            // 128-byte swizzle: 16-byte chunk c of row r sits at chunk c ^ (r % 8)
            const float4 x = *reinterpret_cast<const float4*>(row + ((c ^ (r & 7)) * 16));
            const float xs[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const uint32_t hb = __float_as_uint(xs[e]) & 0xFFFFE000u;
              qh[c * 4 + e] = hb;
              ql[c * 4 + e] = __float_as_uint(xs[e] - __uint_as_float(hb));
            }
          }
          tmem_st32(tmem + lane_off + L::t_qhi(0) + a * 32, qh);
          tmem_st32(tmem + lane_off + L::t_qlo(0) + a * 32, ql);
        }
        tc_wait_st();
        tc_fence_before();
        mbar_arrive(bar_q_ready);
      }
      // Split in the order the MMA consumes: K_0 .. K_{NSB-1}, then V_j, K_{j+NSB}.
      auto split_k = [&](int j) -> bool {
        const int kg = kc + j;
        const int s = kg % KST;
        if (!wait(bar_k_full(s), (kg / KST) & 1)) return false;
        split_tile(L::kK + s * L::kKStage, L::kKVBytes);
        mbar_arrive(bar_k_ready(s));
        return true;
      };
      for (int j = 0; j < NSB && j < w.n_kv && ok; ++j) ok = split_k(j);
      for (int j = 0; j < w.n_kv && ok; ++j) {
        const int vg = vc + j;
        const int sv = vg % VST;
        ok = wait(bar_v_full(sv), (vg / VST) & 1);
        if (!ok) break;
        split_tile(L::kV + sv * L::kVStage, L::kKVBytes);
        mbar_arrive(bar_v_ready(sv));
        if (j + NSB < w.n_kv) ok = split_k(j + NSB);
      }
      kc += w.n_s;
      vc += w.n_kv;
    }
  } else if (warp < L::kSoftmaxWarps) {
    if constexpr (kTwoPass) {
      // -------------------------------------- softmax, 16-bit (two passes)
      // warp = 8t + 4*half + quad: query tile t, key half `half` of every
      // score tile, TMEM lane quadrant `quad`. Two threads share a row; each
      // keeps the max / sum of its half and the pair combines them once, at
      // the end of pass 1.
      constexpr int HB = BN / 2;  // key columns per thread
      const int t = warp >> 3;
      const int half = (warp >> 2) & 1;
      const int quad = warp & 3;
      const int r = quad * 32 + lane;
      const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
      const int c0 = half * HB;  // first key column of this thread within a tile
      const float scale = p.scale;
      const bool pow2 = p.scale_pow2 != 0;
      bool ok = true;
      int kc = 0, vc = 0;
      for (int it = first_item(), k = 0; it < total_items && ok; it = next_item(it), ++k) {
        const Item w = item_at(it);
        const int row0 = w.q0 + t * BM;
        const int m = row0 + r;
        const int warp_row0 = row0 + quad * 32;
        float m_run = -INFINITY;  // running max of this half, log2 units
        float l_run = 0.f;
        float m_fin = 0.f, inv_l = 0.f;  // row max (log2 units) and 1/row sum

        for (int g = 0; g < w.n_s && ok; ++g) {
          const int sg = kc + g;
          const int buf = sg % NSB;
          const bool pass2 = g >= w.n_kv;
          const int j = pass2 ? g - w.n_kv : g;
          ok = __all_sync(0xFFFFFFFFu, wait(bar_s_full(t, buf), (sg / NSB) & 1));
          if (!ok) break;
          tc_fence_after();
          const int n0 = j * BN + c0;  // first key of this thread's columns
          uint32_t raw[HB];
#pragma unroll
          for (int c = 0; c < HB / 32; ++c)
            tmem_ld32(tmem + lane_off + L::t_s(t, buf) + c0 + c * 32,
                      *reinterpret_cast<uint32_t(*)[32]>(&raw[c * 32]));
          uint32_t kbits[HB / 32];
          if constexpr (HAS_MASK) {
#pragma unroll
            for (int wd = 0; wd < HB / 32; ++wd) {
              const int n = n0 + wd * 32 + lane;
              bool valid = false;
              if (n < p.seq) valid = p.mask[w.b * p.mask_sb + n * p.mask_ss] != 0;
              kbits[wd] = __ballot_sync(0xFFFFFFFFu, valid);
            }
          }
          tc_wait_ld();
          if (!pass2) {
            // pass 1 keeps nothing in TMEM: the score buffer is free as soon
            // as it has been read, so the next score tile overlaps this math.
            tc_fence_before();
            mbar_arrive(bar_p_full(t, buf));
          }
          // A key-padding mask only forces the masked path where it drops a
          // key of this half (the ballot words are warp-uniform: every lane
          // of the warp covers the same keys).
          bool pad = false;
          if constexpr (HAS_MASK) {
#pragma unroll
            for (int wd = 0; wd < HB / 32; ++wd) pad = pad || kbits[wd] != 0xFFFFFFFFu;
          }
          const bool masked = pad || (n0 + HB > p.seq) || (CAUSAL && n0 + HB - 1 > warp_row0);

          // Scores with the reference's dtype boundaries, s = T(T(qk) * scale),
          // as fp32 pairs; masked keys become -inf. `mx` = max over the half.
          float sv[HB];
          float mx;
          if (!masked) {
            uint32_t mx2 = std::is_same_v<T, __half> ? 0xFC00FC00u : 0xFF80FF80u;  // (-inf, -inf)
#pragma unroll
            for (int i = 0; i < HB; i += 2) {
              uint32_t r1 = cvt_pack2<T>(__uint_as_float(raw[i]), __uint_as_float(raw[i + 1]));
              float a, c;
              if (std::is_same_v<T, __nv_bfloat16> && pow2) {
                // T(r1 * 2^k) == r1 * 2^k for bf16: the second rounding is exact
                mx2 = max_pack2<T>(mx2, r1);
                unpack2<T>(r1, a, c);
                mul2(a, c, scale, scale);
              } else {
                unpack2<T>(r1, a, c);
                mul2(a, c, scale, scale);
                const uint32_t r2 = cvt_pack2<T>(a, c);
                mx2 = max_pack2<T>(mx2, r2);
                unpack2<T>(r2, a, c);
              }
              sv[i] = a;
              sv[i + 1] = c;
            }
            float ma, mb;
            unpack2<T>(mx2, ma, mb);
            mx = fmaxf(ma, mb);
            if (std::is_same_v<T, __nv_bfloat16> && pow2) mx *= scale;
          } else {
#pragma unroll
            for (int i = 0; i < HB; i += 2) {
              float a = __uint_as_float(raw[i]), c = __uint_as_float(raw[i + 1]);
              round_pair<T>(a, c);
              a *= scale;
              c *= scale;
              round_pair<T>(a, c);
              sv[i] = a;
              sv[i + 1] = c;
            }
#pragma unroll
            for (int i = 0; i < HB; ++i) {
              const int n = n0 + i;
              bool allowed;
              if constexpr (HAS_MASK)
                allowed = (kbits[i / 32] >> (i % 32)) & 1u;
              else
                allowed = n < p.seq;
              if (CAUSAL) allowed = allowed && (n <= m);
              sv[i] = allowed ? sv[i] : -INFINITY;
            }
            mx = row_max(sv);
          }

          if (!pass2) {
            // pass 1: running max and sum of this half
            const float m_new = fmaxf(m_run, mx * kLog2e);
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            const float alpha = m_run == -INFINITY ? 0.f : ex2_approx(m_run - m_use);
            float part[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int i = 0; i < HB; i += 2) {
              float a = sv[i], c = sv[i + 1];
              fma2(a, c, kLog2e, kLog2e, -m_use, -m_use);
              a = ex2_approx(a);
              c = ex2_approx(c);
              add2(part[i % 8], part[i % 8 + 1], a, c);
            }
            add2(part[0], part[1], part[2], part[3]);
            add2(part[4], part[5], part[6], part[7]);
            add2(part[0], part[1], part[4], part[5]);
            l_run = l_run * alpha + (part[0] + part[1]);
            m_run = m_new;
            if (j == w.n_kv - 1) {
              // combine the two halves of the row (once per item)
              float2* stats = reinterpret_cast<float2*>(smem + L::kStats);
              stats[(t * 2 + half) * BM + r] = make_float2(m_run, l_run);
              mbar_arrive(bar_stats(t));
              ok = __all_sync(0xFFFFFFFFu, wait(bar_stats(t), k & 1));
              if (!ok) break;
              const float2 other = stats[(t * 2 + (half ^ 1)) * BM + r];
              const float mm = fmaxf(m_run, other.x);
              const float mu = mm == -INFINITY ? 0.f : mm;
              const float la = m_run == -INFINITY ? 0.f : l_run * ex2_approx(m_run - mu);
              const float lb = other.x == -INFINITY ? 0.f : other.y * ex2_approx(other.x - mu);
              // same association on both threads of the row: (half 0) + (half 1)
              const float l = half == 0 ? la + lb : lb + la;
              m_fin = mu;
              inv_l = l > 0.f ? 1.f / l : 0.f;
            }
            continue;
          }

          // pass 2: normalised probabilities, rounded to T, into TMEM
          uint32_t pk[HB / 2];
#pragma unroll
          for (int i = 0; i < HB; i += 2) {
            float a = sv[i], c = sv[i + 1];
            fma2(a, c, kLog2e, kLog2e, -m_fin, -m_fin);
            a = ex2_approx(a);
            c = ex2_approx(c);
            mul2(a, c, inv_l, inv_l);
            pk[i / 2] = cvt_pack2<T>(a, c);
          }
          if (j > 0) {
            // Waiting for every P@V phase in order keeps the pv_done parity
            // barrier at most one phase ahead of this wait (and, with one
            // score buffer, PV_{j-1} has read P_{j-1} from these columns).
            if (!__all_sync(0xFFFFFFFFu, wait(bar_pv_done(t, 0), (vc + j - 1) & 1))) {
              ok = false;
              break;
            }
          }
#pragma unroll
          for (int c = 0; c < HB / 64; ++c)
            tmem_st32(tmem + lane_off + L::t_s(t, buf) + c0 + c * 32,
                      *reinterpret_cast<const uint32_t(*)[32]>(&pk[c * 32]));
          if constexpr (HB % 64 != 0)
            tmem_st16(tmem + lane_off + L::t_s(t, buf) + c0 + (HB / 64) * 32,
                      &pk[(HB / 64) * 32]);
          tc_wait_st();
          tc_fence_before();
          mbar_arrive(bar_p_full(t, buf));
        }

        // epilogue: this thread stores head_dim columns [half*D/2, (half+1)*D/2)
        if (ok) ok = __all_sync(0xFFFFFFFFu, wait(bar_pv_done(t, 0), (vc + w.n_kv - 1) & 1));
        if (ok) {
          tc_fence_after();
          constexpr int DH = D / 2;
          T* out_row = reinterpret_cast<T*>(p.out) +
                       ((static_cast<int64_t>(w.b) * p.seq + m) * p.heads + w.h) * D + half * DH;
          const bool row_ok = m < p.seq;
#pragma unroll 1
          for (int c = 0; c < DH / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_off + L::t_o(t) + half * DH + c * 32, o);
            tc_wait_ld();
            if (c == DH / 32 - 1) {
              // O has been read: the next item's first P@V may overwrite it
              tc_fence_before();
              mbar_arrive(bar_o_empty(t));
            }
            if (row_ok) {
              uint4* dst = reinterpret_cast<uint4*>(out_row + c * 32);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                uint4 v;
                v.x = cvt_pack2<T>(__uint_as_float(o[8 * i + 0]), __uint_as_float(o[8 * i + 1]));
                v.y = cvt_pack2<T>(__uint_as_float(o[8 * i + 2]), __uint_as_float(o[8 * i + 3]));
                v.z = cvt_pack2<T>(__uint_as_float(o[8 * i + 4]), __uint_as_float(o[8 * i + 5]));
                v.w = cvt_pack2<T>(__uint_as_float(o[8 * i + 6]), __uint_as_float(o[8 * i + 7]));
                dst[i] = v;
              }
            }
          }
        }
        kc += w.n_s;
        vc += w.n_kv;
      }
    } else if constexpr (L::kOnePass16) {
      // ------------------------------------------ softmax, 16-bit (one pass)
      // warp = 8t + 4 * blk + quad: query tile t, rows 32 * quad + 16 * blk
      // .. + 15 (TMEM lane quadrant `quad`, 16-lane block `blk`). Scores are
      // read with the 16x256b shape (lane i: rows i / 4 and i / 4 + 8 of the
      // block, columns 8g + 2(i % 4) and + 1 of every 8-column group g), so
      // the four threads of a row are lanes 4r .. 4r + 3 and combine row
      // maxima and sums with shuffles. P goes back into the first BN / 2
      // columns of the score buffer as packed T pairs (column c: keys 2c,
      // 2c + 1) with the 16x128b shape (lane i: rows i / 4, i / 4 + 8, column
      // 4g + i % 4 of every 4-column group g): the key pair (8g + 2(i % 4),
      // + 1) a thread holds is exactly that column, so the packed registers
      // are stored in the order they are produced.
      //
      // Online softmax: the running row maximum m_ref (log2 units) moves only
      // when a tile's maximum exceeds it by more than kRescaleThreshold, so
      // P <= 2^8 and O / l are rescaled rarely. The reference's dtype
      // boundaries are kept: scores T(T(qk) * scale), probabilities rounded
      // to T before P@V (unnormalised here; normalised by 1 / l at the end).
      //
      // Ordering: the score MMA of step j is committed after the P@V of step
      // j - 1 of the same query tile (one MMA-issuing thread), so once
      // s_full(t, j) has completed, P_{j-1} has been read (its columns may be
      // overwritten) and O_t is not being written (a rescale may read and
      // write it). The final pv_done wait is at most one phase behind for the
      // same reason.
      constexpr int kRep = BN / 8;  // 16x256b repetitions per score tile
      constexpr int NE = 4 * kRep;  // scores per thread: 2 rows x BN / 4 keys
      constexpr int NP = NE / 2;    // packed pairs per thread
      static_assert(BN == 128, "one-pass 16-bit tiles are 128 keys wide");
      static_assert(NSB == 1, "the ordering argument above assumes one score buffer per tile");
      const int t = warp >> 3;
      const int blk = (warp >> 2) & 1;
      const int quad = warp & 3;
      const int rb = quad * 32 + blk * 16;  // first row of this warp's block
      const int ra = rb + (lane >> 2);      // this thread's rows: ra and ra + 8
      const int cq = 2 * (lane & 3);
      const uint32_t lane_off = static_cast<uint32_t>(rb) << 16;
      auto e_row = [&](int e) { return ra + 8 * ((e >> 1) & 1); };
      auto e_col = [&](int e) { return 8 * (e >> 2) + cq + (e & 1); };
      const float scale = p.scale;
      const bool pow2 = std::is_same_v<T, __nv_bfloat16> && p.scale_pow2 != 0;
      // T(qk) * scale * log2e in one rounding when scale is a power of two
      const float scale_log2e = scale * kLog2e;
      constexpr uint32_t kNegInf2 = std::is_same_v<T, __half> ? 0xFC00FC00u : 0xFF80FF80u;
      bool ok = true;
      int kc = 0, vc = 0;
      for (int it = first_item(), k = 0; it < total_items && ok; it = next_item(it), ++k) {
        const Item w = item_at(it);
        const int row0 = w.q0 + t * BM;
        float m_ref[2] = {-INFINITY, -INFINITY};  // running row maxima, log2 units
        float l_sum[2] = {0.f, 0.f};              // partial sums of this thread's columns

        for (int j = 0; j < w.n_s && ok; ++j) {
          const int sg = kc + j;
          const int buf = sg % NSB;
          ok = __all_sync(0xFFFFFFFFu, wait(bar_s_full(t, buf), (sg / NSB) & 1));
          if (!ok) break;
          tc_fence_after();
          const int n0 = j * BN;
          uint32_t pk[NP];  // T(qk) pairs; pair i belongs to row ra + 8 * (i & 1)
          {
            uint32_t raw[NE];
            tmem_ld16x256b<8>(tmem + lane_off + L::t_s(t, buf), raw);
            tmem_ld16x256b<8>(tmem + lane_off + L::t_s(t, buf) + 64, raw + NE / 2);
            uint32_t kbits[BN / 32];
            if constexpr (HAS_MASK) {
#pragma unroll
              for (int wd = 0; wd < BN / 32; ++wd) {
                const int n = n0 + wd * 32 + lane;
                bool valid = false;
                if (n < p.seq) valid = p.mask[w.b * p.mask_sb + n * p.mask_ss] != 0;
                kbits[wd] = __ballot_sync(0xFFFFFFFFu, valid);
              }
            }
            tc_wait_ld();
            bool pad = false;
            if constexpr (HAS_MASK) {
#pragma unroll
              for (int wd = 0; wd < BN / 32; ++wd) pad = pad || kbits[wd] != 0xFFFFFFFFu;
            }
            const bool masked =
                pad || (n0 + BN > p.seq) || (CAUSAL && n0 + BN - 1 > row0 + rb);
            if (masked) {
#pragma unroll
              for (int e = 0; e < NE; ++e) {
                const int c = e_col(e);
                const int n = n0 + c;
                bool allowed;
                if constexpr (HAS_MASK)
                  allowed = (kbits[c / 32] >> (c % 32)) & 1u;
                else
                  allowed = n < p.seq;
                if (CAUSAL) allowed = allowed && (n <= row0 + e_row(e));
                raw[e] = allowed ? raw[e] : __float_as_uint(-INFINITY);
              }
            }
#pragma unroll
            for (int i = 0; i < NP; ++i)
              pk[i] = cvt_pack2<T>(__uint_as_float(raw[2 * i]), __uint_as_float(raw[2 * i + 1]));
          }
          // Row maxima of T(qk) on the packed pairs (exact); T(T(qk) * scale)
          // is monotone in T(qk), so the row maximum of the scores is T(max *
          // scale).
          uint32_t mx2[2] = {kNegInf2, kNegInf2};
#pragma unroll
          for (int i = 0; i < NP; ++i) mx2[i & 1] = max_pack2<T>(mx2[i & 1], pk[i]);
          float mx[2];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float a, c;
            unpack2<T>(mx2[h], a, c);
            float m = fmaxf(a, c) * scale;
            if (!pow2) {
              float z = m;
              round_pair<T>(m, z);
            }
            m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 1));
            mx[h] = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, 2));
          }
          float m_new[2], alpha[2] = {1.f, 1.f};
#pragma unroll
          for (int h = 0; h < 2; ++h) m_new[h] = fmaxf(m_ref[h], mx[h] * kLog2e);  // -inf stays
          bool rescale = false;
          if (j == 0) {
            m_ref[0] = m_new[0];
            m_ref[1] = m_new[1];
          } else if (__any_sync(0xFFFFFFFFu, m_new[0] > m_ref[0] + kRescaleThreshold ||
                                                 m_new[1] > m_ref[1] + kRescaleThreshold)) {
            // a running max grew by more than 2^8: move every row of this
            // warp to its new max (rows whose max did not grow keep alpha = 1)
            rescale = true;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (m_new[h] > m_ref[h]) {
                alpha[h] = ex2_approx(m_ref[h] - m_new[h]);
                m_ref[h] = m_new[h];
              }
              l_sum[h] *= alpha[h];
            }
          }
          if (rescale) {
            // O_t is quiescent here (see "Ordering" above)
#pragma unroll 1
            for (int c = 0; c < D / 64; ++c) {
              uint32_t o[32];
              const uint32_t addr = tmem + lane_off + L::t_o(t) + c * 64;
              tmem_ld16x256b<8>(addr, o);
              tc_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e)
                o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha[(e >> 1) & 1]);
              tmem_st16x256b<8>(addr, o);
            }
          }
          const float m_use[2] = {m_ref[0] == -INFINITY ? 0.f : m_ref[0],
                                  m_ref[1] == -INFINITY ? 0.f : m_ref[1]};
          float part[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
          for (int i = 0; i < NP; ++i) {
            const int h = i & 1;
            float a, c;
            unpack2<T>(pk[i], a, c);
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
            pk[i] = cvt_pack2<T>(a, c);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) l_sum[h] += part[h][0] + part[h][1];
          tmem_st16x128b_x16(tmem + lane_off + L::t_s(t, buf), pk);
          tc_wait_st();
          tc_fence_before();
          mbar_arrive(bar_p_full(t, buf));
        }

        // epilogue: row sums over the row's four threads (every thread adds
        // the same pairs: the result is bitwise the same on all four), then
        // this thread's columns of O for its two rows, rounded to T
        float out_scale[2] = {0.f, 0.f};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float l = l_sum[h] + __shfl_xor_sync(0xFFFFFFFFu, l_sum[h], 1);
          l = l + __shfl_xor_sync(0xFFFFFFFFu, l, 2);
          out_scale[h] = l > 0.f ? 1.f / l : 0.f;
        }
        if (ok) ok = __all_sync(0xFFFFFFFFu, wait(bar_pv_done(t, 0), (vc + w.n_kv - 1) & 1));
        if (ok) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t o[32];
            tmem_ld16x256b<8>(tmem + lane_off + L::t_o(t) + c * 64, o);
            tc_wait_ld();
            if (c == D / 64 - 1) {
              // O has been read: the next item's first P@V may overwrite it
              tc_fence_before();
              mbar_arrive(bar_o_empty(t));
            }
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const int m = row0 + e_row(e);
              if (m < p.seq) {
                T* dst = reinterpret_cast<T*>(p.out) +
                         ((static_cast<int64_t>(w.b) * p.seq + m) * p.heads + w.h) * D + c * 64 +
                         e_col(e);
                const float sc = out_scale[(e >> 1) & 1];
                *reinterpret_cast<uint32_t*>(dst) =
                    cvt_pack2<T>(__uint_as_float(o[e]) * sc, __uint_as_float(o[e + 1]) * sc);
              }
            }
          }
        }
        kc += w.n_s;
        vc += w.n_kv;
      }
    } else {
      // ------------------------------------------ softmax, fp32 (one pass)
      // warp = 4 * blk + quad: rows 32 * quad + 16 * blk .. + 15 of the query
      // tile (TMEM lane quadrant `quad`, 16-lane block `blk`). Scores, P and
      // O are moved with the 16x256b shape: lane t holds rows t / 4 and
      // t / 4 + 8 of the block and two columns of every 8-column group, so the
      // four threads of a row are lanes 4i .. 4i + 3 of one warp and row
      // maxima, rescale decisions and sums combine with shuffles (no shared
      // memory round trip per tile).
      constexpr int kRep = BN / 8;  // 16x256b repetitions per score tile
      constexpr int NE = 4 * kRep;  // elements per thread: 2 rows x BN / 4 keys
      const int quad = warp & 3;
      const int blk = warp >> 2;
      const int rb = quad * 32 + blk * 16;  // first row of this warp's block
      const int ra = rb + (lane >> 2);      // this thread's rows: ra and ra + 8
      const int cq = 2 * (lane & 3);        // its columns within each 8-column group
      const uint32_t lane_off = static_cast<uint32_t>(rb) << 16;
      // element e of a 16x256b fragment: row ra + 8 * ((e >> 1) & 1), column
      // 8 * (e >> 2) + cq + (e & 1)
      auto e_row = [&](int e) { return ra + 8 * ((e >> 1) & 1); };
      auto e_col = [&](int e) { return 8 * (e >> 2) + cq + (e & 1); };
      const float scale = p.scale;
      bool ok = true;
      int kc = 0, vc = 0;
      // P@V completions seen per pv_done barrier. Step G (counted across
      // items) signals barrier G % PVB; the phases of each barrier are
      // waited for in order and exactly once, so none can be skipped.
      int pvs0 = 0, pvs1 = 0;
      auto pv_seen_through = [&](int G) -> bool {  // P@V of every step <= G done
#pragma unroll
        for (int b = 0; b < PVB; ++b) {
          if (G < b) continue;
          const int last_use = (G - b) / PVB;
          int& seen = b == 0 ? pvs0 : pvs1;
          while (seen <= last_use) {
            if (!__all_sync(0xFFFFFFFFu, wait(bar_pv_done(0, b), seen & 1))) return false;
            ++seen;
          }
        }
        return true;
      };
      for (int it = first_item(), k = 0; it < total_items && ok; it = next_item(it), ++k) {
        const Item w = item_at(it);
        const int row0 = w.q0;
        float m_ref[2] = {-INFINITY, -INFINITY};  // running row maxima, log2 units
        float l_sum[2] = {0.f, 0.f};              // partial sums of this thread's columns

        for (int j = 0; j < w.n_s && ok; ++j) {
          const int sg = kc + j;
          const int buf = sg % NSB;
          ok = __all_sync(0xFFFFFFFFu, wait(bar_s_full(0, buf), (sg / NSB) & 1));
          if (!ok) break;
          tc_fence_after();
          const int n0 = j * BN;
          float sv[NE];
          {
            uint32_t raw[NE];
            tmem_ld16x256b<kRep>(tmem + lane_off + L::t_s(0, buf), raw);
            // key-padding bits of the tile's keys (warp-uniform)
            uint64_t kbits = ~0ull;
            if constexpr (HAS_MASK) {
              kbits = 0;
#pragma unroll
              for (int wd = 0; wd < BN / 32; ++wd) {
                const int n = n0 + wd * 32 + lane;
                bool valid = false;
                if (n < p.seq) valid = p.mask[w.b * p.mask_sb + n * p.mask_ss] != 0;
                kbits |= static_cast<uint64_t>(__ballot_sync(0xFFFFFFFFu, valid)) << (32 * wd);
              }
            }
            tc_wait_ld();
#pragma unroll
            for (int e = 0; e < NE; ++e) sv[e] = __uint_as_float(raw[e]) * scale;
            constexpr uint64_t kTileBits = BN >= 64 ? ~0ull : ((1ull << BN) - 1ull);
            const bool pad = HAS_MASK && (kbits & kTileBits) != kTileBits;
            const bool masked =
                pad || (n0 + BN > p.seq) || (CAUSAL && n0 + BN - 1 > row0 + rb);
            if (masked) {
#pragma unroll
              for (int e = 0; e < NE; ++e) {
                const int n = n0 + e_col(e);
                bool allowed = HAS_MASK ? ((kbits >> e_col(e)) & 1ull) != 0 : n < p.seq;
                if (CAUSAL) allowed = allowed && (n <= row0 + e_row(e));
                sv[e] = allowed ? sv[e] : -INFINITY;
              }
            }
          }
          // row maxima: this thread's columns, then the row's four threads
          float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
          for (int e = 0; e < NE; ++e) mx[(e >> 1) & 1] = fmaxf(mx[(e >> 1) & 1], sv[e]);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 1));
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 2));
          }
          float m_new[2], alpha[2] = {1.f, 1.f};
#pragma unroll
          for (int h = 0; h < 2; ++h) m_new[h] = fmaxf(m_ref[h], mx[h] * kLog2e);  // -inf stays
          bool rescale = false;
          if (j == 0) {
            m_ref[0] = m_new[0];
            m_ref[1] = m_new[1];
          } else if (__any_sync(0xFFFFFFFFu, m_new[0] > m_ref[0] + kRescaleThreshold ||
                                                 m_new[1] > m_ref[1] + kRescaleThreshold)) {
            // a running max grew by more than 2^8: move every row of this
            // warp to its new max (rows whose max did not grow keep alpha = 1)
            rescale = true;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (m_new[h] > m_ref[h]) {
                alpha[h] = ex2_approx(m_ref[h] - m_new[h]);
                m_ref[h] = m_new[h];
              }
              l_sum[h] *= alpha[h];
            }
          }
          const float m_use[2] = {m_ref[0] == -INFINITY ? 0.f : m_ref[0],
                                  m_ref[1] == -INFINITY ? 0.f : m_ref[1]};
          float part[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
          for (int e = 0; e < NE; e += 2) {
            const int h = (e >> 1) & 1;  // elements e, e + 1: same row
            float a = sv[e], c = sv[e + 1];
            fma2(a, c, kLog2e, kLog2e, -m_use[h], -m_use[h]);
            a = ex2_approx(a);
            c = ex2_approx(c);
            sv[e] = a;
            sv[e + 1] = c;
            add2(part[h][(e >> 2) & 1 ? 2 : 0], part[h][(e >> 2) & 1 ? 3 : 1], a, c);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            add2(part[h][0], part[h][1], part[h][2], part[h][3]);
            l_sum[h] += part[h][0] + part[h][1];
          }
          // P_j's buffers were last read by PV_{j-PVB} (kPAlias: P hi into
          // the score columns just read, P lo into P-lo buffer buf; else the
          // single P hi / lo pair); an O rescale must also follow PV_{j-1},
          // the last MMA that wrote O.
          if (!pv_seen_through(sg - PVB) || (rescale && !pv_seen_through(sg - 1))) {
            ok = false;
            break;
          }
          if (rescale) {
            tc_fence_after();
#pragma unroll 1
            for (int c = 0; c < D / 64; ++c) {
              uint32_t o[32];
              const uint32_t addr = tmem + lane_off + L::t_o(0) + c * 64;
              tmem_ld16x256b<8>(addr, o);
              tc_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e)
                o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha[(e >> 1) & 1]);
              tmem_st16x256b<8>(addr, o);
            }
          }
          {
            // P hi keeps the tf32 bits, P lo the exact remainder
            uint32_t ph[NE], pl[NE];
#pragma unroll
            for (int e = 0; e < NE; ++e) {
              const uint32_t hb = __float_as_uint(sv[e]) & 0xFFFFE000u;
              ph[e] = hb;
              pl[e] = __float_as_uint(sv[e] - __uint_as_float(hb));
            }
            tmem_st16x256b<kRep>(tmem + lane_off + L::t_phi(0, buf), ph);
            tmem_st16x256b<kRep>(tmem + lane_off + L::t_plo(0, buf), pl);
          }
          tc_wait_st();
          tc_fence_before();
          mbar_arrive(bar_p_full(0, buf));
        }

        // epilogue: row sums over the row's four threads (every thread adds
        // the same pairs: the result is bitwise the same on all four), then
        // this thread's columns of O for its two rows
        float out_scale[2] = {0.f, 0.f};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float l = l_sum[h] + __shfl_xor_sync(0xFFFFFFFFu, l_sum[h], 1);
          l = l + __shfl_xor_sync(0xFFFFFFFFu, l, 2);
          out_scale[h] = l > 0.f ? 1.f / l : 0.f;
        }
        if (ok) ok = pv_seen_through(vc + w.n_kv - 1);
        if (ok) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t o[32];
            tmem_ld16x256b<8>(tmem + lane_off + L::t_o(0) + c * 64, o);
            tc_wait_ld();
            if (c == D / 64 - 1) {
              // O has been read: the next item's first P@V may overwrite it
              tc_fence_before();
              mbar_arrive(bar_o_empty(0));
            }
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              const int m = row0 + e_row(e);
              if (m < p.seq) {
                float* dst = reinterpret_cast<float*>(p.out) +
                             ((static_cast<int64_t>(w.b) * p.seq + m) * p.heads + w.h) * D +
                             c * 64 + e_col(e);
                const float sc = out_scale[(e >> 1) & 1];
                *reinterpret_cast<float2*>(dst) =
                    make_float2(__uint_as_float(o[e]) * sc, __uint_as_float(o[e + 1]) * sc);
              }
            }
          }
        }
        kc += w.n_s;
        vc += w.n_kv;
      }
    }
  }

  // ------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == L::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, L::kTAlloc);
  }
}

template <typename T, int D, int BN, int KST, int VST, int NQ, bool OP, bool CAUSAL,
          bool HAS_MASK>
cudaError_t launch_tc(const AttnTcParams& prm, int grid, cudaStream_t stream) {
  using L = TcLayout<T, D, BN, KST, VST, NQ, OP>;
  auto kernel = attention_fwd_tc_kernel<T, D, BN, KST, VST, NQ, OP, CAUSAL, HAS_MASK>;
  // at least ~116 KB so that one CTA (and one TMEM allocation) owns each SM
  const int smem = L::kBytes > 118 * 1024 ? L::kBytes : 118 * 1024;
  // The opt-in shared-memory size is set once per device and instantiation,
  // so later launches (including ones inside CUDA-graph capture) make no
  // attribute calls.
  static std::atomic<uint64_t> configured{0};
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  const uint64_t bit = device < 64 ? (uint64_t(1) << device) : 0;
  if (bit == 0 || !(configured.load(std::memory_order_acquire) & bit)) {
    err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return err;
    configured.fetch_or(bit, std::memory_order_acq_rel);
  }
  kernel<<<grid, L::kThreads, smem, stream>>>(prm);
  return cudaGetLastError();
}

// Tile configuration per (dtype, head_dim): query tiles per CTA (NQ), keys
// per tile (BN) and the K / V ring depths, chosen so that shared memory stays
// under the 227 KB opt-in limit (fp32 tiles carry both tf32 hi and lo copies)
// and TMEM under 512 columns.
template <typename T, int D>
struct TcTile {
  static constexpr int kNQ = 2, kBN = 128, kKST = D == 64 ? 3 : 2, kVST = D == 64 ? 3 : 2;
};
template <>
struct TcTile<float, 64> {
  static constexpr int kNQ = 1, kBN = 64, kKST = 3, kVST = 2;
};
template <>
struct TcTile<float, 128> {
  static constexpr int kNQ = 1, kBN = 32, kKST = 2, kVST = 2;
};

template <typename T, int D, bool OP>
cudaError_t launch_variant(const AttnTcParams& prm, int grid, bool causal, bool has_mask,
                           cudaStream_t stream) {
  using C = TcTile<T, D>;
  if (causal)
    return has_mask
               ? launch_tc<T, D, C::kBN, C::kKST, C::kVST, C::kNQ, OP, true, true>(prm, grid, stream)
               : launch_tc<T, D, C::kBN, C::kKST, C::kVST, C::kNQ, OP, true, false>(prm, grid,
                                                                                   stream);
  return has_mask
             ? launch_tc<T, D, C::kBN, C::kKST, C::kVST, C::kNQ, OP, false, true>(prm, grid, stream)
             : launch_tc<T, D, C::kBN, C::kKST, C::kVST, C::kNQ, OP, false, false>(prm, grid,
                                                                                  stream);
}

// Fills the grid-dependent parameters and launches the instantiation for
// (schedule, causal, mask).
template <typename T, int D>
cudaError_t launch_dtype_hd(AttnTcParams prm, int num_sms, bool causal, bool has_mask,
                            cudaStream_t stream) {
  using C = TcTile<T, D>;
  const int rows_per_cta = C::kNQ * BM;
  prm.n_qtiles = (prm.seq + rows_per_cta - 1) / rows_per_cta;
  const int64_t items = static_cast<int64_t>(prm.n_qtiles) * prm.batch * prm.heads;
  // the causal pair numbering (2 * ceil(tiles / 2) per batch-head) plus the
  // persistent loop's look-ahead of 2 * grid must stay inside int
  const int64_t numbered = 2 * static_cast<int64_t>((prm.n_qtiles + 1) / 2) * prm.batch * prm.heads;
  if (items > 0x7FFFFFFF || numbered + 2 * static_cast<int64_t>(num_sms) > 0x7FFFFFFF)
    return cudaErrorInvalidConfiguration;
  // Non-causal items all cost the same: one persistent CTA per SM loops over
  // them (barriers and TMEM set up once, the next item's loads overlap the
  // current item's tail). Causal items differ in length by up to the number
  // of query tiles: with causal_pairs the persistent CTAs take equal-cost
  // (long, short) pairs of tiles, otherwise a CTA per item lets the hardware
  // block scheduler balance them (longest first).
  int64_t work = items;  // schedulable units: items, or pairs of items
  if (causal && prm.causal_pairs)
    work = static_cast<int64_t>((prm.n_qtiles + 1) / 2) * prm.batch * prm.heads;
  const bool persistent = !causal || prm.causal_pairs;
  const int grid = static_cast<int>(persistent ? (work < num_sms ? work : num_sms) : work);
  if constexpr (!std::is_same_v<T, float>) {
    if (prm.one_pass) return launch_variant<T, D, true>(prm, grid, causal, has_mask, stream);
  }
  return launch_variant<T, D, false>(prm, grid, causal, has_mask, stream);
}

// Explicit instantiations live in attention_tc_inst.cu, compiled once per
// (dtype, head_dim) so the six variants build in parallel.
#define B200TK_TC_DECLARE(T, D) \
  extern template cudaError_t launch_dtype_hd<T, D>(AttnTcParams, int, bool, bool, cudaStream_t);
B200TK_TC_DECLARE(__nv_bfloat16, 64)
B200TK_TC_DECLARE(__nv_bfloat16, 128)
B200TK_TC_DECLARE(__half, 64)
B200TK_TC_DECLARE(__half, 128)
B200TK_TC_DECLARE(float, 64)
B200TK_TC_DECLARE(float, 128)
#undef B200TK_TC_DECLARE

}  // namespace tc
}  // namespace b200tk
