// residual_layer_norm.cu - fused residual add + LayerNorm (forward only).
//
// Computes, per row of `width` elements (reference semantics:
// transformer_opt/kernels/residual_layer_norm.py:73-126):
//   r = x + update                       rounded to the I/O dtype
//   r = 0            where the row is invalid and ZERO_INVALID_RESIDUAL
//   mean, var of r in fp32 (Welford in ATen's order on the Welford path,
//                    two passes over the register-resident row otherwise)
//   n = (r - mean) * rsqrt(var + eps) * weight + bias
//   n = 0            where the row is invalid and ZERO_INVALID_NORMALIZED
//   n = tf32(n)      with ROUND_TF32 (float32): nearest TF32 value, ties away
//                    from zero, for a tensor-core consumer that truncates
// and writes both r and n. The row lives in registers between the passes, so
// HBM sees exactly one read of x, update and one write of r, n (the roofline
// minimum of 4 * width * sizeof(T) bytes per row).
//
// Welford path (16-bit rows of whole 4-element groups up to 4096 wide): the
// statistics in the order of ATen's vectorised LayerNorm kernel, so the
// normalized output equals torch's layer_norm bit for bit (see
// rln_welford_kernel).
// Vector path: each thread holds VPT 16-byte vectors of the row; TPR threads
// share a row (TPR <= 32: a warp segment reduced with shuffles; TPR > 32: whole
// warps reduced through shared memory). Rows that are not a whole number of
// 16-byte vectors, or unaligned pointers, take the scalar path: one CTA per
// row, three passes, the residual re-read from residual_out (L2-resident).

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <type_traits>

#include "attention.h"
#include "ptx_sm100.cuh"

namespace b200tk {
namespace {

// Nearest TF32 value (10 mantissa bits, ties away from zero) as an fp32.
__device__ __forceinline__ float round_tf32(float v) {
  uint32_t u;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(u) : "f"(v));
  return __uint_as_float(u);
}

template <typename T>
__device__ __forceinline__ float ld_f32(const T* p) {
  if constexpr (std::is_same_v<T, float>)
    return *p;
  else if constexpr (std::is_same_v<T, __half>)
    return __half2float(*p);
  else
    return __bfloat162float(*p);
}

template <typename T>
__device__ __forceinline__ T to_t(float v) {
  if constexpr (std::is_same_v<T, float>)
    return v;
  else if constexpr (std::is_same_v<T, __half>)
    return __float2half_rn(v);
  else
    return __float2bfloat16_rn(v);
}

// Round an fp32 value to T and back.
template <typename T>
__device__ __forceinline__ float round_t(float v) {
  const T vt = to_t<T>(v);
  return ld_f32<T>(&vt);
}

template <typename T>
struct VecIO {
  static constexpr int kEPV = 16 / sizeof(T);
  // unpack one 16-byte vector into floats
  __device__ __forceinline__ static void unpack(const uint4& v, float* f) {
    if constexpr (std::is_same_v<T, float>) {
      f[0] = __uint_as_float(v.x);
      f[1] = __uint_as_float(v.y);
      f[2] = __uint_as_float(v.z);
      f[3] = __uint_as_float(v.w);
    } else {
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (std::is_same_v<T, __nv_bfloat16>) {
          f[2 * i] = __uint_as_float(w[i] << 16);
          f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        } else {
          __half2 hh = *reinterpret_cast<const __half2*>(&w[i]);
          float2 ff = __half22float2(hh);
          f[2 * i] = ff.x;
          f[2 * i + 1] = ff.y;
        }
      }
    }
  }
  __device__ __forceinline__ static uint4 pack(const float* f) {
    uint4 v;
    if constexpr (std::is_same_v<T, float>) {
      v.x = __float_as_uint(f[0]);
      v.y = __float_as_uint(f[1]);
      v.z = __float_as_uint(f[2]);
      v.w = __float_as_uint(f[3]);
    } else {
      uint32_t w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if constexpr (std::is_same_v<T, __nv_bfloat16>) {
          __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
          w[i] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
          w[i] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      v.x = w[0];
      v.y = w[1];
      v.z = w[2];
      v.w = w[3];
    }
    return v;
  }
};

// Sum over the TPR threads that share a row. `red` holds one float per warp.
template <int TPR>
__device__ __forceinline__ float row_sum(float v, float* red) {
  if constexpr (TPR <= 32) {
#pragma unroll
    for (int off = TPR / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    return v;
  } else {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, off);
    constexpr int kWarps = TPR / 32;
    const int warp = threadIdx.x >> 5;
    const int row_warp0 = (warp / kWarps) * kWarps;
    __syncthreads();  // previous readers of red are done
    if ((threadIdx.x & 31) == 0) red[warp] = v;
    __syncthreads();
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[row_warp0 + w];
    return s;
  }
}

template <typename T, int VPT, int TPR>
__global__ void __launch_bounds__(TPR >= 256 ? TPR : 256)
    rln_vec_kernel(const RlnArgs a) {
  using IO = VecIO<T>;
  constexpr int EPV = IO::kEPV;
  constexpr int kBlock = TPR >= 256 ? TPR : 256;
  constexpr int kRowsPerCta = kBlock / TPR;
  __shared__ float red[kBlock / 32];

  const int t = threadIdx.x % TPR;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kRowsPerCta + threadIdx.x / TPR;
  const bool row_in = row < a.rows;
  const int64_t n_vec = a.width / EPV;
  const bool has_update = !(a.flags & B200TK_RLN_NO_UPDATE);
  bool valid = true;
  if (a.mask != nullptr && row_in) valid = a.mask[row] != 0;
  const bool zero_res = !valid && (a.flags & B200TK_RLN_ZERO_INVALID_RESIDUAL);
  const bool zero_norm = !valid && (a.flags & B200TK_RLN_ZERO_INVALID_NORMALIZED);
  const bool tf32 = std::is_same_v<T, float> && (a.flags & B200TK_RLN_ROUND_TF32);

  const uint4* xv = reinterpret_cast<const uint4*>(static_cast<const T*>(a.x) + row * a.width);
  const uint4* uv = reinterpret_cast<const uint4*>(static_cast<const T*>(a.update) + row * a.width);
  uint4* rv = reinterpret_cast<uint4*>(static_cast<T*>(a.residual_out) + row * a.width);
  uint4* nv = reinterpret_cast<uint4*>(static_cast<T*>(a.normalized_out) + row * a.width);

  float r[VPT][EPV];
  uint4 xr[VPT], ur[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t vi = static_cast<int64_t>(i) * TPR + t;
    const bool in = row_in && vi < n_vec;
    xr[i] = in ? xv[vi] : make_uint4(0, 0, 0, 0);
    ur[i] = (in && has_update) ? uv[vi] : make_uint4(0, 0, 0, 0);
  }
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t vi = static_cast<int64_t>(i) * TPR + t;
    const bool in = row_in && vi < n_vec;
    float fx[EPV], fu[EPV];
    IO::unpack(xr[i], fx);
    IO::unpack(ur[i], fu);
#pragma unroll
    for (int e = 0; e < EPV; ++e) {
      float v = has_update ? fx[e] + fu[e] : fx[e];
      if constexpr (!std::is_same_v<T, float>) v = round_t<T>(v);
      r[i][e] = (in && !zero_res) ? v : 0.f;
      sum += r[i][e];
    }
    if (in && has_update) rv[vi] = IO::pack(r[i]);
  }
  const float mean = row_sum<TPR>(sum, red) / static_cast<float>(a.width);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t vi = static_cast<int64_t>(i) * TPR + t;
    const bool in = row_in && vi < n_vec;
#pragma unroll
    for (int e = 0; e < EPV; ++e) {
      const float c = in ? r[i][e] - mean : 0.f;
      sq = fmaf(c, c, sq);
    }
  }
  const float var = row_sum<TPR>(sq, red) / static_cast<float>(a.width);
  const float rstd = rsqrtf(var + a.eps);
  const T* wp = static_cast<const T*>(a.weight);
  const T* bp = static_cast<const T*>(a.bias);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int64_t vi = static_cast<int64_t>(i) * TPR + t;
    const bool in = row_in && vi < n_vec;
    if (!in) continue;
    float fw[EPV], fb[EPV], o[EPV];
    IO::unpack(reinterpret_cast<const uint4*>(wp)[vi], fw);
    if (bp != nullptr)
      IO::unpack(reinterpret_cast<const uint4*>(bp)[vi], fb);
#pragma unroll
    for (int e = 0; e < EPV; ++e) {
      const float nrm = (r[i][e] - mean) * rstd * fw[e];
      o[e] = zero_norm ? 0.f : (bp != nullptr ? nrm + fb[e] : nrm);
      if (tf32) o[e] = round_tf32(o[e]);
    }
    nv[vi] = IO::pack(o);
  }
}

// Scalar path: one CTA of 256 threads per row, any width, any alignment.
template <typename T>
__global__ void __launch_bounds__(256) rln_scalar_kernel(const RlnArgs a) {
  __shared__ float red[8];
  const int64_t row = blockIdx.x;
  const int64_t W = a.width;
  const bool has_update = !(a.flags & B200TK_RLN_NO_UPDATE);
  bool valid = true;
  if (a.mask != nullptr) valid = a.mask[row] != 0;
  const bool zero_res = !valid && (a.flags & B200TK_RLN_ZERO_INVALID_RESIDUAL);
  const bool zero_norm = !valid && (a.flags & B200TK_RLN_ZERO_INVALID_NORMALIZED);
  const bool tf32 = std::is_same_v<T, float> && (a.flags & B200TK_RLN_ROUND_TF32);
  const T* x = static_cast<const T*>(a.x) + row * W;
  const T* u = static_cast<const T*>(a.update) + row * W;
  T* ro = static_cast<T*>(a.residual_out) + row * W;
  T* no = static_cast<T*>(a.normalized_out) + row * W;
  auto residual = [&](int64_t c) -> float {
    if (zero_res) return 0.f;
    const float v = has_update ? ld_f32<T>(x + c) + ld_f32<T>(u + c) : ld_f32<T>(x + c);
    return round_t<T>(v);
  };
  float s = 0.f;
  for (int64_t c = threadIdx.x; c < W; c += 256) {
    const float v = residual(c);
    if (has_update) ro[c] = to_t<T>(v);
    s += v;
  }
  const float mean = row_sum<256>(s, red) / static_cast<float>(W);
  float sq = 0.f;
  for (int64_t c = threadIdx.x; c < W; c += 256) {
    const float d = residual(c) - mean;
    sq = fmaf(d, d, sq);
  }
  const float var = row_sum<256>(sq, red) / static_cast<float>(W);
  const float rstd = rsqrtf(var + a.eps);
  const T* wp = static_cast<const T*>(a.weight);
  const T* bp = static_cast<const T*>(a.bias);
  for (int64_t c = threadIdx.x; c < W; c += 256) {
    const float nrm = (residual(c) - mean) * rstd * ld_f32<T>(wp + c);
    const float o = zero_norm ? 0.f : (bp != nullptr ? nrm + ld_f32<T>(bp + c) : nrm);
    no[c] = to_t<T>(tf32 ? round_tf32(o) : o);
  }
}

// ---------------------------------------------------------------------------
// Welford path: the row statistics in the order of ATen's vectorised
// LayerNorm (PyTorch, aten/src/ATen/native/cuda/layer_norm_kernel.cu,
// BSD-licensed), so that `normalized_out` equals torch.nn.functional.layer_norm
// of the residual bit for bit. 16-bit models are sensitive to this: a
// LayerNorm whose fp32 statistics round differently moves ~1 in 10^3 of its
// 16-bit outputs by one unit, and downstream of attention that difference
// survives to the model output (measured on the BASELINE configurations).
//
// Order: 128 threads per row; thread t takes the 4-element groups t, t + 128,
// ... and folds their elements, in order, into a running (mean, m2, count)
// with Welford's update (mean += delta / count, m2 += delta * (v - mean));
// the 32 lanes of a warp then fold in the state of lane + 16, + 8, ..., + 1
// (Chan's pairwise combination); warps 2 and 3 are folded into warps 0 and 1,
// then warp 1 into warp 0. var = m2 / width, rstd = rsqrtf(var + eps),
// n = weight * (rstd * (r - mean)) + bias. Every fused multiply-add that the
// ordering depends on is spelled out with the _rn intrinsics.
struct WelfordState {
  float mean, m2, count;
};

__device__ __forceinline__ WelfordState welford_add(WelfordState s, float v, float inv_count) {
  const float delta = __fsub_rn(v, s.mean);
  const float mean = __fmaf_rn(delta, inv_count, s.mean);
  return {mean, __fmaf_rn(delta, __fsub_rn(v, mean), s.m2), __fadd_rn(s.count, 1.f)};
}

// own (b) folded with other (a)
__device__ __forceinline__ WelfordState welford_combine(WelfordState b, WelfordState a) {
  const float count = __fadd_rn(a.count, b.count);
  if (!(count > 0.f)) return {0.f, 0.f, count};
  const float delta = __fsub_rn(b.mean, a.mean);
  const float coef = __frcp_rn(count);
  const float na = __fmul_rn(a.count, coef), nb = __fmul_rn(b.count, coef);
  const float mean = __fmaf_rn(na, a.mean, __fmul_rn(nb, b.mean));
  const float m2 = __fmaf_rn(__fmul_rn(__fmul_rn(delta, delta), a.count), nb, __fadd_rn(a.m2, b.m2));
  return {mean, m2, count};
}

template <typename T>
struct Quad {  // 4 consecutive elements: 16 bytes (fp32) or 8 bytes (16-bit)
  using Raw = std::conditional_t<std::is_same_v<T, float>, uint4, uint2>;
  __device__ __forceinline__ static void unpack(const Raw& v, float (&f)[4]) {
    if constexpr (std::is_same_v<T, float>) {
      f[0] = __uint_as_float(v.x), f[1] = __uint_as_float(v.y);
      f[2] = __uint_as_float(v.z), f[3] = __uint_as_float(v.w);
    } else {
      const uint32_t w[2] = {v.x, v.y};
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if constexpr (std::is_same_v<T, __nv_bfloat16>) {
          f[2 * i] = __uint_as_float(w[i] << 16);
          f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
        } else {
          const float2 ff = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
          f[2 * i] = ff.x, f[2 * i + 1] = ff.y;
        }
      }
    }
  }
  __device__ __forceinline__ static Raw pack(const float (&f)[4]) {
    Raw v;
    if constexpr (std::is_same_v<T, float>) {
      v.x = __float_as_uint(f[0]), v.y = __float_as_uint(f[1]);
      v.z = __float_as_uint(f[2]), v.w = __float_as_uint(f[3]);
    } else {
      uint32_t w[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        if constexpr (std::is_same_v<T, __nv_bfloat16>) {
          __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
          w[i] = *reinterpret_cast<uint32_t*>(&h);
        } else {
          __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
          w[i] = *reinterpret_cast<uint32_t*>(&h);
        }
      }
      v.x = w[0], v.y = w[1];
    }
    return v;
  }
  // x + u rounded to T, packed. 16-bit types add in pairs in their own type
  // (add.rn.{bf16,f16}x2: the exact sum rounded once). That equals the fp32
  // sum rounded to T: the fp32 sum of two 16-bit values is exact unless their
  // exponents differ by more than 15 (bf16) / 12 (fp16), and then the smaller
  // one is below half a unit of the larger one's 16-bit last place, so both
  // roundings return the larger one.
  __device__ __forceinline__ static Raw add_round(const Raw& x, const Raw& u) {
    if constexpr (std::is_same_v<T, float>) {
      Raw v;
      v.x = __float_as_uint(__uint_as_float(x.x) + __uint_as_float(u.x));
      v.y = __float_as_uint(__uint_as_float(x.y) + __uint_as_float(u.y));
      v.z = __float_as_uint(__uint_as_float(x.z) + __uint_as_float(u.z));
      v.w = __float_as_uint(__uint_as_float(x.w) + __uint_as_float(u.w));
      return v;
    } else {
      using T2 = std::conditional_t<std::is_same_v<T, __half>, __half2, __nv_bfloat162>;
      const uint32_t xw[2] = {x.x, x.y}, uw[2] = {u.x, u.y};
      uint32_t w[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const T2 sum = __hadd2(*reinterpret_cast<const T2*>(&xw[i]), *reinterpret_cast<const T2*>(&uw[i]));
        w[i] = *reinterpret_cast<const uint32_t*>(&sum);
      }
      Raw v;
      v.x = w[0], v.y = w[1];
      return v;
    }
  }
};

// ATen's kernel uses 128 threads per row; here one warp computes TWO rows,
// lane l standing in for those threads l, l + 32, l + 64 and l + 96 ("virtual
// threads" 32w + l, w = 0..3 being ATen's warp) of both rows. Each virtual
// thread keeps its own Welford state over exactly the elements that ATen
// thread folds; the two rows' states sit in the halves of f32x2 registers,
// so every fold and every combination below is one paired instruction for
// both rows (each half rounded exactly like the scalar operation). The
// combination is ATen's binary tree -- per ATen warp w the shuffle-down
// levels N16[w][l] = C(leaf[w][l], leaf[w][l + 16]), N8 = C(N16[l],
// N16[l + 8]), ..., N1[w]; then C(N1[0], N1[2]), C(N1[1], N1[3]) and their
// combination, C(own, other) with "own" the lower index -- with its nodes
// spread over the lanes (2 + 1 + 1 + 1 + 1 + 2 combinations per lane), with
// every node's coefficients computed once per CTA (they depend only on the
// width and the lane). 8 warps (16 rows) per CTA. Each step's loads (one
// 4-element group of every virtual thread of both rows) are issued before the
// previous step is folded. Rows of at most 1024 elements stay in registers
// between the passes; longer ones are re-read (L2-resident), again one step
// ahead.
constexpr int kAtenThreads = 128;  // ATen's threads per row (4 warps)
constexpr int kWelfordWarpsPerCta = 8;

// Two fp32 values per instruction (sm_100 f32x2, the compiler's paired
// intrinsics): each half is rounded exactly as the scalar operation. a - b is
// computed as fma(-1, b, a): -1 * b is exact, so the one rounding is that of
// a - b (signed zeros included: an exact zero difference is +0 either way).
__device__ __forceinline__ float2 add_x2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 sub_x2(float2 a, float2 b) {
  return __ffma2_rn(make_float2(-1.f, -1.f), b, a);
}
__device__ __forceinline__ float2 mul_x2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma_x2(float2 a, float2 b, float2 c) {
  return __ffma2_rn(a, b, c);
}
__device__ __forceinline__ float2 splat(float v) { return make_float2(v, v); }

// ATen's combination of two Welford states, C(own b, other a): n = n_a + n_b,
// coef = 1 / n (correctly rounded), mean = (n_a coef) mean_a + (n_b coef)
// mean_b (one fused multiply-add), m2 = ((delta^2) n_a)(n_b coef) + (m2_a +
// m2_b) with delta = mean_b - mean_a; n = 0 gives an empty state. Every count
// in the tree depends only on the width and the lane, so the coefficients of
// a lane's eight combination sites (n_a coef, n_b coef, n_a) are found once
// per CTA (tree_coefs) and the per-row tree (pair_tree_c) only moves and
// combines means and m2. A site with n = 0 combines two empty states (mean
// and m2 zero), which its zero coefficients reproduce.
constexpr int kTreeSites = 8;
struct PairMoments {  // mean and m2 of one virtual thread, both rows
  float2 mean, m2;
};
struct SiteCoef {
  float na, nb, ca;
};

__device__ __forceinline__ SiteCoef site_coef(float cb, float ca) {
  const float count = __fadd_rn(ca, cb);
  if (!(count > 0.f)) return {0.f, 0.f, 0.f};
  const float coef = __frcp_rn(count);
  return {__fmul_rn(ca, coef), __fmul_rn(cb, coef), ca};
}

__device__ __forceinline__ PairMoments combine_c(const PairMoments& b, const PairMoments& a,
                                                 const SiteCoef& c) {
  const float2 delta = sub_x2(b.mean, a.mean);
  const float2 mean = fma_x2(splat(c.na), a.mean, mul_x2(splat(c.nb), b.mean));
  const float2 m2 =
      fma_x2(mul_x2(mul_x2(delta, delta), splat(c.ca)), splat(c.nb), add_x2(a.m2, b.m2));
  return {mean, m2};
}

// The tree's sites in order: x, y (N16 of ATen warps 0, 2 / 1, 3), N8, N4,
// N2, N1, C(N1[0], N1[2]) / C(N1[1], N1[3]), root; the counts move between
// lanes as the states do in pair_tree_c.
__device__ __forceinline__ void tree_coefs(const float (&leaf)[4], int lane,
                                           SiteCoef (&site)[kTreeSites]) {
  const bool lo = lane < 16;
  const float ra = __shfl_xor_sync(0xFFFFFFFFu, lo ? leaf[1] : leaf[0], 16);
  const float rb = __shfl_xor_sync(0xFFFFFFFFu, lo ? leaf[3] : leaf[2], 16);
  site[0] = lo ? site_coef(leaf[0], ra) : site_coef(ra, leaf[1]);
  site[1] = lo ? site_coef(leaf[2], rb) : site_coef(rb, leaf[3]);
  const float x = __fadd_rn(lo ? ra : leaf[1], lo ? leaf[0] : ra);
  const float y = __fadd_rn(lo ? rb : leaf[3], lo ? leaf[2] : rb);
  const int w = lane >> 3, l = lane & 7;
  const int s1 = l + 16 * (w & 1), s2 = s1 + 8;
  const float x1 = __shfl_sync(0xFFFFFFFFu, x, s1), x2 = __shfl_sync(0xFFFFFFFFu, x, s2);
  const float y1 = __shfl_sync(0xFFFFFFFFu, y, s1), y2 = __shfl_sync(0xFFFFFFFFu, y, s2);
  site[2] = w < 2 ? site_coef(x1, x2) : site_coef(y1, y2);
  float n = w < 2 ? __fadd_rn(x2, x1) : __fadd_rn(y2, y1);
#pragma unroll
  for (int k = 3, off = 4; off > 0; off >>= 1, ++k) {
    const float o = __shfl_down_sync(0xFFFFFFFFu, n, off);
    site[k] = site_coef(n, o);
    n = __fadd_rn(o, n);
  }
  const float o16 = __shfl_down_sync(0xFFFFFFFFu, n, 16);
  site[6] = site_coef(n, o16);
  n = __fadd_rn(o16, n);
  site[7] = site_coef(n, __shfl_down_sync(0xFFFFFFFFu, n, 8));
}

__device__ __forceinline__ PairMoments shfl_m(const PairMoments& v, int src) {
  return {make_float2(__shfl_sync(0xFFFFFFFFu, v.mean.x, src),
                      __shfl_sync(0xFFFFFFFFu, v.mean.y, src)),
          make_float2(__shfl_sync(0xFFFFFFFFu, v.m2.x, src), __shfl_sync(0xFFFFFFFFu, v.m2.y, src))};
}
__device__ __forceinline__ PairMoments shfl_xor_m(const PairMoments& v, int mask) {
  return {make_float2(__shfl_xor_sync(0xFFFFFFFFu, v.mean.x, mask),
                      __shfl_xor_sync(0xFFFFFFFFu, v.mean.y, mask)),
          make_float2(__shfl_xor_sync(0xFFFFFFFFu, v.m2.x, mask),
                      __shfl_xor_sync(0xFFFFFFFFu, v.m2.y, mask))};
}
__device__ __forceinline__ PairMoments shfl_down_m(const PairMoments& v, int off) {
  return {make_float2(__shfl_down_sync(0xFFFFFFFFu, v.mean.x, off),
                      __shfl_down_sync(0xFFFFFFFFu, v.mean.y, off)),
          make_float2(__shfl_down_sync(0xFFFFFFFFu, v.m2.x, off),
                      __shfl_down_sync(0xFFFFFFFFu, v.m2.y, off))};
}

// The root of ATen's combination tree over the 128 virtual-thread states
// leaf[w] (this lane's virtual threads 32w + lane), both rows, with the
// sites' coefficients (coef(k): this lane's site k); valid in lane 0.
// N16: lane j < 16 builds (w = 0, 2; l = j), lane j >= 16 (w = 1, 3;
// l = j - 16), the partner lane j ^ 16 holding the other leaf of each pair.
// N8[w][l] (l < 8) in lane 8w + l: N16[w][l] and N16[w][l + 8] sit in lanes
// l + 16 (w & 1) and l + 8 + 16 (w & 1), in x for w < 2 and y for w >= 2.
// N4, N2, N1 within each group of 8 lanes (lane 8w holds N1[w]); then
// C(N1[0], N1[2]) in lane 0, C(N1[1], N1[3]) in lane 8, and their combination.
template <typename Coef>
__device__ __forceinline__ PairMoments pair_tree_c(const PairMoments (&leaf)[4], int lane,
                                                   const Coef& coef) {
  const bool lo = lane < 16;
  const PairMoments ra = shfl_xor_m(lo ? leaf[1] : leaf[0], 16);
  const PairMoments rb = shfl_xor_m(lo ? leaf[3] : leaf[2], 16);
  const SiteCoef c0 = coef(0), c1 = coef(1);
  const PairMoments x = lo ? combine_c(leaf[0], ra, c0) : combine_c(ra, leaf[1], c0);
  const PairMoments y = lo ? combine_c(leaf[2], rb, c1) : combine_c(rb, leaf[3], c1);
  const int w = lane >> 3, l = lane & 7;
  const int s1 = l + 16 * (w & 1), s2 = s1 + 8;
  const PairMoments x1 = shfl_m(x, s1), x2 = shfl_m(x, s2);
  const PairMoments y1 = shfl_m(y, s1), y2 = shfl_m(y, s2);
  const SiteCoef c2 = coef(2);
  PairMoments n = w < 2 ? combine_c(x1, x2, c2) : combine_c(y1, y2, c2);
#pragma unroll
  for (int k = 3, off = 4; off > 0; off >>= 1, ++k) n = combine_c(n, shfl_down_m(n, off), coef(k));
  n = combine_c(n, shfl_down_m(n, 16), coef(6));
  return combine_c(n, shfl_down_m(n, 8), coef(7));
}

// Per-row form of the tree (CTAs of one pass over 16 rows, where one set of
// coefficients per CTA would not pay for its barrier): Welford states of one
// virtual thread for the warp's two rows, count shared, combined with the
// counts carried along.
struct PairState {
  float2 mean, m2;
  float count;
};

// own (b) folded with other (a), both rows at once; ATen's formula per half.
__device__ __forceinline__ PairState pair_combine(const PairState& b, const PairState& a) {
  const float count = __fadd_rn(a.count, b.count);
  if (!(count > 0.f)) return {splat(0.f), splat(0.f), count};
  const float coef = __frcp_rn(count);
  const float na = __fmul_rn(a.count, coef), nb = __fmul_rn(b.count, coef);
  const float2 delta = sub_x2(b.mean, a.mean);
  const float2 mean = fma_x2(splat(na), a.mean, mul_x2(splat(nb), b.mean));
  const float2 m2 = fma_x2(mul_x2(mul_x2(delta, delta), splat(a.count)), splat(nb),
                           add_x2(a.m2, b.m2));
  return {mean, m2, count};
}

__device__ __forceinline__ PairState shfl_pair(const PairState& v, int src) {
  return {make_float2(__shfl_sync(0xFFFFFFFFu, v.mean.x, src),
                      __shfl_sync(0xFFFFFFFFu, v.mean.y, src)),
          make_float2(__shfl_sync(0xFFFFFFFFu, v.m2.x, src), __shfl_sync(0xFFFFFFFFu, v.m2.y, src)),
          __shfl_sync(0xFFFFFFFFu, v.count, src)};
}
__device__ __forceinline__ PairState shfl_xor_pair(const PairState& v, int mask) {
  return {make_float2(__shfl_xor_sync(0xFFFFFFFFu, v.mean.x, mask),
                      __shfl_xor_sync(0xFFFFFFFFu, v.mean.y, mask)),
          make_float2(__shfl_xor_sync(0xFFFFFFFFu, v.m2.x, mask),
                      __shfl_xor_sync(0xFFFFFFFFu, v.m2.y, mask)),
          __shfl_xor_sync(0xFFFFFFFFu, v.count, mask)};
}
__device__ __forceinline__ PairState shfl_down_pair(const PairState& v, int off) {
  return {make_float2(__shfl_down_sync(0xFFFFFFFFu, v.mean.x, off),
                      __shfl_down_sync(0xFFFFFFFFu, v.mean.y, off)),
          make_float2(__shfl_down_sync(0xFFFFFFFFu, v.m2.x, off),
                      __shfl_down_sync(0xFFFFFFFFu, v.m2.y, off)),
          __shfl_down_sync(0xFFFFFFFFu, v.count, off)};
}

// The root of ATen's combination tree over the 128 virtual-thread states
// leaf[w] (this lane's virtual threads 32w + lane), for both rows; valid in
// lane 0.
__device__ __forceinline__ PairState pair_tree(const PairState (&leaf)[4], int lane) {
  // N16: lane j < 16 builds (w = 0, 2; l = j), lane j >= 16 (w = 1, 3; l = j - 16);
  // the partner lane j ^ 16 holds the other leaf of each pair.
  const bool lo = lane < 16;
  const PairState ra = shfl_xor_pair(lo ? leaf[1] : leaf[0], 16);
  const PairState rb = shfl_xor_pair(lo ? leaf[3] : leaf[2], 16);
  const PairState x = lo ? pair_combine(leaf[0], ra) : pair_combine(ra, leaf[1]);
  const PairState y = lo ? pair_combine(leaf[2], rb) : pair_combine(rb, leaf[3]);
  // N8[w][l] (l < 8) in lane 8w + l: N16[w][l] and N16[w][l + 8] sit in lanes
  // l + 16 (w & 1) and l + 8 + 16 (w & 1), in x for w < 2 and y for w >= 2.
  const int w = lane >> 3, l = lane & 7;
  const int s1 = l + 16 * (w & 1), s2 = s1 + 8;
  const PairState x1 = shfl_pair(x, s1), x2 = shfl_pair(x, s2);
  const PairState y1 = shfl_pair(y, s1), y2 = shfl_pair(y, s2);
  PairState n = w < 2 ? pair_combine(x1, x2) : pair_combine(y1, y2);
  // N4, N2, N1 within each group of 8 lanes (lane 8w holds N1[w])
#pragma unroll
  for (int off = 4; off > 0; off >>= 1) n = pair_combine(n, shfl_down_pair(n, off));
  // C(N1[0], N1[2]) in lane 0, C(N1[1], N1[3]) in lane 8, then C(that, that)
  n = pair_combine(n, shfl_down_pair(n, 16));
  return pair_combine(n, shfl_down_pair(n, 8));
}

// Rows held in registers (at most 1024 elements): persistent CTAs, each warp
// walking row pairs with stride gridDim.x * 8; the tree coefficients and a
// shared-memory copy of weight and bias are made once per CTA (C5's 768-wide
// rows: 0.27 ms against 0.28-0.30 ms for CTAs of one pass over 16 rows).
// Wider rows: CTAs of one pass over 16 rows with the per-row tree, whose load
// latency the resident CTAs cover better and which need no block barrier
// (C3's 4096-wide rows: 0.36 ms against 0.39-0.41 ms persistent).
template <typename T, int QPV>  // QPV: 4-element groups per ATen thread (width <= 512 * QPV)
__global__ void __launch_bounds__(32 * kWelfordWarpsPerCta, 2) rln_welford_kernel(const RlnArgs a) {
  using Q = Quad<T>;
  using Raw = typename Q::Raw;
  constexpr bool kHold = QPV <= 2;  // keep the rows in registers between the passes
  // 16-bit held rows read their weight / bias groups from a copy in shared
  // memory made once per CTA
  constexpr bool kPrefetch = kHold && !std::is_same_v<T, float>;
  constexpr bool kPersist = kHold;
  const int lane = threadIdx.x & 31;
  const int n_quads = static_cast<int>(a.width / 4);
  const bool has_update = !(a.flags & B200TK_RLN_NO_UPDATE);
  const bool tf32 = std::is_same_v<T, float> && (a.flags & B200TK_RLN_ROUND_TF32);
  const float width = static_cast<float>(a.width);

  const int64_t pairs = (a.rows + 1) / 2;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kWelfordWarpsPerCta;
  int64_t pair = static_cast<int64_t>(blockIdx.x) * kWelfordWarpsPerCta + (threadIdx.x >> 5);
  // rows of a pair; a last odd row is computed twice and stored once
  auto row_of = [&](int64_t pr, int i) {
    const int64_t r = 2 * pr + i;
    return r < a.rows ? r : a.rows - 1;
  };
  // each step's groups of every virtual thread of both rows; the next step's
  // loads are in flight while this step is folded
  Raw xv[2][2][4], uv[2][2][4];  // [buffer][row][virtual thread]
  auto load_step = [&](int64_t pr, int k, int buf) {
    const T* xr[2] = {static_cast<const T*>(a.x) + row_of(pr, 0) * a.width,
                      static_cast<const T*>(a.x) + row_of(pr, 1) * a.width};
    const T* ur[2] = {static_cast<const T*>(a.update) + row_of(pr, 0) * a.width,
                      static_cast<const T*>(a.update) + row_of(pr, 1) * a.width};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const int qi = lane + 32 * w + kAtenThreads * k;
      const bool in = qi < n_quads;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        xv[buf][i][w] = in ? reinterpret_cast<const Raw*>(xr[i])[qi] : Raw{};
        uv[buf][i][w] = (in && has_update) ? reinterpret_cast<const Raw*>(ur[i])[qi] : Raw{};
      }
    }
  };
  // element count of this lane's virtual thread w
  const auto leaf_count = [&](int w) {
    int groups = 0;
#pragma unroll
    for (int k = 0; k < QPV; ++k) groups += (lane + 32 * w + kAtenThreads * k < n_quads) ? 1 : 0;
    return static_cast<float>(4 * groups);
  };
  __shared__ float s_coef[kPersist ? 3 : 1][kTreeSites][32];  // n_a / n, n_b / n, n_a
  if (kPersist && threadIdx.x < 32) {
    float leaf[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) leaf[w] = leaf_count(w);
    SiteCoef site[kTreeSites];
    tree_coefs(leaf, lane, site);
#pragma unroll
    for (int k = 0; k < kTreeSites; ++k) {
      s_coef[0][k][lane] = site[k].na;
      s_coef[1][k][lane] = site[k].nb;
      s_coef[2][k][lane] = site[k].ca;
    }
  }
  const Raw* wq = static_cast<const Raw*>(a.weight);
  const Raw* bq = static_cast<const Raw*>(a.bias);
  __shared__ Raw s_w[kPrefetch ? QPV * kAtenThreads : 1], s_b[kPrefetch ? QPV * kAtenThreads : 1];
  if constexpr (kPrefetch) {
    for (int qi = threadIdx.x; qi < n_quads; qi += blockDim.x) {
      s_w[qi] = wq[qi];
      s_b[qi] = bq != nullptr ? bq[qi] : Raw{};
    }
  }
  if constexpr (kPersist) __syncthreads();
  const auto coef = [&](int k) {
    return SiteCoef{s_coef[0][k][lane], s_coef[kPersist ? 1 : 0][k][lane],
                    s_coef[kPersist ? 2 : 0][k][lane]};
  };

  for (; pair < pairs; pair += stride) {
    load_step(pair, 0, 0);
    const bool two = 2 * pair + 1 < a.rows;
    const int64_t rows[2] = {row_of(pair, 0), row_of(pair, 1)};
    bool zero_res[2], zero_norm[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const bool valid = a.mask == nullptr || a.mask[rows[i]] != 0;
      zero_res[i] = !valid && (a.flags & B200TK_RLN_ZERO_INVALID_RESIDUAL);
      zero_norm[i] = !valid && (a.flags & B200TK_RLN_ZERO_INVALID_NORMALIZED);
    }
    const Raw* xq[2];
    Raw* rq[2];
    Raw* nq[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      xq[i] = reinterpret_cast<const Raw*>(static_cast<const T*>(a.x) + rows[i] * a.width);
      rq[i] = reinterpret_cast<Raw*>(static_cast<T*>(a.residual_out) + rows[i] * a.width);
      nq[i] = reinterpret_cast<Raw*>(static_cast<T*>(a.normalized_out) + rows[i] * a.width);
    }

    Raw held[kHold ? QPV * 4 : 1][2];  // the rounded residual groups of both rows, packed
    PairMoments st[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) st[w] = PairMoments{splat(0.f), splat(0.f)};
#pragma unroll
    for (int k = 0; k < QPV; ++k) {
      const int buf = k & 1;
      if (k + 1 < QPV) load_step(pair, k + 1, buf ^ 1);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const int qi = lane + 32 * w + kAtenThreads * k;
        if (qi >= n_quads) continue;
        float r[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          Raw packed;  // the rounded residual (or x itself), packed
          if (has_update) {
            packed = zero_res[i] ? Raw{} : Q::add_round(xv[buf][i][w], uv[buf][i][w]);
            if (i == 0 || two) rq[i][qi] = packed;
          } else {
            packed = zero_res[i] ? Raw{} : xv[buf][i][w];
          }
          Q::unpack(packed, r[i]);
          if constexpr (kHold) held[k * 4 + w][i] = packed;
        }
        // fold: the count before element e of group k is 4k + e, so
        // 1 / (4k + e + 1) folds to a correctly rounded constant
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 v = make_float2(r[0][e], r[1][e]);
          const float2 delta = sub_x2(v, st[w].mean);
          st[w].mean = fma_x2(delta, splat(1.f / static_cast<float>(4 * k + e + 1)), st[w].mean);
          st[w].m2 = fma_x2(delta, sub_x2(v, st[w].mean), st[w].m2);
        }
      }
    }
    PairMoments root;
    if constexpr (kPersist) {
      root = pair_tree_c(st, lane, coef);
    } else {
      PairState leaf[4];
#pragma unroll
      for (int w = 0; w < 4; ++w) leaf[w] = PairState{st[w].mean, st[w].m2, leaf_count(w)};
      const PairState r = pair_tree(leaf, lane);
      root = PairMoments{r.mean, r.m2};
    }
    const float2 mean = make_float2(__shfl_sync(0xFFFFFFFFu, root.mean.x, 0),
                                    __shfl_sync(0xFFFFFFFFu, root.mean.y, 0));
    const float2 m2 = make_float2(__shfl_sync(0xFFFFFFFFu, root.m2.x, 0),
                                  __shfl_sync(0xFFFFFFFFu, root.m2.y, 0));
    const float2 rstd = make_float2(rsqrtf(__fadd_rn(__fdiv_rn(m2.x, width), a.eps)),
                                    rsqrtf(__fadd_rn(__fdiv_rn(m2.y, width), a.eps)));
    // the second pass reads the rounded residual back (residual_out, or x
    // itself for a plain LayerNorm) unless the rows are held in registers
    const Raw* src[2] = {has_update ? static_cast<const Raw*>(rq[0]) : xq[0],
                         has_update ? static_cast<const Raw*>(rq[1]) : xq[1]};
    // rows that are not held: each step's groups (and weight / bias groups)
    // are re-read, the next step's while this one is normalised
    Raw sv[kHold ? 1 : 2][2][4], wsv[kHold ? 1 : 2][4], bsv[kHold ? 1 : 2][4];
    auto reload_step = [&](int k, int buf) {
      if constexpr (!kHold) {
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int qi = lane + 32 * w + kAtenThreads * k;
          const bool in = qi < n_quads;
          sv[buf][0][w] = (in && !zero_res[0]) ? src[0][qi] : Raw{};
          sv[buf][1][w] = (in && !zero_res[1]) ? src[1][qi] : Raw{};
          if constexpr (!kPrefetch) {
            wsv[buf][w] = in ? wq[qi] : Raw{};
            bsv[buf][w] = (in && bq != nullptr) ? bq[qi] : Raw{};
          }
        }
      }
    };
    reload_step(0, 0);
#pragma unroll
    for (int k = 0; k < QPV; ++k) {
      const int buf = kHold ? 0 : (k & 1);
      if (k + 1 < QPV) reload_step(k + 1, buf ^ 1);
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const int qi = lane + 32 * w + kAtenThreads * k;
        if (qi >= n_quads) continue;
        float2 r[4];
        float fw[4], fb[4] = {0.f, 0.f, 0.f, 0.f};
        {
          float r0[4], r1[4];
          if constexpr (kHold) {
            Q::unpack(held[k * 4 + w][0], r0);
            Q::unpack(held[k * 4 + w][1], r1);
          } else {
            Q::unpack(sv[buf][0][w], r0);
            Q::unpack(sv[buf][1][w], r1);
          }
#pragma unroll
          for (int e = 0; e < 4; ++e) r[e] = make_float2(r0[e], r1[e]);
        }
        if constexpr (kPrefetch) {
          Q::unpack(s_w[qi], fw);
          if (bq != nullptr) Q::unpack(s_b[qi], fb);
        } else {
          Q::unpack(wsv[buf][w], fw);
          if (bq != nullptr) Q::unpack(bsv[buf][w], fb);
        }
        float o[2][4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          // n = w * (rstd * (r - mean)) + b, both rows per instruction
          const float2 c = mul_x2(rstd, sub_x2(r[e], mean));
          const float2 n = bq != nullptr ? fma_x2(splat(fw[e]), c, splat(fb[e]))
                                         : mul_x2(splat(fw[e]), c);
          o[0][e] = tf32 ? round_tf32(n.x) : n.x;
          o[1][e] = tf32 ? round_tf32(n.y) : n.y;
        }
        if (zero_norm[0]) o[0][0] = o[0][1] = o[0][2] = o[0][3] = 0.f;
        if (zero_norm[1]) o[1][0] = o[1][1] = o[1][2] = o[1][3] = 0.f;
        nq[0][qi] = Q::pack(o[0]);
        if (two) nq[1][qi] = Q::pack(o[1]);
      }
    }
  }
}

int current_sm_count();

// Resident CTAs per SM of one Welford instantiation (occupancy query, once).
template <typename T, int QPV>
int welford_ctas_per_sm() {
  static std::atomic<int> cached{0};
  int n = cached.load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, rln_welford_kernel<T, QPV>,
                                                      32 * kWelfordWarpsPerCta, 0) != cudaSuccess ||
        n < 1) {
      (void)cudaGetLastError();
      n = 1;
    }
    cached.store(n, std::memory_order_relaxed);
  }
  return n;
}

template <typename T, int QPV>
cudaError_t launch_welford_q(const RlnArgs& a, cudaStream_t stream) {
  const int64_t pairs = (a.rows + 1) / 2;
  int64_t grid = (pairs + kWelfordWarpsPerCta - 1) / kWelfordWarpsPerCta;
  if (QPV <= 2) {  // the persistent form (kPersist)
    const int64_t resident =
        static_cast<int64_t>(current_sm_count()) * welford_ctas_per_sm<T, QPV>();
    if (grid > resident) grid = resident;
  }
  if (grid > 0x7FFFFFFF) return cudaErrorInvalidConfiguration;
  rln_welford_kernel<T, QPV><<<static_cast<unsigned>(grid), 32 * kWelfordWarpsPerCta, 0, stream>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_welford(const RlnArgs& a, cudaStream_t stream) {
  const int64_t quads = a.width / 4;
  const int qpv = static_cast<int>((quads + kAtenThreads - 1) / kAtenThreads);
  switch (qpv) {
    case 1: return launch_welford_q<T, 1>(a, stream);
    case 2: return launch_welford_q<T, 2>(a, stream);
    case 3: return launch_welford_q<T, 3>(a, stream);
    case 4: return launch_welford_q<T, 4>(a, stream);
    case 5: return launch_welford_q<T, 5>(a, stream);
    case 6: return launch_welford_q<T, 6>(a, stream);
    case 7: return launch_welford_q<T, 7>(a, stream);
    case 8: return launch_welford_q<T, 8>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T, int VPT, int TPR>
cudaError_t launch_vec(const RlnArgs& a, cudaStream_t stream) {
  constexpr int kBlock = TPR >= 256 ? TPR : 256;
  constexpr int kRowsPerCta = kBlock / TPR;
  const int64_t grid = (a.rows + kRowsPerCta - 1) / kRowsPerCta;
  if (grid > 0x7FFFFFFF) return cudaErrorInvalidConfiguration;
  rln_vec_kernel<T, VPT, TPR><<<static_cast<unsigned>(grid), kBlock, 0, stream>>>(a);
  return cudaGetLastError();
}

// Resident CTAs per SM of one instantiation (occupancy query, made once; the
// answer depends only on the kernel's resources and the SM architecture).
template <typename T, int VPT, int TPR>
int vec_ctas_per_sm() {
  static std::atomic<int> cached{0};
  int n = cached.load(std::memory_order_relaxed);
  if (n == 0) {
    constexpr int kBlock = TPR >= 256 ? TPR : 256;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, rln_vec_kernel<T, VPT, TPR>, kBlock,
                                                      0) != cudaSuccess ||
        n < 1) {
      (void)cudaGetLastError();
      n = 1;
    }
    cached.store(n, std::memory_order_relaxed);
  }
  return n;
}

template <typename T, int TPR>
int ctas_per_sm(int vpt) {
  switch (vpt) {
    case 1: return vec_ctas_per_sm<T, 1, TPR>();
    case 2: return vec_ctas_per_sm<T, 2, TPR>();
    case 3: return vec_ctas_per_sm<T, 3, TPR>();
    case 4: return vec_ctas_per_sm<T, 4, TPR>();
    case 5: return vec_ctas_per_sm<T, 5, TPR>();
    case 6: return vec_ctas_per_sm<T, 6, TPR>();
    case 7: return vec_ctas_per_sm<T, 7, TPR>();
    default: return vec_ctas_per_sm<T, 8, TPR>();
  }
}

// SM count of the current device, queried once per device.
int current_sm_count() {
  static std::atomic<int> counts[64] = {};
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return 148;
  int n = counts[device].load(std::memory_order_relaxed);
  if (n == 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess || n < 1)
      n = 148;
    counts[device].store(n, std::memory_order_relaxed);
  }
  return n;
}

template <typename T, int TPR>
cudaError_t launch_vpt(const RlnArgs& a, int vpt, cudaStream_t stream) {
  switch (vpt) {
    case 1: return launch_vec<T, 1, TPR>(a, stream);
    case 2: return launch_vec<T, 2, TPR>(a, stream);
    case 3: return launch_vec<T, 3, TPR>(a, stream);
    case 4: return launch_vec<T, 4, TPR>(a, stream);
    case 5: return launch_vec<T, 5, TPR>(a, stream);
    case 6: return launch_vec<T, 6, TPR>(a, stream);
    case 7: return launch_vec<T, 7, TPR>(a, stream);
    case 8: return launch_vec<T, 8, TPR>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_typed(const RlnArgs& a, cudaStream_t stream) {
  constexpr int EPV = VecIO<T>::kEPV;
  auto aligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  // 16-bit rows of whole 4-element groups, up to 4096 wide, take the Welford
  // path (statistics in ATen's order, so the 16-bit output equals torch's
  // bit for bit); fp32, wider or unaligned rows the paths below (fp32 output
  // within ~1e-6 of torch's, where one unit of a 16-bit output is 2^-8 or
  // 2^-11 relative).
  const bool welford_ok = !std::is_same_v<T, float> && a.width % 4 == 0 &&
                          a.width <= 4 * kAtenThreads * 8 &&
                          aligned(a.x) && aligned(a.weight) && aligned(a.normalized_out) &&
                          (a.bias == nullptr || aligned(a.bias)) &&
                          ((a.flags & B200TK_RLN_NO_UPDATE) ||
                           (aligned(a.update) && aligned(a.residual_out)));
  if (welford_ok) return launch_welford<T>(a, stream);
  const bool vec_ok = a.width % EPV == 0 && aligned(a.x) && aligned(a.weight) &&
                      aligned(a.normalized_out) && (a.bias == nullptr || aligned(a.bias)) &&
                      ((a.flags & B200TK_RLN_NO_UPDATE) ||
                       (aligned(a.update) && aligned(a.residual_out)));
  if (vec_ok) {
    const int64_t n_vec = a.width / EPV;
    // Threads per row: the smallest group that keeps <= 8 vectors per thread,
    // unless a wider group (never wider than the row's vectors) fills the
    // last wave of CTAs clearly better. With few rows the number of waves is
    // small and a mostly empty last wave dominates (fp32 d=4096, 2048 rows:
    // 2.3 waves of 128-thread rows at 3 CTAs per SM).
    const int tprs[4] = {32, 128, 256, 512};
    const int sms = current_sm_count();
    int best_tpr = 0, best_vpt = 0;
    double best_fill = -1.0;
    for (int tpr : tprs) {
      const int64_t vpt = (n_vec + tpr - 1) / tpr;
      if (vpt > 8) continue;
      if (best_tpr != 0 && tpr > n_vec) break;
      const int block = tpr >= 256 ? tpr : 256;
      const int64_t grid = (a.rows + block / tpr - 1) / (block / tpr);
      int per_sm = 1;
      switch (tpr) {
        case 32: per_sm = ctas_per_sm<T, 32>(static_cast<int>(vpt)); break;
        case 128: per_sm = ctas_per_sm<T, 128>(static_cast<int>(vpt)); break;
        case 256: per_sm = ctas_per_sm<T, 256>(static_cast<int>(vpt)); break;
        default: per_sm = ctas_per_sm<T, 512>(static_cast<int>(vpt)); break;
      }
      const double waves = static_cast<double>(grid) / (static_cast<double>(per_sm) * sms);
      const double fill = waves / static_cast<double>(static_cast<int64_t>(waves) +
                                                      (waves > static_cast<int64_t>(waves)));
      if (best_tpr == 0 || fill > best_fill + 0.05) {
        best_tpr = tpr;
        best_vpt = static_cast<int>(vpt);
        best_fill = fill;
      }
    }
    switch (best_tpr) {
      case 32: return launch_vpt<T, 32>(a, best_vpt, stream);
      case 128: return launch_vpt<T, 128>(a, best_vpt, stream);
      case 256: return launch_vpt<T, 256>(a, best_vpt, stream);
      case 512: return launch_vpt<T, 512>(a, best_vpt, stream);
      default: break;
    }
  }
  if (a.rows > 0x7FFFFFFF) return cudaErrorInvalidConfiguration;
  rln_scalar_kernel<T><<<static_cast<unsigned>(a.rows), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_residual_layer_norm(const RlnArgs& a, cudaStream_t stream) {
  if (a.rows == 0) return cudaSuccess;
  switch (a.dtype) {
    case B200TK_DTYPE_FLOAT32: return launch_typed<float>(a, stream);
    case B200TK_DTYPE_FLOAT16: return launch_typed<__half>(a, stream);
    case B200TK_DTYPE_BFLOAT16: return launch_typed<__nv_bfloat16>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace b200tk
