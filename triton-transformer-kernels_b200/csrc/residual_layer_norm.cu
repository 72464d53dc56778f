// residual_layer_norm.cu - fused residual add + LayerNorm (forward only).
//
// Computes, per row of `width` elements (reference semantics:
// transformer_opt/kernels/residual_layer_norm.py:73-126):
//   r = x + update                       rounded to the I/O dtype
//   r = 0            where the row is invalid and ZERO_INVALID_RESIDUAL
//   mean = sum(r) / width; var = sum((r - mean)^2) / width   (fp32, two-pass)
//   n = (r - mean) * rsqrt(var + eps) * weight + bias
//   n = 0            where the row is invalid and ZERO_INVALID_NORMALIZED
//   n = tf32(n)      with ROUND_TF32 (float32): nearest TF32 value, ties away
//                    from zero, for a tensor-core consumer that truncates
// and writes both r and n. The row lives in registers between the passes, so
// HBM sees exactly one read of x, update and one write of r, n (the roofline
// minimum of 4 * width * sizeof(T) bytes per row).
//
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
