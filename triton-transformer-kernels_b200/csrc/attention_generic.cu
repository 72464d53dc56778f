// attention_generic.cu - CUDA-core attention forward for the shapes the
// tcgen05 kernel does not take: head_dim 8/16/32, and q/k/v views whose base
// addresses or strides are not 16-byte aligned (TMA cannot describe them).
//
// Same algorithm and dtype boundaries as the tensor-core route (and as the
// reference kernel transformer_opt/kernels/attention.py:103-265): fp32 online
// softmax over 16-key steps of 64-key smem tiles (32 for head_dim 128),
// scores rounded to the input dtype before and after the scale, probabilities rounded to the value dtype before P@V,
// all-masked rows produce zeros. fp32 inputs use IEEE fp32 FMAs throughout.
// Each query row is owned by D/DPT consecutive threads (DPT = min(D, 32)
// head-dim elements per thread); a CTA covers 128 threads' worth of rows.

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "attention.h"
#include "ptx_sm100.cuh"

namespace b200tk {
namespace {

constexpr int kThreads = 128;
constexpr int kChunk = 16;  // keys per online-softmax step
constexpr float kLog2e = 1.4426950408889634f;

template <typename T>
__device__ __forceinline__ float to_f32(T v) {
  if constexpr (std::is_same_v<T, float>)
    return v;
  else if constexpr (std::is_same_v<T, __half>)
    return __half2float(v);
  else
    return __bfloat162float(v);
}

template <typename T>
__device__ __forceinline__ T from_f32(float v) {
  if constexpr (std::is_same_v<T, float>)
    return v;
  else if constexpr (std::is_same_v<T, __half>)
    return __float2half_rn(v);
  else
    return __float2bfloat16_rn(v);
}

template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return to_f32<T>(from_f32<T>(v));
}

template <typename T, int D, bool CAUSAL, bool HAS_MASK>
__global__ void __launch_bounds__(kThreads) attention_fwd_generic_kernel(const AttnGenericArgs a) {
  constexpr int DPT = D < 32 ? D : 32;
  constexpr int TPR = D / DPT;
  constexpr int ROWS = kThreads / TPR;
  constexpr int kBN = D <= 64 ? 64 : 32;  // keys per smem tile (32 KB of K+V)
  __shared__ float ks[kBN][D];
  __shared__ float vs[kBN][D];
  __shared__ int kvalid[kBN];

  const int tid = threadIdx.x;
  const int sub = tid % TPR;  // which slice of head_dim this thread owns
  const int rloc = tid / TPR;
  const int64_t S = a.seq;
  const int n_qtiles = static_cast<int>((S + ROWS - 1) / ROWS);
  const int bh = blockIdx.x / n_qtiles;
  const int qt = blockIdx.x - bh * n_qtiles;
  const int b = bh / static_cast<int>(a.heads);
  const int h = bh - b * static_cast<int>(a.heads);
  const int64_t q0 = static_cast<int64_t>(qt) * ROWS;
  const int64_t m = q0 + rloc;
  const bool row_ok = m < S;

  const T* qp = static_cast<const T*>(a.q);
  const T* kp = static_cast<const T*>(a.k);
  const T* vp = static_cast<const T*>(a.v);

  float q[DPT], o[DPT];
#pragma unroll
  for (int i = 0; i < DPT; ++i) {
    q[i] = row_ok ? to_f32<T>(qp[b * a.qs[0] + m * a.qs[1] + h * a.qs[2] + sub * DPT + i]) : 0.f;
    o[i] = 0.f;
  }
  float m_run = -INFINITY, l_run = 0.f;
  const int64_t kv_end = CAUSAL ? (q0 + ROWS < S ? q0 + ROWS : S) : S;

  for (int64_t n0 = 0; n0 < kv_end; n0 += kBN) {
    __syncthreads();
    for (int idx = tid; idx < kBN * D; idx += kThreads) {
      const int r = idx / D, c = idx % D;
      const int64_t n = n0 + r;
      float kv = 0.f, vv = 0.f;
      if (n < S) {
        kv = to_f32<T>(kp[b * a.ks[0] + n * a.ks[1] + h * a.ks[2] + c]);
        vv = to_f32<T>(vp[b * a.vs[0] + n * a.vs[1] + h * a.vs[2] + c]);
      }
      ks[r][c] = kv;
      vs[r][c] = vv;
    }
    for (int r = tid; r < kBN; r += kThreads) {
      const int64_t n = n0 + r;
      int valid = n < S;
      if (HAS_MASK && valid) valid = a.mask[b * a.mask_sb + n * a.mask_ss] != 0;
      kvalid[r] = valid;
    }
    __syncthreads();

    // online softmax over 16-key chunks of the smem tile
#pragma unroll 1
    for (int c0 = 0; c0 < kBN; c0 += kChunk) {
      float s[kChunk];
      float mx = -INFINITY;
#pragma unroll
      for (int rr = 0; rr < kChunk; ++rr) {
        const int r = c0 + rr;
        float dot = 0.f;
#pragma unroll
        for (int i = 0; i < DPT; ++i) dot = fmaf(q[i], ks[r][sub * DPT + i], dot);
#pragma unroll
        for (int off = 1; off < TPR; off <<= 1) dot += __shfl_xor_sync(0xFFFFFFFFu, dot, off);
        float sc;
        if constexpr (std::is_same_v<T, float>)
          sc = dot * a.scale;
        else
          sc = round_to<T>(round_to<T>(dot) * a.scale);
        bool allowed = kvalid[r] != 0;
        if (CAUSAL) allowed = allowed && (n0 + r <= m);
        sc = allowed ? sc : -INFINITY;
        s[rr] = sc;
        mx = fmaxf(mx, sc);
      }
      const float m_new = fmaxf(m_run, mx * kLog2e);
      const float m_use = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = m_run == -INFINITY ? 0.f : ex2_approx(m_run - m_use);
      l_run *= alpha;
#pragma unroll
      for (int i = 0; i < DPT; ++i) o[i] *= alpha;
#pragma unroll
      for (int rr = 0; rr < kChunk; ++rr) {
        const float pv = ex2_approx(fmaf(s[rr], kLog2e, -m_use));
        l_run += pv;
        const float pr = round_to<T>(pv);
#pragma unroll
        for (int i = 0; i < DPT; ++i) o[i] = fmaf(pr, vs[c0 + rr][sub * DPT + i], o[i]);
      }
      m_run = m_new;
    }
  }

  if (row_ok) {
    T* op = static_cast<T*>(a.out) + ((b * S + m) * a.heads + h) * D + sub * DPT;
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
    for (int i = 0; i < DPT; ++i) op[i] = from_f32<T>(l_run > 0.f ? o[i] * inv : 0.f);
  }
}

template <typename T, int D>
cudaError_t launch_d(const AttnGenericArgs& a, cudaStream_t stream) {
  constexpr int DPT = D < 32 ? D : 32;
  constexpr int ROWS = kThreads / (D / DPT);
  const int64_t n_qtiles = (a.seq + ROWS - 1) / ROWS;
  const int64_t grid = n_qtiles * a.batch * a.heads;
  if (grid > 0x7FFFFFFF) return cudaErrorInvalidConfiguration;
  const bool causal = a.causal != 0, has_mask = a.mask != nullptr;
  if (causal && has_mask)
    attention_fwd_generic_kernel<T, D, true, true><<<grid, kThreads, 0, stream>>>(a);
  else if (causal)
    attention_fwd_generic_kernel<T, D, true, false><<<grid, kThreads, 0, stream>>>(a);
  else if (has_mask)
    attention_fwd_generic_kernel<T, D, false, true><<<grid, kThreads, 0, stream>>>(a);
  else
    attention_fwd_generic_kernel<T, D, false, false><<<grid, kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_t(const AttnGenericArgs& a, cudaStream_t stream) {
  switch (a.head_dim) {
    case 8: return launch_d<T, 8>(a, stream);
    case 16: return launch_d<T, 16>(a, stream);
    case 32: return launch_d<T, 32>(a, stream);
    case 64: return launch_d<T, 64>(a, stream);
    case 128: return launch_d<T, 128>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_attention_generic(const AttnGenericArgs& a, cudaStream_t stream) {
  switch (a.dtype) {
    case B200TK_DTYPE_FLOAT32: return launch_t<float>(a, stream);
    case B200TK_DTYPE_FLOAT16: return launch_t<__half>(a, stream);
    case B200TK_DTYPE_BFLOAT16: return launch_t<__nv_bfloat16>(a, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace b200tk
