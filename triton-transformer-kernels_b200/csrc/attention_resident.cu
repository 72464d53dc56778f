// attention_resident.cu - launcher and instantiations of the row-resident
// 16-bit attention schedule (kernel: attention_resident.cuh).
#include "attention_resident.cuh"

namespace b200tk {
namespace tc {

template <typename T, bool CAUSAL, bool HAS_MASK>
cudaError_t launch_rr(const AttnTcParams& prm, int grid, cudaStream_t stream) {
  auto kernel = attention_resident_kernel<T, CAUSAL, HAS_MASK>;
  // at least ~116 KB so that one CTA (and one TMEM allocation) owns each SM
  const int smem = RrLayout::kBytes > 118 * 1024 ? RrLayout::kBytes : 118 * 1024;
  // set once per device and instantiation: launches inside CUDA-graph
  // capture make no attribute calls
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
  kernel<<<grid, RrLayout::kThreads, smem, stream>>>(prm);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_resident(AttnTcParams prm, int num_sms, bool causal, bool has_mask,
                            cudaStream_t stream) {
  if (prm.seq < 1 || prm.seq > RrLayout::kMaxSeq || !(prm.scale > 0.f))
    return cudaErrorInvalidValue;
  prm.n_qtiles = (prm.seq + BM - 1) / BM;
  const int64_t items = static_cast<int64_t>(prm.n_qtiles) * prm.batch * prm.heads;
  // item indices advance by the grid size: the last step must stay in int
  if (items + static_cast<int64_t>(num_sms) > 0x7FFFFFFF) return cudaErrorInvalidConfiguration;
  const int grid = static_cast<int>(items < num_sms ? items : num_sms);
  if (causal)
    return has_mask ? launch_rr<T, true, true>(prm, grid, stream)
                    : launch_rr<T, true, false>(prm, grid, stream);
  return has_mask ? launch_rr<T, false, true>(prm, grid, stream)
                  : launch_rr<T, false, false>(prm, grid, stream);
}

template cudaError_t launch_resident<__half>(AttnTcParams, int, bool, bool, cudaStream_t);
template cudaError_t launch_resident<__nv_bfloat16>(AttnTcParams, int, bool, bool, cudaStream_t);

}  // namespace tc
}  // namespace b200tk
