// attention_tc.cu - host-side launcher of the tcgen05 attention kernels
// (kernel: attention_tc.cuh): fills the kernel parameter block and picks the
// (dtype, head_dim, causal, mask) instantiation.
#include "attention_tc.cuh"

namespace b200tk {

int attention_tc_block_n(int dtype, int head_dim) {
  if (dtype == B200TK_DTYPE_FLOAT32) return head_dim == 128 ? tc::TcTile<float, 128>::kBN
                                                            : tc::TcTile<float, 64>::kBN;
  return head_dim == 128 ? tc::TcTile<__half, 128>::kBN : tc::TcTile<__half, 64>::kBN;
}

cudaError_t launch_attention_tc(const AttnTcArgs& a, cudaStream_t stream) {
  tc::AttnTcParams prm;
  prm.tm_q = *reinterpret_cast<const CUtensorMap*>(a.tm_q);
  prm.tm_k = *reinterpret_cast<const CUtensorMap*>(a.tm_k);
  prm.tm_v = *reinterpret_cast<const CUtensorMap*>(a.tm_v);
  prm.out = a.out;
  prm.mask = a.mask;
  prm.mask_sb = a.mask_sb;
  prm.mask_ss = a.mask_ss;
  prm.batch = static_cast<int>(a.batch);
  prm.seq = static_cast<int>(a.seq);
  prm.heads = static_cast<int>(a.heads);
  prm.n_qtiles = static_cast<int>((a.seq + tc::BM - 1) / tc::BM);
  prm.scale = a.scale;
  prm.causal_reverse = 1;
  prm.status = a.status;
  const int64_t grid64 = static_cast<int64_t>(prm.n_qtiles) * a.batch * a.heads;
  if (grid64 > 0x7FFFFFFF) return cudaErrorInvalidConfiguration;
  const int grid = static_cast<int>(grid64);
  const bool causal = a.causal != 0;
  const bool has_mask = a.mask != nullptr;
  const bool d64 = a.head_dim == 64;
  if (a.head_dim != 64 && a.head_dim != 128) return cudaErrorInvalidValue;
  switch (a.dtype) {
    case B200TK_DTYPE_BFLOAT16:
      return d64 ? tc::launch_dtype_hd<__nv_bfloat16, 64>(prm, grid, causal, has_mask, stream)
                 : tc::launch_dtype_hd<__nv_bfloat16, 128>(prm, grid, causal, has_mask, stream);
    case B200TK_DTYPE_FLOAT16:
      return d64 ? tc::launch_dtype_hd<__half, 64>(prm, grid, causal, has_mask, stream)
                 : tc::launch_dtype_hd<__half, 128>(prm, grid, causal, has_mask, stream);
    case B200TK_DTYPE_FLOAT32:
      return d64 ? tc::launch_dtype_hd<float, 64>(prm, grid, causal, has_mask, stream)
                 : tc::launch_dtype_hd<float, 128>(prm, grid, causal, has_mask, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace b200tk
