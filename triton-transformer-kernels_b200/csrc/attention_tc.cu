// attention_tc.cu - host-side launcher of the tcgen05 attention kernels
// (kernels: attention_tc.cuh, attention_resident.cuh): fills the kernel
// parameter block and picks the schedule and the (dtype, head_dim, causal,
// mask) instantiation.
#include <atomic>
#include <cmath>

#include "attention_resident.cuh"
#include "attention_tc.cuh"

namespace b200tk {

int attention_tc_block_n(int dtype, int head_dim) {
  if (dtype == B200TK_DTYPE_FLOAT32) return head_dim == 128 ? tc::TcTile<float, 128>::kBN
                                                            : tc::TcTile<float, 64>::kBN;
  return head_dim == 128 ? tc::TcTile<__half, 128>::kBN : tc::TcTile<__half, 64>::kBN;
}

bool attention_tc_one_pass(int dtype, int64_t seq, float scale, int schedule) {
  // fp32 has one schedule (3xTF32, one pass). The 16-bit one-pass kernel
  // finds row maxima before scaling, which needs scale > 0.
  if (dtype == B200TK_DTYPE_FLOAT32 || !(scale > 0.f)) return false;
  if (schedule == B200TK_SCHEDULE_ONE_PASS) return true;
  if (schedule == B200TK_SCHEDULE_TWO_PASS) return false;
  return seq >= kOnePassMinSeq;
}

bool attention_tc_resident_fits(int dtype, int64_t head_dim, int64_t seq, float scale) {
  return dtype != B200TK_DTYPE_FLOAT32 && head_dim == tc::RrLayout::D && seq >= 1 &&
         seq <= tc::RrLayout::kMaxSeq && scale > 0.f;
}

bool attention_tc_resident(int dtype, int64_t head_dim, int64_t seq, float scale, int schedule) {
  return (schedule == B200TK_SCHEDULE_AUTO || schedule == B200TK_SCHEDULE_RESIDENT) &&
         attention_tc_resident_fits(dtype, head_dim, seq, scale);
}

bool attention_tc_items_fit(int dtype, int head_dim, int64_t batch, int64_t seq, int64_t heads) {
  // The row-resident schedule takes one 128-row query tile per item (the
  // most items of any schedule for its shapes).
  int nq = 1;
  if (dtype != B200TK_DTYPE_FLOAT32 && !(head_dim == tc::RrLayout::D && seq <= tc::RrLayout::kMaxSeq))
    nq = head_dim == 128 ? tc::TcTile<__half, 128>::kNQ : tc::TcTile<__half, 64>::kNQ;
  const int64_t rows_per_item = static_cast<int64_t>(nq) * tc::BM;
  const int64_t tiles = (seq + rows_per_item - 1) / rows_per_item;
  // pair numbering rounds the tile count up to even; the persistent loop's
  // next-item arithmetic adds up to 2 * grid (grid <= SM count < 1024)
  const int64_t numbered = 2 * ((tiles + 1) / 2) * batch * heads;
  return numbered + 2 * 1024 <= 0x7FFFFFFF;
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
  prm.n_qtiles = 0;  // set per tile configuration
  prm.scale = a.scale;
  prm.causal_reverse = 1;
  prm.causal_pairs = 1;
  // T(T(qk) * 2^k) == T(qk) * 2^k for bf16 (fp32 exponent range), so the
  // kernel may skip the second rounding; not for fp16 (subnormals round).
  int exponent = 0;
  prm.scale_pow2 = a.dtype == B200TK_DTYPE_BFLOAT16 && a.scale > 0.f &&
                   std::frexp(a.scale, &exponent) == 0.5f;
  prm.one_pass = attention_tc_one_pass(a.dtype, a.seq, a.scale, a.schedule) ? 1 : 0;
  prm.status = a.status;
  const bool causal = a.causal != 0;
  const bool has_mask = a.mask != nullptr;
  const bool d64 = a.head_dim == 64;
  if (a.head_dim != 64 && a.head_dim != 128) return cudaErrorInvalidValue;
  // SM count per device, queried once (no device queries on later launches)
  static std::atomic<int> sm_count[64] = {};
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) return err;
  if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
  int num_sms = sm_count[device].load(std::memory_order_relaxed);
  if (num_sms == 0) {
    err = cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, device);
    if (err != cudaSuccess) return err;
    sm_count[device].store(num_sms, std::memory_order_relaxed);
  }
  if (attention_tc_resident(a.dtype, a.head_dim, a.seq, a.scale, a.schedule)) {
    return a.dtype == B200TK_DTYPE_BFLOAT16
               ? tc::launch_resident<__nv_bfloat16>(prm, num_sms, causal, has_mask, stream)
               : tc::launch_resident<__half>(prm, num_sms, causal, has_mask, stream);
  }
  switch (a.dtype) {
    case B200TK_DTYPE_BFLOAT16:
      return d64 ? tc::launch_dtype_hd<__nv_bfloat16, 64>(prm, num_sms, causal, has_mask, stream)
                 : tc::launch_dtype_hd<__nv_bfloat16, 128>(prm, num_sms, causal, has_mask, stream);
    case B200TK_DTYPE_FLOAT16:
      return d64 ? tc::launch_dtype_hd<__half, 64>(prm, num_sms, causal, has_mask, stream)
                 : tc::launch_dtype_hd<__half, 128>(prm, num_sms, causal, has_mask, stream);
    case B200TK_DTYPE_FLOAT32:
      return d64 ? tc::launch_dtype_hd<float, 64>(prm, num_sms, causal, has_mask, stream)
                 : tc::launch_dtype_hd<float, 128>(prm, num_sms, causal, has_mask, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace b200tk
