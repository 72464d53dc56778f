// attention.h - internal launch interfaces shared by the C ABI (capi.cu) and
// the kernels (attention, residual + LayerNorm, linear + GELU). Not part of
// the public ABI.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/b200tk.h"

namespace b200tk {

// Arguments of the tcgen05 route. Tensor maps are built by the host (capi.cu)
// and passed as opaque 128-byte blobs.
struct AttnTcArgs {
  alignas(64) unsigned char tm_q[128];
  alignas(64) unsigned char tm_k[128];
  alignas(64) unsigned char tm_v[128];
  void* out;
  const uint8_t* mask;
  int64_t mask_sb, mask_ss;
  int64_t batch, seq, heads, head_dim;
  int dtype;
  int causal;
  float scale;
  int schedule;  // B200TK_SCHEDULE_*
  unsigned int* status;
};

// Keys per tile of the tcgen05 kernel for (dtype, head_dim); the query tile
// is always 128 rows.
int attention_tc_block_n(int dtype, int head_dim);
// Sequence length from which B200TK_SCHEDULE_AUTO runs 16-bit inputs on the
// one-pass schedule; shorter sequences keep the two-pass schedule.
constexpr int64_t kOnePassMinSeq = 4096;
// Whether a 16-bit tcgen05 launch takes the one-pass schedule.
bool attention_tc_one_pass(int dtype, int64_t seq, float scale, int schedule);
// Whether the arguments are inside the row-resident schedule's envelope
// (16-bit, head_dim 64, 1 <= seq <= 512, scale > 0), and whether a launch
// with this schedule request takes it.
bool attention_tc_resident_fits(int dtype, int64_t head_dim, int64_t seq, float scale);
bool attention_tc_resident(int dtype, int64_t head_dim, int64_t seq, float scale, int schedule);
// Whether the tcgen05 kernel's work-item numbering fits in int for this
// shape: the causal pair schedule numbers 2 * ceil(tiles / 2) items per
// (batch, head) and looks up to 2 * grid items ahead. Host-only arithmetic.
bool attention_tc_items_fit(int dtype, int head_dim, int64_t batch, int64_t seq, int64_t heads);
cudaError_t launch_attention_tc(const AttnTcArgs& args, cudaStream_t stream);

// Arguments of the CUDA-core route (any supported head_dim, any strides).
struct AttnGenericArgs {
  const void* q;
  const void* k;
  const void* v;
  int64_t qs[3], ks[3], vs[3];  // element strides {batch, seq, head}
  const uint8_t* mask;
  int64_t mask_sb, mask_ss;
  void* out;
  int64_t batch, seq, heads, head_dim;
  int dtype;
  int causal;
  float scale;
};
cudaError_t launch_attention_generic(const AttnGenericArgs& args, cudaStream_t stream);

// Residual + LayerNorm.
struct RlnArgs {
  const void* x;
  const void* update;
  const void* weight;
  const void* bias;
  const uint8_t* mask;
  void* residual_out;
  void* normalized_out;
  int64_t rows, width;
  int dtype;
  float eps;
  uint32_t flags;
  unsigned int* status;  // device status word (the LayerNorm kernels have no waits to bound)
};
cudaError_t launch_residual_layer_norm(const RlnArgs& args, cudaStream_t stream);

// Linear + exact GELU (the FFN input projection) and Linear + residual add
// (out_proj / ffn_out). Tensor maps are built by the host: x [rows, k_in],
// weight [n_out, k_in] and out [rows, n_out], all row-major; residual
// [rows, n_out] row-major and row_mask [rows] (residual form only).
struct LinearGeluArgs {
  alignas(64) unsigned char tm_x[128];
  alignas(64) unsigned char tm_w[128];
  alignas(64) unsigned char tm_out[128];
  const void* bias;
  const void* residual;
  const uint8_t* row_mask;
  void* out;
  int64_t rows, k_in, n_out;
  int dtype;
  unsigned int* status;
};
cudaError_t launch_linear_gelu(const LinearGeluArgs& args, cudaStream_t stream);
cudaError_t launch_linear_residual(const LinearGeluArgs& args, cudaStream_t stream);

// Failure-detection self test (bounded wait on an mbarrier nobody completes).
cudaError_t launch_selftest_wait_timeout(unsigned int* status, uint32_t timeout_us,
                                         cudaStream_t stream);

}  // namespace b200tk
