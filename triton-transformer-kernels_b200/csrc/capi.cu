// capi.cu - the extern "C" boundary of libb200tk.so (declared in
// include/b200tk.h): argument validation, route selection, TMA tensor-map
// construction, the per-device status word, and the self-test kernel.

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "attention.h"
#include "ptx_sm100.cuh"

namespace b200tk {
namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(B200TK_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

// Per-device status word. Kernels receive its device address as a pointer.
__device__ unsigned int g_device_status;

constexpr int kMaxDevices = 64;
std::mutex g_mu;
unsigned int* g_status_addr[kMaxDevices] = {};

int status_address(unsigned int** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(B200TK_ERR_UNSUPPORTED, "device index too large");
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_status_addr[dev] == nullptr) {
    void* p = nullptr;
    err = cudaGetSymbolAddress(&p, g_device_status);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(status)");
    g_status_addr[dev] = static_cast<unsigned int*>(p);
  }
  *out = g_status_addr[dev];
  return B200TK_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int get_encoder(PFN_cuTensorMapEncodeTiled_v12000* fn) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_encode == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (err != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      return fail(B200TK_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  *fn = g_encode;
  return B200TK_OK;
}

int elem_size(int dtype) {
  switch (dtype) {
    case B200TK_DTYPE_FLOAT32: return 4;
    case B200TK_DTYPE_FLOAT16:
    case B200TK_DTYPE_BFLOAT16: return 2;
    default: return 0;
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// TMA can describe a [batch, seq, heads, head_dim] view when its base is
// 16-byte aligned and every stride of a dimension longer than 1 is a positive
// multiple of 16 bytes below 2^40.
bool tma_describable(const void* ptr, const int64_t* st, int64_t batch, int64_t seq,
                     int64_t heads, int es) {
  if (!aligned16(ptr)) return false;
  const int64_t ext[3] = {batch, seq, heads};
  for (int i = 0; i < 3; ++i) {
    if (ext[i] <= 1) continue;
    const int64_t bytes = st[i] * es;
    if (st[i] <= 0 || bytes % 16 != 0 || bytes >= (int64_t(1) << 40)) return false;
  }
  return true;
}

int encode_map(void* out, const void* ptr, const int64_t* st, int64_t batch, int64_t seq,
               int64_t heads, int64_t head_dim, int dtype, int box_rows,
               CUtensorMapSwizzle swizzle) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  int rc = get_encoder(&enc);
  if (rc != B200TK_OK) return rc;
  const int es = elem_size(dtype);
  auto stride_or_default = [&](int64_t ext, int64_t s) -> cuuint64_t {
    if (ext <= 1) return 16;  // never stepped over
    return static_cast<cuuint64_t>(s * es);
  };
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(seq), static_cast<cuuint64_t>(batch)};
  cuuint64_t strides[3] = {stride_or_default(heads, st[2]), stride_or_default(seq, st[1]),
                           stride_or_default(batch, st[0])};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / es), 1, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMapDataType dt = dtype == B200TK_DTYPE_FLOAT32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : dtype == B200TK_DTYPE_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = enc(reinterpret_cast<CUtensorMap*>(out), dt, 4, const_cast<void*>(ptr), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    std::snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
    return fail(B200TK_ERR_CUDA, buf);
  }
  return B200TK_OK;
}

// Row-major [rows, cols] matrix as a 2D tensor map: box {128 bytes of
// columns, box_rows rows}, 128-byte swizzle. Out-of-range rows and columns
// read as zero.
int encode_matrix_map(void* out, const void* ptr, int64_t rows, int64_t cols, int dtype,
                      int box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  int rc = get_encoder(&enc);
  if (rc != B200TK_OK) return rc;
  const int es = elem_size(dtype);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * es)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / es), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapDataType dt = dtype == B200TK_DTYPE_FLOAT32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                           : dtype == B200TK_DTYPE_FLOAT16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                           : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = enc(reinterpret_cast<CUtensorMap*>(out), dt, 2, const_cast<void*>(ptr), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    std::snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
    return fail(B200TK_ERR_CUDA, buf);
  }
  return B200TK_OK;
}

int validate_attention(const void* q, const int64_t* qs, const void* k, const int64_t* ks,
                       const void* v, const int64_t* vs, int dtype, int64_t batch, int64_t seq,
                       int64_t heads, int64_t head_dim) {
  if (elem_size(dtype) == 0) return fail(B200TK_ERR_INVALID_ARGUMENT, "unknown dtype code");
  if (batch < 0 || seq <= 0 || heads <= 0 || head_dim <= 0)
    return fail(B200TK_ERR_INVALID_ARGUMENT,
                "sequence length, head count, and head dimension must be positive");
  if (head_dim != 8 && head_dim != 16 && head_dim != 32 && head_dim != 64 && head_dim != 128)
    return fail(B200TK_ERR_UNSUPPORTED, "head_dim must be one of 8, 16, 32, 64, 128");
  if (seq > (int64_t(1) << 30) || heads > (int64_t(1) << 20) || batch > (int64_t(1) << 30))
    return fail(B200TK_ERR_UNSUPPORTED, "tensor extent exceeds the kernel's index range");
  if (qs == nullptr || ks == nullptr || vs == nullptr)
    return fail(B200TK_ERR_INVALID_ARGUMENT, "stride arrays must not be NULL");
  if (batch > 0 && (q == nullptr || k == nullptr || v == nullptr))
    return fail(B200TK_ERR_INVALID_ARGUMENT, "q, k and v must not be NULL");
  return B200TK_OK;
}

int route_for(const void* q, const int64_t* qs, const void* k, const int64_t* ks, const void* v,
              const int64_t* vs, int dtype, int64_t batch, int64_t seq, int64_t heads,
              int64_t head_dim) {
  const int es = elem_size(dtype);
  if ((head_dim == 64 || head_dim == 128) && tma_describable(q, qs, batch, seq, heads, es) &&
      tma_describable(k, ks, batch, seq, heads, es) && tma_describable(v, vs, batch, seq, heads, es))
    return B200TK_ROUTE_TCGEN05;
  return B200TK_ROUTE_GENERIC;
}

// The chosen kernel numbers its work items with int: reject shapes whose
// item count would overflow (the launch would otherwise do no work and
// report success). Rows per CTA of the generic kernel: 128 / (D / min(D, 32)).
int check_item_range(int route, int dtype, int64_t batch, int64_t seq, int64_t heads,
                     int64_t head_dim) {
  bool fits;
  if (route == B200TK_ROUTE_TCGEN05) {
    fits = attention_tc_items_fit(dtype, static_cast<int>(head_dim), batch, seq, heads);
  } else {
    const int64_t rows = 128 / (head_dim / (head_dim < 32 ? head_dim : 32));
    fits = ((seq + rows - 1) / rows) * batch * heads <= 0x7FFFFFFF;
  }
  if (!fits)
    return fail(B200TK_ERR_UNSUPPORTED,
                "batch x heads x query tiles exceeds the kernel's work-item range");
  return B200TK_OK;
}

__global__ void selftest_wait_kernel(unsigned int* status, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_mbarrier_init();
  }
  __syncthreads();
  // Nothing ever arrives on `bar`: the wait must give up by itself.
  if (threadIdx.x == 0)
    mbar_wait(smem_u32(&bar), 0, &abort_flag, status, B200TK_STATUS_SELFTEST_TIMEOUT, limit_ns);
  __syncthreads();
}

}  // namespace

cudaError_t launch_selftest_wait_timeout(unsigned int* status, uint32_t timeout_us,
                                         cudaStream_t stream) {
  selftest_wait_kernel<<<1, 32, 0, stream>>>(status, uint64_t(timeout_us) * 1000ull);
  return cudaGetLastError();
}

}  // namespace b200tk

using namespace b200tk;

extern "C" {

int b200tk_abi_version(void) { return B200TK_ABI_VERSION; }

const char* b200tk_last_error(void) { return g_last_error.c_str(); }

int b200tk_attention_route(const void* q, const int64_t* q_strides, const void* k,
                           const int64_t* k_strides, const void* v, const int64_t* v_strides,
                           int dtype, int64_t batch, int64_t seq_len, int64_t heads,
                           int64_t head_dim) {
  int rc = validate_attention(q, q_strides, k, k_strides, v, v_strides, dtype, batch, seq_len,
                              heads, head_dim);
  if (rc != B200TK_OK) return rc;
  const int route = route_for(q, q_strides, k, k_strides, v, v_strides, dtype, batch, seq_len,
                              heads, head_dim);
  rc = check_item_range(route, dtype, batch, seq_len, heads, head_dim);
  return rc != B200TK_OK ? rc : route;
}

int b200tk_attention_fwd(const void* q, const int64_t* q_strides, const void* k,
                         const int64_t* k_strides, const void* v, const int64_t* v_strides,
                         const uint8_t* valid_token_mask, const int64_t* mask_strides, void* out,
                         int dtype, int64_t batch, int64_t seq_len, int64_t heads,
                         int64_t head_dim, int causal, float scale, void* stream) {
  return b200tk_attention_fwd_scheduled(q, q_strides, k, k_strides, v, v_strides,
                                        valid_token_mask, mask_strides, out, dtype, batch,
                                        seq_len, heads, head_dim, causal, scale,
                                        B200TK_SCHEDULE_AUTO, stream);
}

int b200tk_attention_fwd_scheduled(const void* q, const int64_t* q_strides, const void* k,
                                   const int64_t* k_strides, const void* v,
                                   const int64_t* v_strides, const uint8_t* valid_token_mask,
                                   const int64_t* mask_strides, void* out, int dtype,
                                   int64_t batch, int64_t seq_len, int64_t heads,
                                   int64_t head_dim, int causal, float scale, int schedule,
                                   void* stream) {
  if (schedule != B200TK_SCHEDULE_AUTO && schedule != B200TK_SCHEDULE_TWO_PASS &&
      schedule != B200TK_SCHEDULE_ONE_PASS && schedule != B200TK_SCHEDULE_RESIDENT)
    return fail(B200TK_ERR_INVALID_ARGUMENT, "unknown attention schedule");
  int rc = validate_attention(q, q_strides, k, k_strides, v, v_strides, dtype, batch, seq_len,
                              heads, head_dim);
  if (rc != B200TK_OK) return rc;
  if (batch == 0) return B200TK_OK;
  if (out == nullptr) return fail(B200TK_ERR_INVALID_ARGUMENT, "out must not be NULL");
  if (valid_token_mask != nullptr && mask_strides == nullptr)
    return fail(B200TK_ERR_INVALID_ARGUMENT, "mask_strides must be given with a mask");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int route = route_for(q, q_strides, k, k_strides, v, v_strides, dtype, batch, seq_len, heads,
                        head_dim);
  if (route == B200TK_ROUTE_TCGEN05 && !aligned16(out)) route = B200TK_ROUTE_GENERIC;
  rc = check_item_range(route, dtype, batch, seq_len, heads, head_dim);
  if (rc != B200TK_OK) return rc;
  if (schedule == B200TK_SCHEDULE_RESIDENT &&
      (route != B200TK_ROUTE_TCGEN05 ||
       !attention_tc_resident_fits(dtype, head_dim, seq_len, scale)))
    return fail(B200TK_ERR_UNSUPPORTED,
                "the resident schedule needs float16/bfloat16, head_dim 64, seq_len <= 512, "
                "scale > 0 and tensor-core-route strides");
  if (route == B200TK_ROUTE_TCGEN05) {
    AttnTcArgs a;
    std::memset(&a, 0, sizeof(a));
    const int bn = attention_tc_block_n(dtype, static_cast<int>(head_dim));
    // Q and K feed the MMA K-major (128-byte swizzle). V feeds it MN-major:
    // 16-bit V uses the same swizzle, fp32 (tf32) V needs 32-byte swizzle atoms.
    const CUtensorMapSwizzle v_swizzle = dtype == B200TK_DTYPE_FLOAT32
                                             ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                             : CU_TENSOR_MAP_SWIZZLE_128B;
    rc = encode_map(a.tm_q, q, q_strides, batch, seq_len, heads, head_dim, dtype, 128,
                    CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == B200TK_OK)
      rc = encode_map(a.tm_k, k, k_strides, batch, seq_len, heads, head_dim, dtype, bn,
                      CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc == B200TK_OK)
      rc = encode_map(a.tm_v, v, v_strides, batch, seq_len, heads, head_dim, dtype, bn, v_swizzle);
    if (rc != B200TK_OK) return rc;
    rc = status_address(&a.status);
    if (rc != B200TK_OK) return rc;
    a.out = out;
    a.mask = valid_token_mask;
    a.mask_sb = valid_token_mask ? mask_strides[0] : 0;
    a.mask_ss = valid_token_mask ? mask_strides[1] : 0;
    a.batch = batch;
    a.seq = seq_len;
    a.heads = heads;
    a.head_dim = head_dim;
    a.dtype = dtype;
    a.causal = causal;
    a.scale = scale;
    a.schedule = schedule;
    cudaError_t err = launch_attention_tc(a, st);
    if (err != cudaSuccess) return cuda_fail(err, "attention tcgen05 launch");
    return B200TK_OK;
  }
  AttnGenericArgs g;
  g.q = q;
  g.k = k;
  g.v = v;
  for (int i = 0; i < 3; ++i) {
    g.qs[i] = q_strides[i];
    g.ks[i] = k_strides[i];
    g.vs[i] = v_strides[i];
  }
  g.mask = valid_token_mask;
  g.mask_sb = valid_token_mask ? mask_strides[0] : 0;
  g.mask_ss = valid_token_mask ? mask_strides[1] : 0;
  g.out = out;
  g.batch = batch;
  g.seq = seq_len;
  g.heads = heads;
  g.head_dim = head_dim;
  g.dtype = dtype;
  g.causal = causal;
  g.scale = scale;
  cudaError_t err = launch_attention_generic(g, st);
  if (err != cudaSuccess) return cuda_fail(err, "attention generic launch");
  return B200TK_OK;
}

int b200tk_residual_layer_norm_fwd(const void* x, const void* update, const void* weight,
                                   const void* bias, const uint8_t* valid_mask,
                                   void* residual_out, void* normalized_out, int dtype,
                                   int64_t rows, int64_t width, float eps, uint32_t flags,
                                   void* stream) {
  if (elem_size(dtype) == 0) return fail(B200TK_ERR_INVALID_ARGUMENT, "unknown dtype code");
  if (rows < 0 || width <= 0) return fail(B200TK_ERR_INVALID_ARGUMENT, "rows >= 0 and width > 0");
  if (width > 65536)
    return fail(B200TK_ERR_UNSUPPORTED, "normalized feature dimension exceeds the fused kernel limit");
  if (flags & ~15u) return fail(B200TK_ERR_INVALID_ARGUMENT, "unknown flag bits");
  if ((flags & B200TK_RLN_ROUND_TF32) && dtype != B200TK_DTYPE_FLOAT32)
    return fail(B200TK_ERR_INVALID_ARGUMENT, "TF32 rounding applies to float32 only");
  if ((flags & 3u) && valid_mask == nullptr)
    return fail(B200TK_ERR_INVALID_ARGUMENT, "invalid-row zeroing requires valid_token_mask");
  if (rows == 0) return B200TK_OK;
  const bool has_update = !(flags & B200TK_RLN_NO_UPDATE);
  if (x == nullptr || weight == nullptr || normalized_out == nullptr ||
      (has_update && (update == nullptr || residual_out == nullptr)))
    return fail(B200TK_ERR_INVALID_ARGUMENT, "required pointer is NULL");
  RlnArgs a;
  a.x = x;
  a.update = update;
  a.weight = weight;
  a.bias = bias;
  a.mask = valid_mask;
  a.residual_out = residual_out;
  a.normalized_out = normalized_out;
  a.rows = rows;
  a.width = width;
  a.dtype = dtype;
  a.eps = eps;
  a.flags = flags;
  int rc = status_address(&a.status);
  if (rc != B200TK_OK) return rc;
  cudaError_t err = launch_residual_layer_norm(a, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "residual layer norm launch");
  return B200TK_OK;
}

int b200tk_linear_gelu_fwd(const void* x, const void* weight, const void* bias, void* out,
                           int dtype, int64_t rows, int64_t in_features, int64_t out_features,
                           void* stream) {
  const int es = elem_size(dtype);
  if (es == 0) return fail(B200TK_ERR_INVALID_ARGUMENT, "unknown dtype code");
  if (rows < 0 || in_features <= 0 || out_features <= 0)
    return fail(B200TK_ERR_INVALID_ARGUMENT, "rows >= 0, in_features > 0 and out_features > 0");
  if (rows > (int64_t(1) << 31) - 256 || out_features > (int64_t(1) << 30) ||
      in_features > (int64_t(1) << 30))
    return fail(B200TK_ERR_UNSUPPORTED, "matrix extent exceeds the kernel's index range");
  if ((in_features * es) % 16 != 0 || (out_features * es) % 16 != 0)
    return fail(B200TK_ERR_UNSUPPORTED,
                "in_features and out_features must be multiples of 16 bytes of elements");
  if (rows == 0) return B200TK_OK;
  if (x == nullptr || weight == nullptr || out == nullptr)
    return fail(B200TK_ERR_INVALID_ARGUMENT, "x, weight and out must not be NULL");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out) ||
      (bias != nullptr && !aligned16(bias)))
    return fail(B200TK_ERR_UNSUPPORTED, "x, weight, bias and out must be 16-byte aligned");
  LinearGeluArgs a;
  std::memset(&a, 0, sizeof(a));
  int rc = encode_matrix_map(a.tm_x, x, rows, in_features, dtype, 128);
  if (rc == B200TK_OK) rc = encode_matrix_map(a.tm_w, weight, out_features, in_features, dtype, 128);
  if (rc == B200TK_OK) rc = encode_matrix_map(a.tm_out, out, rows, out_features, dtype, 32);
  if (rc != B200TK_OK) return rc;
  rc = status_address(&a.status);
  if (rc != B200TK_OK) return rc;
  a.bias = bias;
  a.out = out;
  a.rows = rows;
  a.k_in = in_features;
  a.n_out = out_features;
  a.dtype = dtype;
  cudaError_t err = launch_linear_gelu(a, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "linear gelu launch");
  return B200TK_OK;
}

int b200tk_linear_residual_fwd(const void* x, const void* weight, const void* bias,
                               const void* residual, const uint8_t* valid_rows, void* out,
                               int dtype, int64_t rows, int64_t in_features,
                               int64_t out_features, void* stream) {
  const int es = elem_size(dtype);
  if (es == 0) return fail(B200TK_ERR_INVALID_ARGUMENT, "unknown dtype code");
  if (rows < 0 || in_features <= 0 || out_features <= 0)
    return fail(B200TK_ERR_INVALID_ARGUMENT, "rows >= 0, in_features > 0 and out_features > 0");
  if (rows > (int64_t(1) << 31) - 256 || out_features > (int64_t(1) << 30) ||
      in_features > (int64_t(1) << 30))
    return fail(B200TK_ERR_UNSUPPORTED, "matrix extent exceeds the kernel's index range");
  if ((in_features * es) % 16 != 0 || (out_features * es) % 16 != 0)
    return fail(B200TK_ERR_UNSUPPORTED,
                "in_features and out_features must be multiples of 16 bytes of elements");
  if (rows == 0) return B200TK_OK;
  if (x == nullptr || weight == nullptr || residual == nullptr || out == nullptr)
    return fail(B200TK_ERR_INVALID_ARGUMENT, "x, weight, residual and out must not be NULL");
  if (!aligned16(x) || !aligned16(weight) || !aligned16(out) || !aligned16(residual) ||
      (bias != nullptr && !aligned16(bias)))
    return fail(B200TK_ERR_UNSUPPORTED,
                "x, weight, bias, residual and out must be 16-byte aligned");
  LinearGeluArgs a;
  std::memset(&a, 0, sizeof(a));
  int rc = encode_matrix_map(a.tm_x, x, rows, in_features, dtype, 128);
  if (rc == B200TK_OK) rc = encode_matrix_map(a.tm_w, weight, out_features, in_features, dtype, 128);
  if (rc == B200TK_OK) rc = encode_matrix_map(a.tm_out, out, rows, out_features, dtype, 32);
  if (rc != B200TK_OK) return rc;
  rc = status_address(&a.status);
  if (rc != B200TK_OK) return rc;
  a.bias = bias;
  a.residual = residual;
  a.row_mask = valid_rows;
  a.out = out;
  a.rows = rows;
  a.k_in = in_features;
  a.n_out = out_features;
  a.dtype = dtype;
  cudaError_t err = launch_linear_residual(a, static_cast<cudaStream_t>(stream));
  if (err != cudaSuccess) return cuda_fail(err, "linear residual launch");
  return B200TK_OK;
}

int b200tk_device_status(int device, uint32_t* status, int clear) {
  if (status == nullptr) return fail(B200TK_ERR_INVALID_ARGUMENT, "status must not be NULL");
  int prev = 0;
  cudaError_t err = cudaGetDevice(&prev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  err = cudaSetDevice(device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
  unsigned int value = 0;
  err = cudaDeviceSynchronize();
  if (err == cudaSuccess) err = cudaMemcpyFromSymbol(&value, g_device_status, sizeof(value));
  if (err == cudaSuccess && clear) {
    const unsigned int zero = 0;
    err = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(zero));
  }
  cudaSetDevice(prev);
  if (err != cudaSuccess) return cuda_fail(err, "reading the device status word");
  *status = value;
  return B200TK_OK;
}

int b200tk_selftest_wait_timeout(int device, uint32_t timeout_us, void* stream) {
  int prev = 0;
  cudaError_t err = cudaGetDevice(&prev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  err = cudaSetDevice(device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
  unsigned int* st = nullptr;
  int rc = status_address(&st);
  if (rc == B200TK_OK) {
    err = launch_selftest_wait_timeout(st, timeout_us, static_cast<cudaStream_t>(stream));
    if (err == cudaSuccess) err = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (err != cudaSuccess) rc = cuda_fail(err, "self-test wait kernel");
  }
  cudaSetDevice(prev);
  return rc;
}

}  // extern "C"
