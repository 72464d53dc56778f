/*
 * b200tk.h - C ABI of libb200tk.so, the sm_100a (B200) kernels behind the
 * Transformer inference hot path: fused attention forward, fused
 * residual-add + LayerNorm, and the FFN input projection with its GELU.
 *
 * Every entry point takes plain device pointers, element strides, sizes and a
 * cudaStream_t passed as void*. Nothing here allocates device memory, blocks
 * the host, or depends on PyTorch, so each call is safe inside CUDA-graph
 * capture once the library has been initialised on the device (the first
 * call on a device resolves the status-word address; make it outside capture).
 *
 * Return value: B200TK_OK or a negative B200TK_ERR_* code. The message for
 * the most recent failure on the calling thread is b200tk_last_error().
 * Device-side pipeline timeouts are not return codes: they are recorded in a
 * per-device status word that b200tk_device_status() reads.
 *
 * The reference implements attention and residual + LayerNorm as Triton
 * kernels behind Python wrappers, and the FFN projection as a cuBLAS GEMM
 * followed by an elementwise GELU; it has no C ABI. The citations below name
 * the reference code each entry point replaces (paths inside the reference
 * project).
 */
#ifndef B200TK_H
#define B200TK_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define B200TK_ABI_VERSION 1

#if defined(__GNUC__)
#define B200TK_API __attribute__((visibility("default")))
#else
#define B200TK_API
#endif

/* Return codes. */
#define B200TK_OK 0
#define B200TK_ERR_INVALID_ARGUMENT (-1) /* shapes, strides, pointers, flags */
#define B200TK_ERR_UNSUPPORTED (-2)      /* valid but outside the kernel envelope */
#define B200TK_ERR_CUDA (-3)             /* a CUDA runtime/driver call failed */

/* Element types. */
#define B200TK_DTYPE_FLOAT32 0
#define B200TK_DTYPE_FLOAT16 1
#define B200TK_DTYPE_BFLOAT16 2

/* Residual LayerNorm flags (bit set). */
#define B200TK_RLN_ZERO_INVALID_RESIDUAL 1u   /* residual_out row := 0 where mask is false */
#define B200TK_RLN_ZERO_INVALID_NORMALIZED 2u /* normalized_out row := 0 where mask is false */
#define B200TK_RLN_NO_UPDATE 4u               /* plain LayerNorm: update and residual_out unused */
#define B200TK_RLN_ROUND_TF32 8u              /* float32: normalized_out rounded to TF32 (see below) */

/* Device status bits (b200tk_device_status). */
#define B200TK_STATUS_PIPELINE_TIMEOUT 1u /* an mbarrier wait hit its iteration/time limit */
#define B200TK_STATUS_SELFTEST_TIMEOUT 2u /* set only by b200tk_selftest_wait_timeout */

/* Softmax schedules of the 16-bit tensor-core attention
 * (b200tk_attention_fwd_scheduled). TWO_PASS computes every row's maximum and
 * sum first and then rounds the already normalised probabilities to the
 * input dtype before P@V -- the explicit reference's rounding boundary, at
 * the cost of a second Q K^T and a second exp per score. ONE_PASS is the
 * online softmax: unnormalised probabilities are rounded to the input dtype
 * and the output is divided by the row sum at the end (one Q K^T, one exp).
 * RESIDENT keeps TWO_PASS's rounding boundary with one Q K^T and one exp per
 * score: the whole score row of a 128-row query tile stays in tensor memory
 * (float16/bfloat16, head_dim 64, seq_len <= 512, scale > 0 only).
 * AUTO picks per call (b200tk_attention_fwd): RESIDENT where it applies,
 * ONE_PASS from seq_len 4096, else TWO_PASS. float32 always runs its single
 * 3xTF32 schedule; the CUDA-core route is always online. */
#define B200TK_SCHEDULE_AUTO 0
#define B200TK_SCHEDULE_TWO_PASS 1
#define B200TK_SCHEDULE_ONE_PASS 2
#define B200TK_SCHEDULE_RESIDENT 3

/* Attention kernel routes reported by b200tk_attention_route. */
#define B200TK_ROUTE_TCGEN05 1 /* TMA + tcgen05.mma + TMEM pipeline */
#define B200TK_ROUTE_GENERIC 2 /* CUDA-core kernel for shapes outside the tcgen05 envelope */

/* ABI version of the loaded library (B200TK_ABI_VERSION at build time). */
B200TK_API int b200tk_abi_version(void);

/* Human-readable message for the last failed call on this host thread. */
B200TK_API const char* b200tk_last_error(void);

/*
 * Fused attention forward: out = softmax(scale * q k^T + masks) v, per
 * (batch, head), without materialising the score matrix.
 *
 * Replaces: transformer_opt/kernels/attention.py:268-360 (triton_attention,
 * launching _attention_fwd at :103-265). Semantics follow the explicit
 * reference math, transformer_opt/dispatch.py:69-96.
 *
 * q, k, v : [batch, seq_len, heads, head_dim] in `dtype`, arbitrary element
 *           strides for the first three dims (packed QKV views included);
 *           the head_dim stride must be 1. Strides are given as 3 int64
 *           element strides {batch, seq, head}.
 * valid_token_mask : optional [batch, seq_len] bool (1 byte per element,
 *           strides {batch, seq} in elements); NULL means all keys valid.
 *           A false entry removes that key for every query.
 * out     : contiguous [batch, seq_len, heads, head_dim] in `dtype`.
 * causal  : nonzero applies the key <= query constraint.
 * scale   : multiplies q k^T (head_dim^-0.5 in the model).
 * Rows whose keys are all masked produce zeros.
 * head_dim in {8, 16, 32, 64, 128}; dtype float32 runs a 3xTF32 split on the
 * tensor cores, float16/bfloat16 run native f16-kind MMAs with fp32
 * accumulation.
 */
B200TK_API int b200tk_attention_fwd(const void* q, const int64_t* q_strides, const void* k,
                         const int64_t* k_strides, const void* v, const int64_t* v_strides,
                         const uint8_t* valid_token_mask, const int64_t* mask_strides,
                         void* out, int dtype, int64_t batch, int64_t seq_len, int64_t heads,
                         int64_t head_dim, int causal, float scale, void* stream);

/*
 * b200tk_attention_fwd with an explicit softmax schedule for 16-bit inputs
 * (B200TK_SCHEDULE_*; AUTO is b200tk_attention_fwd itself). A schedule
 * outside that set is B200TK_ERR_INVALID_ARGUMENT; ONE_PASS with scale <= 0
 * runs TWO_PASS; RESIDENT on arguments outside its envelope (or that leave
 * the tensor-core route) is B200TK_ERR_UNSUPPORTED.
 *
 * Replaces: the same reference kernel as b200tk_attention_fwd; the schedule
 * choice has no counterpart there (its fp16 kernel is online,
 * attention.py:236-247).
 */
B200TK_API int b200tk_attention_fwd_scheduled(
    const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
    const void* v, const int64_t* v_strides, const uint8_t* valid_token_mask,
    const int64_t* mask_strides, void* out, int dtype, int64_t batch, int64_t seq_len,
    int64_t heads, int64_t head_dim, int causal, float scale, int schedule, void* stream);

/*
 * Which kernel b200tk_attention_fwd would launch for these arguments
 * (B200TK_ROUTE_*), or a negative error code. Pure host-side query.
 */
B200TK_API int b200tk_attention_route(const void* q, const int64_t* q_strides, const void* k,
                           const int64_t* k_strides, const void* v, const int64_t* v_strides,
                           int dtype, int64_t batch, int64_t seq_len, int64_t heads,
                           int64_t head_dim);

/*
 * Fused residual add + LayerNorm over the last dimension of contiguous rows:
 *   residual_out   = x + update           (rounded to dtype)
 *   normalized_out = (r - mean(r)) * rsqrt(var(r) + eps) * weight + bias
 * with fp32 statistics. With valid_mask (one bool per row) and the
 * B200TK_RLN_ZERO_* flags, invalid rows are zeroed in the chosen outputs.
 * B200TK_RLN_NO_UPDATE turns the call into a plain LayerNorm of x.
 * B200TK_RLN_ROUND_TF32 (float32 only) rounds normalized_out to the nearest
 * TF32 value (10 mantissa bits, ties away from zero) -- the operand rounding
 * of a TF32 matmul, done once here for a consumer whose tensor cores read
 * the operand as stored (b200tk_linear_gelu_fwd).
 *
 * Replaces: transformer_opt/kernels/residual_layer_norm.py:159-238
 * (fused_residual_layer_norm, launching _residual_layer_norm_fwd at :73-126).
 *
 * x, update, residual_out, normalized_out : [rows, width] contiguous.
 * weight : [width]; bias : [width] or NULL. valid_mask : [rows] or NULL.
 */
B200TK_API int b200tk_residual_layer_norm_fwd(const void* x, const void* update, const void* weight,
                                   const void* bias, const uint8_t* valid_mask,
                                   void* residual_out, void* normalized_out, int dtype,
                                   int64_t rows, int64_t width, float eps, uint32_t flags,
                                   void* stream);

/*
 * FFN input projection with its activation fused into the GEMM epilogue:
 *   out[m, n] = gelu(sum_k x[m, k] * weight[n, k] + bias[n])
 * with the exact (erf) GELU, v * 0.5 * (1 + erf(v / sqrt(2))).
 *
 * Replaces: the `F.gelu(layer.ffn_in(h), approximate="none")` pair of the
 * reference's block (benchmarks/torch_transformer_benchmark.py:131, 141), as
 * placed by its fused layer loop at transformer_opt/submission.py:506-508
 * (there: a cuBLAS GEMM followed by a separate elementwise GELU pass).
 *
 * x      : [rows, in_features] row-major.   weight : [out_features, in_features]
 *          row-major (nn.Linear layout).     bias : [out_features] or NULL.
 * out    : [rows, out_features] row-major, in `dtype`.
 * Accumulation and bias are fp32. float32 multiplies as TF32: the tensor
 * cores read the top 19 bits of each operand (they truncate), so callers
 * matching a round-to-nearest TF32 matmul pass x and weight already rounded
 * (B200TK_RLN_ROUND_TF32 for x; the weight once, when it is loaded).
 * float16/bfloat16 round the biased sum to dtype before the GELU, as the
 * unfused Linear's output tensor does.
 * in_features and out_features must be multiples of 16 bytes of elements and
 * every pointer 16-byte aligned (B200TK_ERR_UNSUPPORTED otherwise).
 */
B200TK_API int b200tk_linear_gelu_fwd(const void* x, const void* weight, const void* bias,
                                      void* out, int dtype, int64_t rows, int64_t in_features,
                                      int64_t out_features, void* stream);

/*
 * out_proj / ffn_out with the residual add that follows it fused into the
 * GEMM epilogue:
 *   out[m, n] = residual[m, n] + (sum_k x[m, k] * weight[n, k] + bias[n])
 * and, when valid_rows is given, out[m, :] = 0 for every row m whose byte is 0
 * (the block-end zeroing of padded rows).
 *
 * Replaces: the `x + layer.attention(...)` / `x + layer.ffn_out(...)` pairs of
 * the reference's block (benchmarks/torch_transformer_benchmark.py:140-141),
 * as placed by its fused layer loop at transformer_opt/submission.py:499-523
 * (there: a cuBLAS GEMM writing the projection, then the residual-add kernel
 * reading it back).
 *
 * x : [rows, in_features], weight : [out_features, in_features] (nn.Linear
 * layout), residual and out : [rows, out_features], all row-major in `dtype`;
 * bias : [out_features] or NULL; valid_rows : [rows] bytes or NULL. out may
 * not alias x; it may alias residual. Accumulation and bias are fp32; the
 * projection is rounded to dtype before the add (16-bit), as the unfused
 * Linear's output tensor is, and the sum is rounded to dtype. float32
 * multiplies as TF32 with truncated operands (see b200tk_linear_gelu_fwd).
 * Alignment and size rules are those of b200tk_linear_gelu_fwd.
 */
B200TK_API int b200tk_linear_residual_fwd(const void* x, const void* weight, const void* bias,
                                          const void* residual, const uint8_t* valid_rows,
                                          void* out, int dtype, int64_t rows,
                                          int64_t in_features, int64_t out_features,
                                          void* stream);

/*
 * Read (and, with clear != 0, reset) the device status word of `device`.
 * Synchronises the device. Not for use inside stream capture.
 */
B200TK_API int b200tk_device_status(int device, uint32_t* status, int clear);

/*
 * Failure-detection self test: launches one CTA that waits on an mbarrier
 * nothing arrives on, with a wait limit of timeout_us microseconds. The
 * kernel gives up, records B200TK_STATUS_SELFTEST_TIMEOUT in the status word
 * and returns; the GPU context stays usable. Synchronises the stream.
 */
B200TK_API int b200tk_selftest_wait_timeout(int device, uint32_t timeout_us, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* B200TK_H */
