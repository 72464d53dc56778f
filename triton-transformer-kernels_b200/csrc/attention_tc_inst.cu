// attention_tc_inst.cu - one explicit instantiation of the tcgen05 attention
// kernel family, selected at compile time by B200TK_TC_DTYPE (0 fp32, 1 fp16,
// 2 bf16) and B200TK_TC_HEAD_DIM (64 or 128). The build compiles this file
// once per combination.
#include "attention_tc.cuh"

#if !defined(B200TK_TC_DTYPE) || !defined(B200TK_TC_HEAD_DIM)
#error "define B200TK_TC_DTYPE and B200TK_TC_HEAD_DIM"
#endif

#if B200TK_TC_DTYPE == 0
#define B200TK_TC_T float
#elif B200TK_TC_DTYPE == 1
#define B200TK_TC_T __half
#else
#define B200TK_TC_T __nv_bfloat16
#endif

namespace b200tk {
namespace tc {
template cudaError_t launch_dtype_hd<B200TK_TC_T, B200TK_TC_HEAD_DIM>(AttnTcParams, int, bool,
                                                                      bool, cudaStream_t);
}  // namespace tc
}  // namespace b200tk
