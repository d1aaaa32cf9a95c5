// prep.h -- operand preparation kernels (prep.cu).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace vx {

// How the fp16 GEMM operand relates to the stored rows (for the error bound).
enum OperandKind : int {
  kOperandUnitRows = 0,  // fp16(x / |x|): both operands rounded
  kOperandExactRows = 1, // rows already fp16 (FP16 quantizer): only the query is rounded
};

struct Sq8Consts {
  float min_q, max_q, scale, alpha, cm;
  int max_value;  // ScalarBits.maxValue(): 127 (INT8) or 15 (INT4)
};
Sq8Consts sq8_consts(float min_q, float max_q, int max_value = 127);

cudaError_t launch_rows_to_f16(const float* src, int64_t n, int dim, int64_t src_stride, int Dp,
                               bool unit, __half* dst, float* norms, float* norms_sq,
                               float* max_norm, cudaStream_t st, float* errs = nullptr,
                               float* max_err = nullptr);
cudaError_t launch_f16_rows_pad(const __half* src, int64_t n, int dim, int Dp, __half* dst,
                                float* norms_sq, float* max_norm, cudaStream_t st);
cudaError_t launch_zero_f16_rows(__half* dst, int64_t first, int64_t last, int Dp, cudaStream_t st);
cudaError_t launch_margin(const float* qnorm, const float* qerr, int nq, int D, int metric,
                          int operand_kind, const float* max_norm, const float* max_err,
                          float* margin, cudaStream_t st);
cudaError_t launch_sq8_encode_queries(const float* q, int nq, int dim, int Dp8, Sq8Consts k,
                                      int8_t* codes, float* corr, int32_t* sumsq, cudaStream_t st);
// Sign-bit BQ as +-1 int8 operands for the tensor-core Hamming scan: bit set (v >= 0) -> +1,
// clear -> -1, dims [dim, Dp8) -> 0.  Rows from packed words [n][nwp]; queries from fp32.
// With zero_one the clear bits become 0 instead (BBQ rows: the 0/1 operand of rawAsymDot).
cudaError_t launch_bq_words_to_i8(const uint64_t* words, int64_t n, int nwp, int dim, int Dp8, int8_t* dst,
                                  cudaStream_t st, bool zero_one = false);
cudaError_t launch_bq_queries_to_i8(const float* q, int nq, int dim, int Dp8, int8_t* dst, cudaStream_t st);
cudaError_t launch_sq8_rows_pad(const int8_t* src, int64_t n, int dim, int Dp8, int8_t* dst,
                                int32_t* sumsq, cudaStream_t st);

}  // namespace vx
