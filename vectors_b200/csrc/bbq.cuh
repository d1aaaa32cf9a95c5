// bbq.cuh -- BBQ score arithmetic shared by the popcount scan (bq_scan.cu) and the epilogue of
// the int8 tensor-core scan (gemm_scan.cu), so that both produce the same float bits.
//
// BinaryQuantizedVectors.bbqScoreFunction (vectors-quantization/.../BinaryQuantizedVectors.java:
// 110-275): computeBbqDot in Java's float order, without fused multiply-adds,
//     approx = queryMin * (vl * D + width * pop) + (queryWidth / 15) * (vl * querySum + width * raw)
// where raw = rawAsymDot is an exact integer, followed by the metric's transform (:155-225).
#pragma once
#include <cstdint>
#include "kernels.h"

namespace vx {

// The row's own term vl * D + width * popcount(bits).
__device__ __forceinline__ float bbq_row_term(float vl, float width, int dim, int32_t pop) {
  return __fadd_rn(__fmul_rn(vl, (float)dim), __fmul_rn(width, (float)pop));
}

// computeBbqDot from the query's (queryMin, queryWidth / 15, querySum), the row's (vl, width,
// row term) and rawAsymDot as a float (exact: |raw| <= 15 * 1024).
__device__ __forceinline__ float bbq_approx(float qmin, float w15, float qsum, float vl, float width, float s1,
                                            float raw) {
  const float s2 = __fadd_rn(__fmul_rn(vl, qsum), __fmul_rn(width, raw));
  return __fadd_rn(__fmul_rn(qmin, s1), __fmul_rn(w15, s2));
}

// EUCLIDEAN: max(queryNormSq + |v - c|^2 - 2 approx, 0) (NaN -> 0); the score is 1 / (1 + that),
// non-increasing in it.
__device__ __forceinline__ float bbq_l2_adj(float approx, float nsq, float dist_c) {
  const float adj = __fsub_rn(__fadd_rn(nsq, dist_c), __fmul_rn(2.0f, approx));
  return adj > 0.0f ? adj : 0.0f;
}
__device__ __forceinline__ float bbq_l2_score(float clamped_adj) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, clamped_adj));
}

// DOT_PRODUCT: max((1 + approx) / 2, 0) (NaN -> 0); x / 2f and x * 0.5f round alike.
__device__ __forceinline__ float bbq_dot_score(float approx) {
  const float s = __fmul_rn(__fadd_rn(1.0f, approx), 0.5f);
  return s > 0.0f ? s : 0.0f;
}

// COSINE: approx / (|q - c| |v - c|), 0 when either norm is 0, then as DOT_PRODUCT.
__device__ __forceinline__ float bbq_cos_score(float approx, float qnorm, float vnorm) {
  if (qnorm == 0.0f || vnorm == 0.0f) return 0.0f;
  return bbq_dot_score(__fdiv_rn(approx, __fmul_rn(qnorm, vnorm)));
}

// |v - c| from |v - c|^2: (float) Math.sqrt((double) x).
__device__ __forceinline__ float bbq_vnorm(float dist_c) { return (float)sqrt((double)dist_c); }

}  // namespace vx
