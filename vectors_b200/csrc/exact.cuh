// exact.cuh -- warp-cooperative restatements of the reference fp32 kernels, evaluated in the
// Java Vector API's operation order so that re-scored candidates carry the reference's
// scores.  One warp scores one (query, row) pair; lane l owns Java accumulator l/8, vector
// lane l%8 (8-lane FloatVector at the 256-bit cap, PanamaConstants.java:47).
//
//   dotProduct      PanamaVectorUtilSupport.java:208-271 (lane sum order :1377-1386)
//   squareDistance  PanamaVectorUtilSupport.java:280-343
//   cosine          PanamaVectorUtilSupport.java:347-456
// The scalar tails use Math.fma where Java does (dot, cosine) and two roundings where Java
// writes "res += diff * diff" (squareDistance).  All arithmetic uses explicit _rn intrinsics,
// so no contraction can change the result.
#pragma once
#include <cuda_fp16.h>
#include "common.cuh"
#include "kernels.h"

namespace vx {

// Row sources: fp32 rows, or fp16 rows decoded exactly to fp32 (Fp16Quantizer.decodeInto,
// Fp16Quantizer.java:94-106).
struct RowF32 {
  const float* p;
  __device__ __forceinline__ float operator[](int i) const { return p[i]; }
};
struct RowF16 {
  const __half* p;
  __device__ __forceinline__ float operator[](int i) const { return __half2float(p[i]); }
};

// Sum of the 8 vector lanes held by lanes 0..7 in PanamaVectorUtilSupport.reduceAdd order;
// the result is valid in lane 0.
__device__ __forceinline__ float warp_reduce_add8(float v) {
  const unsigned F = 0xFFFFFFFFu;
  float l0 = __shfl_sync(F, v, 0), l1 = __shfl_sync(F, v, 1), l2 = __shfl_sync(F, v, 2),
        l3 = __shfl_sync(F, v, 3), l4 = __shfl_sync(F, v, 4), l5 = __shfl_sync(F, v, 5),
        l6 = __shfl_sync(F, v, 6), l7 = __shfl_sync(F, v, 7);
  float even = __fadd_rn(__fadd_rn(l4, l0), __fadd_rn(l6, l2));
  float odd = __fadd_rn(__fadd_rn(l5, l1), __fadd_rn(l7, l3));
  return __fadd_rn(even, odd);
}

// (acc1 + acc2) + (acc3 + acc4) lane-wise, from lanes j, j+8, j+16, j+24 into lane j.
__device__ __forceinline__ float warp_combine4(float acc) {
  const unsigned F = 0xFFFFFFFFu;
  const int lane = threadIdx.x & 31;
  float a2 = __shfl_sync(F, acc, (lane & 7) + 8);
  float a3 = __shfl_sync(F, acc, (lane & 7) + 16);
  float a4 = __shfl_sync(F, acc, (lane & 7) + 24);
  return __fadd_rn(__fadd_rn(acc, a2), __fadd_rn(a3, a4));
}

// Java dotProduct(a, b, len); result valid in every lane.
template <class A, class B>
__device__ __forceinline__ float warp_dot(A a, B b, int len) {
  const int lane = threadIdx.x & 31;
  float res = 0.0f;
  int i = 0;
  if (len > 16) {
    const int limit = len & ~7;
    const int unrolled = limit - 24;
    float acc = 0.0f;
    int p = 0;
    for (; p < unrolled; p += 32) acc = __fmaf_rn(a[p + lane], b[p + lane], acc);
    if (lane < 8)
      for (int r = p; r < limit; r += 8) acc = __fmaf_rn(a[r + lane], b[r + lane], acc);
    float s = warp_combine4(acc);
    float total = warp_reduce_add8(s);
    res = __fadd_rn(res, total);
    i = limit;
  }
  for (; i < len; i++) res = __fmaf_rn(a[i], b[i], res);  // uniform across lanes
  return __shfl_sync(0xFFFFFFFFu, res, 0);
}

// Java squareDistance(a, b, len); result valid in every lane.
template <class A, class B>
__device__ __forceinline__ float warp_sqdist(A a, B b, int len) {
  const int lane = threadIdx.x & 31;
  float res = 0.0f;
  int i = 0;
  if (len > 16) {
    const int limit = len & ~7;
    const int unrolled = limit - 24;
    float acc = 0.0f;
    int p = 0;
    for (; p < unrolled; p += 32) {
      float d = __fsub_rn(a[p + lane], b[p + lane]);
      acc = __fmaf_rn(d, d, acc);
    }
    if (lane < 8)
      for (int r = p; r < limit; r += 8) {
        float d = __fsub_rn(a[r + lane], b[r + lane]);
        acc = __fmaf_rn(d, d, acc);
      }
    float s = warp_combine4(acc);
    float total = warp_reduce_add8(s);
    res = __fadd_rn(res, total);
    i = limit;
  }
  for (; i < len; i++) {
    float d = __fsub_rn(a[i], b[i]);
    res = __fadd_rn(res, __fmul_rn(d, d));
  }
  return __shfl_sync(0xFFFFFFFFu, res, 0);
}

// Java cosine(a, b); result valid in every lane.
template <class A, class B>
__device__ __forceinline__ float warp_cosine(A a, B b, int len) {
  const int lane = threadIdx.x & 31;
  float sum = 0.0f, n1 = 0.0f, n2 = 0.0f;
  int i = 0;
  if (len >= 32) {
    const int limit = len & ~7;
    const int unrolled = limit - 24;
    float s = 0.0f, x = 0.0f, y = 0.0f;
    int p = 0;
    for (; p < unrolled; p += 32) {
      float va = a[p + lane], vb = b[p + lane];
      s = __fmaf_rn(va, vb, s);
      x = __fmaf_rn(va, va, x);
      y = __fmaf_rn(vb, vb, y);
    }
    if (lane < 8)
      for (int r = p; r < limit; r += 8) {
        float va = a[r + lane], vb = b[r + lane];
        s = __fmaf_rn(va, vb, s);
        x = __fmaf_rn(va, va, x);
        y = __fmaf_rn(vb, vb, y);
      }
    sum = warp_reduce_add8(warp_combine4(s));
    n1 = warp_reduce_add8(warp_combine4(x));
    n2 = warp_reduce_add8(warp_combine4(y));
    i = limit;
  } else if (len >= 8) {
    const int limit = len & ~7;
    float s = 0.0f, x = 0.0f, y = 0.0f;
    if (lane < 8)
      for (int r = 0; r < limit; r += 8) {
        float va = a[r + lane], vb = b[r + lane];
        s = __fmaf_rn(va, vb, s);
        x = __fmaf_rn(va, va, x);
        y = __fmaf_rn(vb, vb, y);
      }
    sum = warp_reduce_add8(s);
    n1 = warp_reduce_add8(x);
    n2 = warp_reduce_add8(y);
    i = limit;
  }
  sum = __shfl_sync(0xFFFFFFFFu, sum, 0);
  n1 = __shfl_sync(0xFFFFFFFFu, n1, 0);
  n2 = __shfl_sync(0xFFFFFFFFu, n2, 0);
  for (; i < len; i++) {
    float va = a[i], vb = b[i];
    sum = __fmaf_rn(va, vb, sum);
    n1 = __fmaf_rn(va, va, n1);
    n2 = __fmaf_rn(vb, vb, n2);
  }
  double den = __dsqrt_rn(__dmul_rn((double)n1, (double)n2));
  return __double2float_rn(__ddiv_rn((double)sum, den));
}

// Score transforms.  Flat: SimilarityFunction.compare (SimilarityFunction.java:36-120).
// Fp16Quantized: Fp16QuantizedVectors.scoreFunctionFor (Fp16QuantizedVectors.java:70-94),
// which clamps DOT/COSINE at 0 and treats COSINE like DOT.
// IvfRaw: IvfIndex.score (vectors-ivf/.../IvfIndex.java:623-629), the untransformed similarity
// used by the IVF rescore pass.  (ScoreFlavor is declared in kernels.h.)

template <class A, class B>
__device__ __forceinline__ float warp_exact_score(int flavor, int metric, A q, B x, int dim) {
  if (flavor == kFlavorIvfRaw) {
    if (metric == kEuclidean) return -warp_sqdist(q, x, dim);
    if (metric == kCosine) return warp_cosine(q, x, dim);
    return warp_dot(q, x, dim);
  }
  if (metric == kEuclidean) {
    float d = warp_sqdist(q, x, dim);
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, d));
  }
  if (metric == kCosine && flavor == kFlavorFlat) {
    float c = warp_cosine(q, x, dim);
    return __fdiv_rn(__fadd_rn(1.0f, c), 2.0f);
  }
  float dot = warp_dot(q, x, dim);
  if (metric == kMaxInnerProduct) return scale_mip(dot);
  float h = __fdiv_rn(__fadd_rn(1.0f, dot), 2.0f);
  if (flavor == kFlavorFp16Quantized) return h >= 0.0f ? h : (h != h ? h : 0.0f);
  return h;
}

}  // namespace vx
