// prep.cu -- operand preparation for the scans: fp16 GEMM operands with their norms, the
// per-query bound on the approximate key error, and the SQ8 query encoder.
#include <cuda_fp16.h>
#include "common.cuh"
#include "prep.h"

namespace vx {

namespace {

__device__ __forceinline__ void atomic_max_pos_float(float* addr, float v) {
  // non-negative floats order like their bit patterns
  atomicMax((int*)addr, __float_as_int(v));
}

// One warp per row: norm in double, then fp16(x / |x|) (or fp16(x) when !unit) into a
// zero-padded row of Dp halves.  Also the Euclidean norm of the rounding error
// |fp16(x/|x|) - x/|x||, which bounds the operand's contribution to the approximate key's
// error by Cauchy-Schwarz (per row into errs, and its maximum into max_err).
__global__ void rows_to_f16_kernel(const float* __restrict__ src, int64_t n, int dim,
                                   int64_t src_stride, int Dp, int unit, __half* __restrict__ dst,
                                   float* __restrict__ norms, float* __restrict__ norms_sq,
                                   float* __restrict__ max_norm, float* __restrict__ errs,
                                   float* __restrict__ max_err) {
  const int lane = threadIdx.x & 31;
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= n) return;
  const float* x = src + row * src_stride;
  double s = 0.0;
  for (int i = lane; i < dim; i += 32) s += (double)x[i] * (double)x[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  const double normd = sqrt(s);
  const float norm = (float)normd;
  const float inv = (unit && norm > 0.0f) ? 1.0f / norm : 1.0f;
  const double invd = (unit && normd > 0.0) ? 1.0 / normd : 1.0;
  __half* d = dst + row * (int64_t)Dp;
  double e = 0.0;
  for (int i = lane; i < Dp; i += 32) {
    const __half h = __float2half_rn(i < dim ? x[i] * inv : 0.0f);
    d[i] = h;
    if (i < dim) {
      const double diff = (double)__half2float(h) - (double)x[i] * invd;
      e += diff * diff;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xFFFFFFFFu, e, o);
  if (lane == 0) {
    if (norms) norms[row] = unit ? norm : 1.0f;
    if (norms_sq) norms_sq[row] = (float)s;
    if (max_norm) atomic_max_pos_float(max_norm, norm);
    // rounded up so that the float never understates the double
    const float ef = __double2float_ru(sqrt(e));
    if (errs) errs[row] = ef;
    if (max_err) atomic_max_pos_float(max_err, ef);
  }
}

// fp16 rows given in the reference encoding (little-endian binary16, Fp16Quantizer.java:72-85):
// copy into padded rows and compute norms of the decoded values.
__global__ void f16_rows_pad_kernel(const __half* __restrict__ src, int64_t n, int dim, int Dp,
                                    __half* __restrict__ dst, float* __restrict__ norms_sq,
                                    float* __restrict__ max_norm) {
  const int lane = threadIdx.x & 31;
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= n) return;
  const __half* x = src + row * (int64_t)dim;
  double s = 0.0;
  __half* d = dst + row * (int64_t)Dp;
  for (int i = lane; i < Dp; i += 32) {
    __half h = i < dim ? x[i] : __float2half_rn(0.0f);
    d[i] = h;
    double v = (double)__half2float(h);
    s += v * v;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  if (lane == 0) {
    norms_sq[row] = (float)s;
    atomic_max_pos_float(max_norm, (float)sqrt(s));
  }
}

// Bound on |approximate key - exact key| per query (see rescore.cu for the argument).
// With unit vectors q^ = q/|q|, x^ = x/|x| and their fp16 roundings q^ + e_q, x^ + e_x:
//   |(q^+e_q).(x^+e_x) - q^.x^| <= |e_q| + |e_x| + |e_q||e_x|      (Cauchy-Schwarz),
// using the measured error norms (qerr per query, rerr_max over all rows; 0 for rows that are
// stored in fp16 already).  The tensor core's fp32 accumulation adds at most (D+1) 2^-23 of the
// sum of |products| (<= 1 + |e| terms); the reference's own fp32 evaluation (32 lane partial
// sums of ~D/32 terms, then a 5-level combine, plus a scalar tail) adds (D/32 + 24) 2^-24; the
// final score transform's rounding adds 2^-21 of the score scale.
__global__ void margin_kernel(const float* __restrict__ qnorm, const float* __restrict__ qerr,
                              int nq, int D, int metric, int operand_kind,
                              const float* __restrict__ max_norm_ptr,
                              const float* __restrict__ max_err_ptr, float* __restrict__ margin) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const double xmax = (double)*max_norm_ptr;
  const double qn = (double)qnorm[q];
  const double eq = (double)qerr[q];
  const double ex = (operand_kind == kOperandUnitRows) ? (double)*max_err_ptr : 0.0;
  const double acc = (D + 1) * 0x1.0p-23 * (1.0 + eq + ex + eq * ex);
  const double ref = (D / 32 + 24) * 0x1.0p-24;
  // error of the normalised dot, per unit of |x| (rows stored in fp16 are exact, not unit)
  const double c = eq + ex + eq * ex + acc;
  double m;
  if (metric == 2 /* COSINE */ && operand_kind == kOperandUnitRows) {
    m = c + ref + 0x1.0p-21;
  } else if (metric == 0 /* EUCLIDEAN */) {
    const double big = (qn + xmax) * (qn + xmax);
    m = 2.0 * qn * xmax * (c + ref) + ref * big + 0x1.0p-21 * (1.0 + big) + 0x1.0p-22 * big;
  } else {  // DOT_PRODUCT / MAXIMUM_INNER_PRODUCT (and COSINE over fp16-quantized rows)
    m = (qn > 0.0) ? xmax * (c + ref) + 0x1.0p-21 * (1.0 + qn * xmax) / qn : INFINITY;
  }
  if (!(qn > 0.0) && metric != 0) m = INFINITY;
  margin[q] = (float)(m * 1.0001 + 1e-30);
}

// SQ8 / SQ4 query encoder: ScalarQuantizer.encodeInt8 / encodeInt4Unpacked / quantizeValue /
// correctionTerm (ScalarQuantizer.java:243-272,343-351), sequential over dimensions, one thread per query, every
// operation rounded as Java rounds it.  Also returns sum of squared codes for EUCLIDEAN.
__global__ void sq8_encode_queries_kernel(const float* __restrict__ q, int nq, int dim, int Dp8,
                                          Sq8Consts k, int8_t* __restrict__ codes,
                                          float* __restrict__ corr, int32_t* __restrict__ sumsq) {
  const int qi = blockIdx.x * blockDim.x + threadIdx.x;
  if (qi >= nq) return;
  const float* v = q + (size_t)qi * dim;
  int8_t* out = codes + (size_t)qi * Dp8;
  float c = 0.0f;
  int32_t ss = 0;
  const float half = __fdiv_rn(k.min_q, 2.0f);
  for (int i = 0; i < dim; i++) {
    const float x = v[i];
    // Math.max(minQ, Math.min(maxQ, v)) - minQ
    float clamped = fminf(k.max_q, x);
    if (x != x) clamped = x;
    float lo = fmaxf(k.min_q, clamped);
    if (clamped != clamped) lo = clamped;
    const float dxc = __fsub_rn(lo, k.min_q);
    // Math.round(scale * dxc): nearest, ties toward +infinity; NaN -> 0
    const float t = __fmul_rn(k.scale, dxc);
    int32_t qv;
    if (t != t) {
      qv = 0;
    } else {
      const float f = floorf(t);
      qv = (int32_t)f + ((__fsub_rn(t, f) >= 0.5f) ? 1 : 0);
    }
    qv = qv < 0 ? 0 : (qv > k.max_value ? k.max_value : qv);
    out[i] = (int8_t)qv;
    ss += qv * qv;
    const float dx = __fsub_rn(x, k.min_q);
    const float dxq = __fmul_rn((float)qv, k.alpha);
    const float t1 = __fmul_rn(k.min_q, __fsub_rn(x, half));
    const float t2 = __fmul_rn(__fsub_rn(dx, dxq), dxq);
    c = __fadd_rn(c, __fadd_rn(t1, t2));
  }
  for (int i = dim; i < Dp8; i++) out[i] = 0;
  corr[qi] = c;
  sumsq[qi] = ss;
}

// Row codes for SQ8: copy into padded rows and compute sum of squared codes.
__global__ void sq8_rows_pad_kernel(const int8_t* __restrict__ src, int64_t n, int dim, int Dp8,
                                    int8_t* __restrict__ dst, int32_t* __restrict__ sumsq) {
  const int lane = threadIdx.x & 31;
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (row >= n) return;
  int32_t s = 0;
  for (int i = lane; i < Dp8; i += 32) {
    int8_t c = i < dim ? src[row * dim + i] : (int8_t)0;
    dst[row * Dp8 + i] = c;
    s += (int32_t)c * (int32_t)c;
  }
  s = __reduce_add_sync(0xFFFFFFFFu, s);
  if (lane == 0) sumsq[row] = s;
}

__global__ void zero_rows_kernel(__half* dst, int64_t first, int64_t last, int Dp) {
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t total = (last - first) * Dp;
  if (i < total) dst[first * Dp + i] = __float2half_rn(0.0f);
}

}  // namespace

cudaError_t launch_rows_to_f16(const float* src, int64_t n, int dim, int64_t src_stride, int Dp,
                               bool unit, __half* dst, float* norms, float* norms_sq,
                               float* max_norm, cudaStream_t st, float* errs, float* max_err) {
  if (n <= 0) return cudaSuccess;
  const int64_t threads = n * 32;
  const int blocks = (int)((threads + 255) / 256);
  rows_to_f16_kernel<<<blocks, 256, 0, st>>>(src, n, dim, src_stride, Dp, unit ? 1 : 0, dst, norms,
                                             norms_sq, max_norm, errs, max_err);
  return cudaGetLastError();
}

cudaError_t launch_f16_rows_pad(const __half* src, int64_t n, int dim, int Dp, __half* dst,
                                float* norms_sq, float* max_norm, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int blocks = (int)((n * 32 + 255) / 256);
  f16_rows_pad_kernel<<<blocks, 256, 0, st>>>(src, n, dim, Dp, dst, norms_sq, max_norm);
  return cudaGetLastError();
}

cudaError_t launch_zero_f16_rows(__half* dst, int64_t first, int64_t last, int Dp, cudaStream_t st) {
  if (last <= first) return cudaSuccess;
  const int64_t total = (last - first) * Dp;
  zero_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(dst, first, last, Dp);
  return cudaGetLastError();
}

cudaError_t launch_margin(const float* qnorm, const float* qerr, int nq, int D, int metric,
                          int operand_kind, const float* max_norm, const float* max_err,
                          float* margin, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  margin_kernel<<<(nq + 127) / 128, 128, 0, st>>>(qnorm, qerr, nq, D, metric, operand_kind,
                                                 max_norm, max_err, margin);
  return cudaGetLastError();
}

cudaError_t launch_sq8_encode_queries(const float* q, int nq, int dim, int Dp8, Sq8Consts k,
                                      int8_t* codes, float* corr, int32_t* sumsq, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  sq8_encode_queries_kernel<<<(nq + 127) / 128, 128, 0, st>>>(q, nq, dim, Dp8, k, codes, corr, sumsq);
  return cudaGetLastError();
}

cudaError_t launch_sq8_rows_pad(const int8_t* src, int64_t n, int dim, int Dp8, int8_t* dst,
                                int32_t* sumsq, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int blocks = (int)((n * 32 + 255) / 256);
  sq8_rows_pad_kernel<<<blocks, 256, 0, st>>>(src, n, dim, Dp8, dst, sumsq);
  return cudaGetLastError();
}

// ScalarQuantizer constructor constants (ScalarQuantizer.java:59-69): maxValue 127 for INT8,
// 15 for INT4 (ScalarBits.java:30-33); the int is promoted to float as in Java.
Sq8Consts sq8_consts(float min_q, float max_q, int max_value) {
  Sq8Consts k;
  k.min_q = min_q;
  k.max_q = max_q;
  k.max_value = max_value;
  const float range = max_q - min_q;
  k.scale = (range == 0.0f) ? 0.0f : (float)max_value / range;
  k.alpha = (range == 0.0f) ? 0.0f : range / (float)max_value;
  k.cm = k.alpha * k.alpha;
  return k;
}

// Four bits -> four bytes: bit j of b lands in bit 0 of byte j (b * 0x00204081 places copies of b
// at bit offsets 0, 7, 14 and 21, so bit j of the copy at 7j sits at bit 8j).
__device__ __forceinline__ uint32_t spread4(uint32_t b) { return (b * 0x00204081u) & 0x01010101u; }

// One thread per 16 output bytes of a row (Dp8 is a multiple of 128, so of 16): the 16 bits at
// column c0 of one word, set -> 1, clear -> `clear` (-1 or 0), columns >= dim -> 0; one 16-byte
// store.  Row windows of the tensor scan run this at search time, so it is a plain stream
// (8 bytes of bits read per 128 bytes written, the bit word shared by four threads through L1).
__global__ void bq_words_to_i8_kernel(const uint64_t* __restrict__ words, int64_t n, int nwp, int dim,
                                      int Dp8, int8_t clear, int8_t* __restrict__ dst) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int per_row = Dp8 / 16;
  if (t >= n * per_row) return;
  const int64_t r = t / per_row;
  const int c0 = (int)(t - r * per_row) * 16;
  const int nvalid = min(max(dim - c0, 0), 16);
  const uint32_t vm = nvalid >= 16 ? 0xFFFFu : ((1u << nvalid) - 1u);
  const uint32_t bits = nvalid > 0 ? (uint32_t)(words[r * nwp + (c0 >> 6)] >> (c0 & 63)) & vm : 0u;
  const uint32_t fill = (uint32_t)(uint8_t)clear;  // 0xFF or 0: per byte, no carries below
  uint32_t o[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const uint32_t m = spread4((bits >> (4 * j)) & 0xFu);
    const uint32_t valid = spread4((vm >> (4 * j)) & 0xFu);
    o[j] = m | ((m ^ valid) * fill);  // set: 0x01; clear and valid: fill; past dim: 0
  }
  reinterpret_cast<uint4*>(dst + r * Dp8)[c0 / 16] = make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void bq_queries_to_i8_kernel(const float* __restrict__ q, int nq, int dim, int Dp8,
                                        int8_t* __restrict__ dst) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= (int64_t)nq * Dp8) return;
  const int64_t r = t / Dp8;
  const int c = (int)(t - r * Dp8);
  // BinaryQuantizer.packBits: bit = v >= 0 (NaN -> 0)
  dst[t] = c < dim ? (q[r * dim + c] >= 0.0f ? (int8_t)1 : (int8_t)-1) : (int8_t)0;
}

cudaError_t launch_bq_words_to_i8(const uint64_t* words, int64_t n, int nwp, int dim, int Dp8, int8_t* dst,
                                  cudaStream_t st, bool zero_one) {
  if (n <= 0) return cudaSuccess;
  const int64_t total = n * (Dp8 / 16);
  bq_words_to_i8_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(words, n, nwp, dim, Dp8,
                                                                         zero_one ? (int8_t)0 : (int8_t)-1, dst);
  return cudaGetLastError();
}

cudaError_t launch_bq_queries_to_i8(const float* q, int nq, int dim, int Dp8, int8_t* dst, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  const int64_t total = (int64_t)nq * Dp8;
  bq_queries_to_i8_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(q, nq, dim, Dp8, dst);
  return cudaGetLastError();
}

}  // namespace vx
