// ivfpq.cu -- IVF-PQ search: coarse routing, (query, list) grouping and the ADC list scan.
//
// Restates IvfIndex.pqSearch (vectors-ivf/.../IvfIndex.java:539-619):
//   route:  CentroidIndex.routeWithSpillDistances with gamma = 0 (CentroidIndex.java:89-211),
//           distances from VectorUtil.batchSquaredL2 / batchDotProduct
//           (PanamaVectorUtilSupport.java:5353-5397, 5547-5598), evaluated here in the same
//           lane order; the nprobe nearest lists by (distance asc, list id asc), which is the
//           set the reference's bounded max-heap keeps (it admits only d < root).
//   table:  ProductQuantizer.buildADCTable (ProductQuantizer.java:521-544) of the residual
//           q - c_list (EUCLIDEAN) or of q (dot metrics); for sub-vectors of <= 16 floats the
//           reference takes the scalar tail: res += diff * diff, two roundings, in order.
//   scan:   sum = table[0][code[0]] + table[1][code[1]] + ... sequentially in fp32
//           (IvfIndex.java:581-588); score = -sum (EUCLIDEAN) or q.c + sum.
// Everything on this path is fixed by the Java source, so scores are bit-identical.
//
// Work decomposition.  The nq * nprobe (query, list) pairs are bucketed by list so that
// consecutive CTAs scan the same list (its codes stay in L2).  A CTA builds one pair's
// 96 x 256 fp32 table in shared memory, then its 8 warps stream the list's codes (lane = row)
// through table gathers into warp-owned candidate buffers; the CTA writes the pair's best
// K keys and a final per-query merge combines the nprobe lists.
#include <algorithm>

#include "common.cuh"
#include "exact.cuh"
#include "ivfpq.h"
#include "select.cuh"

namespace vx {

namespace {

constexpr int kQG = 8;  // queries per routing block

__device__ __forceinline__ float reduce_add8_local(const float* l) {
  float even = __fadd_rn(__fadd_rn(l[4], l[0]), __fadd_rn(l[6], l[2]));
  float odd = __fadd_rn(__fadd_rn(l[5], l[1]), __fadd_rn(l[7], l[3]));
  return __fadd_rn(even, odd);
}

// Serial restatements (one thread) of squareDistance / dotProduct over sub-vectors
// (PanamaVectorUtilSupport.java:208-343).
__device__ float serial_sqdist(const float* a, const float* b, int len) {
  float res = 0.0f;
  int i = 0;
  if (len > 16) {
    const int limit = len & ~7;
    float acc[4][8];
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
      for (int j = 0; j < 8; j++) acc[u][j] = 0.0f;
    int p = 0;
    for (; p < limit - 24; p += 32)
      for (int u = 0; u < 4; u++)
        for (int j = 0; j < 8; j++) {
          float d = __fsub_rn(a[p + 8 * u + j], b[p + 8 * u + j]);
          acc[u][j] = __fmaf_rn(d, d, acc[u][j]);
        }
    for (; p < limit; p += 8)
      for (int j = 0; j < 8; j++) {
        float d = __fsub_rn(a[p + j], b[p + j]);
        acc[0][j] = __fmaf_rn(d, d, acc[0][j]);
      }
    float s[8];
    for (int j = 0; j < 8; j++) s[j] = __fadd_rn(__fadd_rn(acc[0][j], acc[1][j]), __fadd_rn(acc[2][j], acc[3][j]));
    res = __fadd_rn(res, reduce_add8_local(s));
    i = limit;
  }
  for (; i < len; i++) {
    float d = __fsub_rn(a[i], b[i]);
    res = __fadd_rn(res, __fmul_rn(d, d));
  }
  return res;
}
__device__ float serial_dot(const float* a, const float* b, int len) {
  float res = 0.0f;
  int i = 0;
  if (len > 16) {
    const int limit = len & ~7;
    float acc[4][8];
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
      for (int j = 0; j < 8; j++) acc[u][j] = 0.0f;
    int p = 0;
    for (; p < limit - 24; p += 32)
      for (int u = 0; u < 4; u++)
        for (int j = 0; j < 8; j++) acc[u][j] = __fmaf_rn(a[p + 8 * u + j], b[p + 8 * u + j], acc[u][j]);
    for (; p < limit; p += 8)
      for (int j = 0; j < 8; j++) acc[0][j] = __fmaf_rn(a[p + j], b[p + j], acc[0][j]);
    float s[8];
    for (int j = 0; j < 8; j++) s[j] = __fadd_rn(__fadd_rn(acc[0][j], acc[1][j]), __fadd_rn(acc[2][j], acc[3][j]));
    res = __fadd_rn(res, reduce_add8_local(s));
    i = limit;
  }
  for (; i < len; i++) res = __fmaf_rn(a[i], b[i], res);
  return res;
}

// Distances from kQG queries to centroids [c_begin, nlist); one thread per centroid row.
// EUCLIDEAN: matVecSquaredL2; otherwise -matVecDot (queries already normalised for COSINE).
__global__ void __launch_bounds__(256) route_dist_kernel(const float* __restrict__ queries, int nq,
                                                         int dim, const float* __restrict__ cent,
                                                         int nlist, int metric,
                                                         float* __restrict__ dist, int c_begin) {
  extern __shared__ float s_q[];  // [kQG][dim]
  const int q0 = blockIdx.x * kQG;
  const int nqg = min(kQG, nq - q0);
  for (int i = threadIdx.x; i < kQG * dim; i += blockDim.x) {
    const int g = i / dim;
    s_q[i] = g < nqg ? queries[(size_t)(q0 + g) * dim + (i % dim)] : 0.0f;
  }
  __syncthreads();
  const int group = nlist & ~3;
  const int limit = dim & ~7;
  const bool l2 = metric == kEuclidean;
  for (int c = c_begin + threadIdx.x; c < nlist; c += blockDim.x) {
    const float* row = cent + (size_t)c * dim;
    if (c < group) {
      float acc[kQG][8];
#pragma unroll
      for (int g = 0; g < kQG; g++)
#pragma unroll
        for (int j = 0; j < 8; j++) acc[g][j] = 0.0f;
      for (int i = 0; i < limit; i += 8) {
        float r[8];
        if ((dim & 3) == 0) {
          const float4 r0 = *reinterpret_cast<const float4*>(row + i);
          const float4 r1 = *reinterpret_cast<const float4*>(row + i + 4);
          r[0] = r0.x; r[1] = r0.y; r[2] = r0.z; r[3] = r0.w;
          r[4] = r1.x; r[5] = r1.y; r[6] = r1.z; r[7] = r1.w;
        } else {
#pragma unroll
          for (int j = 0; j < 8; j++) r[j] = row[i + j];
        }
#pragma unroll
        for (int g = 0; g < kQG; g++)
#pragma unroll
          for (int j = 0; j < 8; j++) {
            const float qv = s_q[g * dim + i + j];
            if (l2) {
              const float d = __fsub_rn(qv, r[j]);
              acc[g][j] = __fmaf_rn(d, d, acc[g][j]);
            } else {
              acc[g][j] = __fmaf_rn(qv, r[j], acc[g][j]);
            }
          }
      }
#pragma unroll
      for (int g = 0; g < kQG; g++) {
        float s = reduce_add8_local(acc[g]);
        for (int i = limit; i < dim; i++) {
          const float qv = s_q[g * dim + i];
          if (l2) {
            const float e = __fsub_rn(qv, row[i]);
            s = __fmaf_rn(e, e, s);
          } else {
            s = __fmaf_rn(qv, row[i], s);
          }
        }
        if (g < nqg) dist[(size_t)(q0 + g) * nlist + c] = l2 ? s : -s;
      }
    } else {
      for (int g = 0; g < nqg; g++) {
        const float s = l2 ? serial_sqdist(s_q + g * dim, row, dim) : serial_dot(s_q + g * dim, row, dim);
        dist[(size_t)(q0 + g) * nlist + c] = l2 ? s : -s;
      }
    }
  }
}

// Register-tiled form of the same arithmetic for the centroids in 4-row groups when the
// dimension is a multiple of 64: a block scores 64 queries x 32 centroids, dims staged
// through shared memory 64 at a time; each thread keeps 4 queries x 2 centroids x the 8
// accumulator lanes of matVecSquaredL2 / matVecDot (lane j takes dims j, j+8, ... in order,
// FMA for dot, subtract-then-FMA for L2), then sums the lanes in the reference's order.
constexpr int kRtQ = 64, kRtC = 32, kRtK = 64, kRtStride = kRtK + 4;

// 16-byte asynchronous global -> shared copy; src_bytes 0 writes zeros (rows past the end).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(smem_dst)),
               "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

// Stages one 64-dim chunk of the block's 64 query rows and 32 centroid rows.
__device__ __forceinline__ void route_stage(float* s_q, float* s_c, const float* __restrict__ queries, int nq,
                                            const float* __restrict__ cent, int ngroup, int dim, int q0, int c0,
                                            int k0) {
  for (int i = threadIdx.x; i < (kRtQ + kRtC) * (kRtK / 4); i += 256) {
    const int r = i / (kRtK / 4), v = i % (kRtK / 4);
    if (r < kRtQ) {
      const bool in = q0 + r < nq;
      cp_async16(s_q + r * kRtStride + 4 * v, queries + (in ? (size_t)(q0 + r) * dim + k0 + 4 * v : 0), in ? 16u : 0u);
    } else {
      const int rc = r - kRtQ;
      const bool in = c0 + rc < ngroup;
      cp_async16(s_c + rc * kRtStride + 4 * v, cent + (in ? (size_t)(c0 + rc) * dim + k0 + 4 * v : 0), in ? 16u : 0u);
    }
  }
  cp_async_commit();
}

// Packed pairs of fp32 lanes: each lane of sub / fma.rn.f32x2 is the IEEE single-precision
// operation with round-to-nearest, so a pair of accumulator lanes updated together gets the
// same bits as two scalar updates.
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float2 f2_unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}

template <bool kL2>
__global__ void __launch_bounds__(256, 2) route_tile_kernel(const float* __restrict__ queries, int nq, int dim,
                                                             const float* __restrict__ cent, int ngroup, int nlist,
                                                             float* __restrict__ dist) {
  extern __shared__ __align__(16) float s_route[];  // 2 x ([64][68] queries, [32][68] centroids)
  constexpr int kStage = (kRtQ + kRtC) * kRtStride;
  const int q0 = blockIdx.y * kRtQ, c0 = blockIdx.x * kRtC;
  const int tq = threadIdx.x >> 4, tc = threadIdx.x & 15;  // queries tq + 16a, centroids tc + 16b
  uint64_t acc[4][2][4];  // accumulator lanes (2p, 2p + 1) packed in acc[a][b][p]
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 2; b++)
#pragma unroll
      for (int p = 0; p < 4; p++) acc[a][b][p] = 0ull;
  route_stage(s_route, s_route + kRtQ * kRtStride, queries, nq, cent, ngroup, dim, q0, c0, 0);
  int buf = 0;
  for (int k0 = 0; k0 < dim; k0 += kRtK) {
    // the next chunk streams in while this one is scored (double buffer)
    if (k0 + kRtK < dim) {
      float* nb = s_route + (buf ^ 1) * kStage;
      route_stage(nb, nb + kRtQ * kRtStride, queries, nq, cent, ngroup, dim, q0, c0, k0 + kRtK);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const float* s_q = s_route + buf * kStage;
    const float* s_c = s_q + kRtQ * kRtStride;
#pragma unroll 4
    for (int kk = 0; kk < kRtK; kk += 4) {
      ulonglong2 qv[4], cv[2];  // dims (kk, kk + 1) and (kk + 2, kk + 3) as packed pairs
#pragma unroll
      for (int a = 0; a < 4; a++) qv[a] = *reinterpret_cast<const ulonglong2*>(s_q + (tq + 16 * a) * kRtStride + kk);
#pragma unroll
      for (int b = 0; b < 2; b++) cv[b] = *reinterpret_cast<const ulonglong2*>(s_c + (tc + 16 * b) * kRtStride + kk);
      const int pb = (kk & 4) >> 1;  // accumulator lanes 2 pb .. 2 pb + 3 take dims kk .. kk + 3
#pragma unroll
      for (int a = 0; a < 4; a++) {
#pragma unroll
        for (int b = 0; b < 2; b++) {
          if (kL2) {
            const uint64_t d0 = f2_sub(qv[a].x, cv[b].x), d1 = f2_sub(qv[a].y, cv[b].y);
            acc[a][b][pb] = f2_fma(d0, d0, acc[a][b][pb]);
            acc[a][b][pb + 1] = f2_fma(d1, d1, acc[a][b][pb + 1]);
          } else {
            acc[a][b][pb] = f2_fma(qv[a].x, cv[b].x, acc[a][b][pb]);
            acc[a][b][pb + 1] = f2_fma(qv[a].y, cv[b].y, acc[a][b][pb + 1]);
          }
        }
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
    buf ^= 1;
  }
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 2; b++) {
      const int q = q0 + tq + 16 * a, c = c0 + tc + 16 * b;
      if (q < nq && c < ngroup) {
        float lanes[8];
#pragma unroll
        for (int p = 0; p < 4; p++) {
          const float2 v = f2_unpack(acc[a][b][p]);
          lanes[2 * p] = v.x;
          lanes[2 * p + 1] = v.y;
        }
        const float sum = reduce_add8_local(lanes);
        dist[(size_t)q * nlist + c] = kL2 ? sum : -sum;
      }
    }
}

// COSINE routing normalises a copy of the query first: l2normalize
// (PanamaVectorUtilSupport.java:5178-5194).  One warp per query.
__global__ void l2normalize_kernel(const float* __restrict__ src, int nq, int dim,
                                   float* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  const int q = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (q >= nq) return;
  const float* v = src + (size_t)q * dim;
  float* o = dst + (size_t)q * dim;
  const float dotf = warp_dot(RowF32{v}, RowF32{v}, dim);
  const double sq = (double)dotf;
  float inv = 1.0f;
  bool scale = !(sq == 0.0) && !(fabsf(__fsub_rn((float)sq, 1.0f)) < 1e-5f);
  if (scale) inv = __fdiv_rn(1.0f, __double2float_rn(__dsqrt_rn(sq)));
  for (int i = lane; i < dim; i += 32) o[i] = scale ? __fmul_rn(v[i], inv) : v[i];
}

// nprobe nearest lists per query, ascending distance (ties: lower list id).
__global__ void __launch_bounds__(256) route_select_kernel(const float* __restrict__ dist, int nlist,
                                                           int nprobe, int32_t* __restrict__ lists) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int q = blockIdx.x;
  uint32_t cap = 1;
  while (cap < (uint32_t)nlist) cap <<= 1;
  uint64_t* s_keys = (uint64_t*)smem_raw;
  uint64_t* s_tmp = s_keys + cap;
  uint32_t* s_red = (uint32_t*)(s_tmp + cap);
  uint32_t* s_counter = s_red + 32;
  for (int c = threadIdx.x; c < nlist; c += blockDim.x)
    s_keys[c] = make_key(~float_order_bits(dist[(size_t)q * nlist + c]), (uint32_t)c);
  __syncthreads();
  uint32_t n = block_keep_top(s_keys, (uint32_t)nlist, (uint32_t)nprobe, s_tmp, s_red, s_counter);
  block_sort_desc(s_keys, n, cap);
  for (int i = threadIdx.x; i < nprobe; i += blockDim.x)
    lists[(size_t)q * nprobe + i] = (uint32_t)i < n ? (int32_t)key_id(s_keys[i]) : -1;
}

// Copies caller-routed list ids, replacing ids outside [-1, nlist) by -1 and counting them.
__global__ void copy_lists_kernel(const int32_t* __restrict__ src, int n, int nlist, int32_t* __restrict__ dst,
                                  int32_t* __restrict__ bad) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int32_t l = src[i];
  const bool ok = l >= -1 && l < nlist;
  dst[i] = ok ? l : -1;
  if (!ok) atomicAdd(bad, 1);
}

// A pair takes part when its list is routed (id >= 0) and holds rows on this device (a
// list-sharded index keeps only its own lists' rows).
__device__ __forceinline__ bool pair_live(const int32_t* lists, const int64_t* list_off, int i) {
  const int32_t l = lists[i];
  return l >= 0 && list_off[l + 1] > list_off[l];
}

__global__ void pair_hist_kernel(const int32_t* __restrict__ lists, const int64_t* __restrict__ list_off,
                                 int npairs, int32_t* __restrict__ counts) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < npairs && pair_live(lists, list_off, i)) atomicAdd(&counts[lists[i]], 1);
}

// Exclusive scan of nlist counts (single block), also resets the scatter cursors.
__global__ void pair_scan_kernel(const int32_t* __restrict__ counts, int nlist,
                                 int32_t* __restrict__ offsets, int32_t* __restrict__ cursor) {
  __shared__ int32_t s_part[1024];
  const int per = (nlist + blockDim.x - 1) / blockDim.x;
  const int b = threadIdx.x * per;
  int32_t sum = 0;
  for (int i = b; i < b + per && i < nlist; i++) sum += counts[i];
  s_part[threadIdx.x] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t run = 0;
    for (int t = 0; t < (int)blockDim.x; t++) {
      int32_t v = s_part[t];
      s_part[t] = run;
      run += v;
    }
  }
  __syncthreads();
  int32_t run = s_part[threadIdx.x];
  for (int i = b; i < b + per && i < nlist; i++) {
    offsets[i] = run;
    cursor[i] = run;
    run += counts[i];
  }
  if (threadIdx.x == blockDim.x - 1) offsets[nlist] = run;
}

__global__ void pair_scatter_kernel(const int32_t* __restrict__ lists, const int64_t* __restrict__ list_off,
                                    int npairs, int32_t* __restrict__ cursor, int32_t* __restrict__ pairs) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < npairs && pair_live(lists, list_off, i)) pairs[atomicAdd(&cursor[lists[i]], 1)] = i;
}

// Warp-owned candidate buffer in shared memory: all 32 lanes offer one key each.
template <int R>
struct WarpStream {
  uint64_t* buf;
  uint32_t cnt;
  uint64_t thr;
  __device__ __forceinline__ void offer32(uint64_t key, bool valid, int C, int K) {
    const int lane = threadIdx.x & 31;
    const bool pass = valid && key > thr;
    const unsigned m = __ballot_sync(0xFFFFFFFFu, pass);
    if (pass) buf[cnt + __popc(m & ((1u << lane) - 1u))] = key;
    cnt += __popc(m);
    if (cnt > (uint32_t)(C - 32)) {
      __syncwarp();
      warp_compact_one<R>(buf, cnt, (uint32_t)K, thr, cnt);
      __syncwarp();
    }
  }
};

// PQVectors' score of a row from its ADC sum (PQVectors.java:113-191): DOT_PRODUCT
// max((1 + sum) / 2, 0); EUCLIDEAN 1 / (1 + sum); MAXIMUM_INNER_PRODUCT
// scaleMaxInnerProductScore(sum); COSINE sum / (|q - gc| * (float) sqrt(vsq)) -> max((1 + cos) / 2, 0),
// 0 when either norm is 0.  No fused multiply-add, as in Java.
__device__ __forceinline__ float pq_flat_score(int metric, float sum, float qn, float vsq) {
  float h;
  switch (metric) {
    case kEuclidean: return __fdiv_rn(1.0f, __fadd_rn(1.0f, sum));
    case kMaxInnerProduct: return scale_mip(sum);
    case kCosine: {
      const float vn = (float)sqrt((double)vsq);
      if (qn == 0.0f || vn == 0.0f) return 0.0f;
      h = __fdiv_rn(__fadd_rn(1.0f, __fdiv_rn(sum, __fmul_rn(qn, vn))), 2.0f);
      break;
    }
    default: h = __fdiv_rn(__fadd_rn(1.0f, sum), 2.0f); break;
  }
  return h >= 0.0f ? h : (h != h ? h : 0.0f);  // Math.max(h, 0f)
}

template <int R>
__global__ void __launch_bounds__(256) adc_scan_kernel(AdcArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int C = 32 * R;
  float* s_lut = (float*)smem_raw;                            // [M][Ks]
  float* s_res = s_lut + (size_t)a.M * a.Ks;                  // [dim]
  uint64_t* s_wbuf = (uint64_t*)(((uintptr_t)(s_res + a.dim) + 15) & ~(uintptr_t)15);  // [nwarps][C]
  uint64_t* s_merge = s_wbuf + (size_t)nwarps * C;            // [2][mcap]
  const uint32_t mcap = (uint32_t)(nwarps * a.K);
  uint32_t* s_red = (uint32_t*)(s_merge + 2 * (size_t)mcap);
  uint32_t* s_counter = s_red + 32;
  __shared__ float s_base;

  const int64_t live = *a.pair_count;  // pairs grouped by list (routed, non-empty lists)
  for (int64_t w = blockIdx.x; w < live; w += gridDim.x) {
    const int32_t pair = a.pairs[w];
    const int q = pair / a.nprobe;
    const int p = pair % a.nprobe;
    const int l = a.lists[pair];
    const float* qv = a.queries + (size_t)q * a.dim;
    const float* c = a.cent + (size_t)l * a.dim;
    const bool l2 = a.metric == kEuclidean;
    __syncthreads();  // previous pair fully consumed the shared buffers
    // IVF residual q - c for EUCLIDEAN (IvfIndex.java:570); PQ as a flat quantizer centres the
    // query on the global centroid for every metric (buildADCTable's subInPlace)
    for (int i = threadIdx.x; i < a.dim; i += blockDim.x)
      s_res[i] = (l2 || a.pq_flat) ? __fsub_rn(qv[i], c[i]) : qv[i];
    if (warp == 0) {
      float base = 0.0f;
      if (!l2 && a.metric != kCosine) base = warp_dot(RowF32{qv}, RowF32{c}, a.dim);
      if (lane == 0) s_base = base;
    }
    __syncthreads();
    const int entries = a.M * a.Ks;
    for (int e = threadIdx.x; e < entries; e += blockDim.x) {
      const int m = e / a.Ks, cc = e - m * a.Ks;
      const int sub = a.sub[2 * m], off = a.sub[2 * m + 1];
      const float* cb = a.codebooks + a.cb_off[m] + (size_t)cc * sub;
      s_lut[e] = l2 ? serial_sqdist(s_res + off, cb, sub) : serial_dot(s_res + off, cb, sub);
    }
    __syncthreads();
    const float base = s_base;
    WarpStream<R> ws{s_wbuf + (size_t)warp * C, 0u, 0ull};
    const int64_t b = a.list_off[l], e = a.list_off[l + 1];
    for (int64_t r0 = b + (int64_t)warp * 32; r0 < e; r0 += (int64_t)nwarps * 32) {
      const int64_t r = r0 + lane;
      const bool valid = r < e;
      uint64_t key = 0;
      if (valid) {
        const uint8_t* code = a.codes + r * (int64_t)a.Mp;
        float sum = 0.0f;
        int m = 0;
        for (; m + 16 <= a.M; m += 16) {
          const uint4 v = *reinterpret_cast<const uint4*>(code + m);
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int t = 0; t < 16; t++) {
            const uint32_t cv = (w4[t >> 2] >> (8 * (t & 3))) & 0xFFu;
            sum = __fadd_rn(sum, s_lut[(m + t) * a.Ks + cv]);
          }
        }
        for (; m < a.M; m++) sum = __fadd_rn(sum, s_lut[m * a.Ks + code[m]]);
        const float score = a.pq_flat ? pq_flat_score(a.metric, sum, a.qnorm ? a.qnorm[q] : 0.0f,
                                                      a.rnorm ? a.rnorm[r] : 0.0f)
                                      : (l2 ? -sum : __fadd_rn(base, sum));
        key = float_key(score, (uint32_t)a.ordinals[r]);
      }
      ws.offer32(key, valid, C, a.K);
    }
    // Shrink each warp's buffer to K and gather all warps' survivors.
    __syncwarp();
    if (ws.cnt > (uint32_t)a.K) warp_compact_one<R>(ws.buf, ws.cnt, (uint32_t)a.K, ws.thr, ws.cnt);
    __syncwarp();
    if (lane == 0) s_red[warp] = ws.cnt;
    __syncthreads();
    uint32_t at = 0;
    for (int i = 0; i < warp; i++) at += s_red[i];
    uint32_t total = 0;
    for (int i = 0; i < nwarps; i++) total += s_red[i];
    for (uint32_t i = lane; i < ws.cnt; i += 32) s_merge[at + i] = ws.buf[i];
    __syncthreads();
    const uint32_t n = block_keep_top(s_merge, total, (uint32_t)a.K, s_merge + mcap, s_red, s_counter);
    const size_t sidx = (size_t)p * a.nq + q;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) a.out[sidx * a.K + i] = s_merge[i];
    if (threadIdx.x == 0) a.out_cnt[sidx] = n;
  }
}

// ---------------------------------------------------------------------------------------
// Grouped ADC scan (8-dimensional subspaces, 256 centroids, M a multiple of 16).
//
// A CTA takes a group of up to four (query, list) pairs that probe the same list.  The
// subspaces are processed in chunks of 16: for each chunk the CTA builds the four queries'
// tables, interleaved as table[m][code] = float4(query 0..3) (64 KB), with the codebook row
// of (m, code) read once for all four queries; then every thread adds the chunk's 16 entries
// of each of its rows into per-(row, query) running sums held in registers.  Chunks run in
// subspace order, so each sum is table[0][c0] + table[1][c1] + ... in fp32 exactly as
// IvfIndex.java:581-588 adds it, and each table entry is ProductQuantizer.buildADCTable's
// scalar tail for 8-float sub-vectors (ProductQuantizer.java:521-544,
// PanamaVectorUtilSupport.java:285-296).  One 16-byte shared load serves four queries.
// Keys go to per-warp, per-query candidate buffers; a query's best key so far over all its
// lists (its floor, raised by atomicMax) bounds admission in every later group.
constexpr int kAdcThreads = 256;
constexpr int kAdcWarps = kAdcThreads / 32;
constexpr int kMChunk = 16;  // subspaces per table chunk
constexpr int kRowsPerThread = 12;
constexpr int kRowsPerPass = kAdcThreads * kRowsPerThread;

// Lists in `order` (null: by id), each cut into groups of up to wmax consecutive pairs; with
// rmax > 0 (the IVF-flat scan) a list longer than rmax rows also into row parts of rmax rows,
// every pair group once per part: group = (first pair, pairs | part << 8).
__global__ void make_groups_kernel(const int32_t* __restrict__ counts, const int32_t* __restrict__ offsets,
                                   const int32_t* __restrict__ order, int nlist, int wmax,
                                   const int64_t* __restrict__ list_off, int rmax, int2* __restrict__ groups,
                                   int32_t* __restrict__ ngroups) {
  __shared__ uint32_t s_red[32];
  __shared__ int32_t s_carry;
  if (threadIdx.x == 0) s_carry = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int base = 0; base < nlist; base += blockDim.x) {
    const int i = base + threadIdx.x;
    const int l = i < nlist ? (order ? order[i] : i) : 0;
    const int c = i < nlist ? counts[l] : 0;
    const int parts = (rmax > 0 && i < nlist) ? max(1, (int)((list_off[l + 1] - list_off[l] + rmax - 1) / rmax)) : 1;
    const int g = (c + wmax - 1) / wmax * parts;
    int incl = g;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) s_red[warp] = (uint32_t)incl;
    __syncthreads();
    int before = s_carry, total = 0;
    for (int i = 0; i < nw; i++) {
      before += i < warp ? (int)s_red[i] : 0;
      total += (int)s_red[i];
    }
    const int first = before + incl - g;
    for (int j = 0; j < g; j++) {
      const int run = j / parts, part = j - run * parts;
      groups[first + j] = make_int2(offsets[l] + run * wmax, min(wmax, c - run * wmax) | (part << 8));
    }
    __syncthreads();
    if (threadIdx.x == 0) s_carry += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) *ngroups = s_carry;
}

// Table entries of subspace m for code c and the group's (up to) four queries.
template <bool kDot>
__device__ __forceinline__ float4 group_entry(const float* __restrict__ cb, const float* s_res, int dim, int m) {
  const float4 b0 = *reinterpret_cast<const float4*>(cb);
  const float4 b1 = *reinterpret_cast<const float4*>(cb + 4);
  const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
  float out[kAdcGroupQ];
#pragma unroll
  for (int g = 0; g < kAdcGroupQ; g++) {
    const float4 r0 = *reinterpret_cast<const float4*>(s_res + g * dim + 8 * m);
    const float4 r1 = *reinterpret_cast<const float4*>(s_res + g * dim + 8 * m + 4);
    const float rv[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
    float res = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      if (kDot) {
        res = __fmaf_rn(rv[i], bv[i], res);
      } else {
        const float d = __fsub_rn(rv[i], bv[i]);
        res = __fadd_rn(res, __fmul_rn(d, d));
      }
    }
    out[g] = res;
  }
  return make_float4(out[0], out[1], out[2], out[3]);
}

template <bool kDot, int R>
__global__ void __launch_bounds__(kAdcThreads, 2) adc_group_kernel(AdcArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int C = 32 * R;
  float4* s_lut = reinterpret_cast<float4*>(smem_raw);                       // [kMChunk][256]
  float* s_res = reinterpret_cast<float*>(s_lut + kMChunk * 256);            // [4][dim]
  uint64_t* s_wbuf = reinterpret_cast<uint64_t*>(s_res + kAdcGroupQ * a.dim);  // [warps][4][C]
  uint64_t* s_mrg = s_wbuf + (size_t)kAdcWarps * kAdcGroupQ * C;              // [4][C]
  __shared__ uint32_t s_wcnt[kAdcWarps][kAdcGroupQ];
  __shared__ int s_q[kAdcGroupQ], s_p[kAdcGroupQ];
  __shared__ float s_base[kAdcGroupQ];
  __shared__ float s_qn[kAdcGroupQ];
  __shared__ uint64_t s_floor[kAdcGroupQ];
  __shared__ int s_gi;
  const int ng = a.ngroups[0];
  const int nchunks = a.M / kMChunk;
  for (;;) {
    __syncthreads();  // the previous group is finished with every shared buffer (and s_gi)
    if (threadIdx.x == 0) s_gi = atomicAdd(a.ngroups + 1, 1);  // longest lists first
    __syncthreads();
    const int gi = s_gi;
    if (gi >= ng) break;
    const int2 grp = a.groups[gi];
    const int npq = grp.y;  // pairs in this group (1..4)
    if (threadIdx.x < kAdcGroupQ) {
      const int g = threadIdx.x;
      int q = -1, p = 0;
      uint64_t f = 0;
      if (g < npq) {
        const int32_t pair = a.pairs[grp.x + g];
        q = pair / a.nprobe;
        p = pair - q * a.nprobe;
        f = a.floor[q];
      }
      s_q[g] = q;
      s_p[g] = p;
      s_floor[g] = f;
      s_qn[g] = (g < npq && a.qnorm) ? a.qnorm[q] : 0.0f;
    }
    __syncthreads();
    const int l = a.lists[(size_t)s_q[0] * a.nprobe + s_p[0]];
    const float* c = a.cent + (size_t)l * a.dim;
    for (int i = threadIdx.x; i < kAdcGroupQ * a.dim; i += kAdcThreads) {
      const int g = i / a.dim, d = i - g * a.dim;
      float v = 0.0f;
      if (g < npq) {
        const float qv = a.queries[(size_t)s_q[g] * a.dim + d];
        // IvfIndex.java:570 residual; PQ as a flat quantizer: the query minus the global centroid
        v = (kDot && !a.pq_flat) ? qv : __fsub_rn(qv, c[d]);
      }
      s_res[i] = v;
    }
    if (kDot && warp < kAdcGroupQ) {
      float base = 0.0f;
      if (warp < npq && a.metric != kCosine)
        base = warp_dot(RowF32{a.queries + (size_t)s_q[warp] * a.dim}, RowF32{c}, a.dim);
      if (lane == 0) s_base[warp] = base;
    }
    // per-warp streams of the group's queries, seeded with the queries' floors
    uint32_t wcnt[kAdcGroupQ];
    uint64_t wthr[kAdcGroupQ];
#pragma unroll
    for (int g = 0; g < kAdcGroupQ; g++) wcnt[g] = 0;
    __syncthreads();
#pragma unroll
    for (int g = 0; g < kAdcGroupQ; g++) wthr[g] = s_floor[g] > 0 ? s_floor[g] - 1 : 0ull;
    const int64_t b = a.list_off[l], e = a.list_off[l + 1];
    for (int64_t pass0 = b; pass0 < e; pass0 += kRowsPerPass) {
      float ps[kRowsPerThread][kAdcGroupQ];
#pragma unroll
      for (int j = 0; j < kRowsPerThread; j++)
#pragma unroll
        for (int g = 0; g < kAdcGroupQ; g++) ps[j][g] = 0.0f;
      for (int ch = 0; ch < nchunks; ch++) {
        __syncthreads();  // readers of the previous chunk are done
        {
          const int code = threadIdx.x;  // 256 threads <-> 256 centroids
#pragma unroll 1
          for (int ml = 0; ml < kMChunk; ml++) {
            const int m = ch * kMChunk + ml;
            const float* cb = a.codebooks + a.cb_off[m] + (size_t)code * 8;
            s_lut[ml * 256 + code] = group_entry<kDot>(cb, s_res, a.dim, m);
          }
        }
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kRowsPerThread; j++) {
          const int64_t r = pass0 + threadIdx.x + (int64_t)kAdcThreads * j;
          if (r < e) {
            const uint4 cv = *reinterpret_cast<const uint4*>(a.codes + r * (int64_t)a.Mp + ch * kMChunk);
            const uint32_t w4[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
            for (int ml = 0; ml < kMChunk; ml++) {
              const uint32_t code = (w4[ml >> 2] >> (8 * (ml & 3))) & 0xFFu;
              const float4 t = s_lut[ml * 256 + code];
              ps[j][0] = __fadd_rn(ps[j][0], t.x);
              ps[j][1] = __fadd_rn(ps[j][1], t.y);
              ps[j][2] = __fadd_rn(ps[j][2], t.z);
              ps[j][3] = __fadd_rn(ps[j][3], t.w);
            }
          }
        }
      }
      // keys of this pass's rows into the per-warp streams
#pragma unroll
      for (int j = 0; j < kRowsPerThread; j++) {
        const int64_t r = pass0 + threadIdx.x + (int64_t)kAdcThreads * j;
        const bool in = r < e;
        const uint32_t ord = in ? (uint32_t)a.ordinals[r] : 0u;
        const float vsq = (in && a.rnorm) ? a.rnorm[r] : 0.0f;
#pragma unroll
        for (int g = 0; g < kAdcGroupQ; g++) {
          const float score = a.pq_flat ? pq_flat_score(a.metric, ps[j][g], s_qn[g], vsq)
                                        : (kDot ? __fadd_rn(s_base[g], ps[j][g]) : -ps[j][g]);
          const uint64_t key = float_key(score, ord);
          const bool pass = in && g < npq && key > wthr[g];
          const unsigned mk = __ballot_sync(0xFFFFFFFFu, pass);
          uint64_t* buf = s_wbuf + ((size_t)warp * kAdcGroupQ + g) * C;
          if (pass) buf[wcnt[g] + __popc(mk & ((1u << lane) - 1u))] = key;
          wcnt[g] += __popc(mk);
          if (wcnt[g] > (uint32_t)(C - 32)) {
            __syncwarp();
            warp_compact_one<R>(buf, wcnt[g], (uint32_t)a.K, wthr[g], wcnt[g]);
            __syncwarp();
          }
        }
      }
    }
    // each warp shrinks its buffers to K and publishes the counts
#pragma unroll
    for (int g = 0; g < kAdcGroupQ; g++) {
      uint64_t* buf = s_wbuf + ((size_t)warp * kAdcGroupQ + g) * C;
      __syncwarp();
      if (wcnt[g] > (uint32_t)a.K) warp_compact_one<R>(buf, wcnt[g], (uint32_t)a.K, wthr[g], wcnt[g]);
      __syncwarp();
      if (lane == 0) s_wcnt[warp][g] = wcnt[g];
    }
    __syncthreads();
    // warp g merges query g's buffers (each <= K keys) into its K best; C >= 2K keeps every
    // append within the buffer
    if (warp < npq) {
      const int g = warp;
      uint64_t* mrg = s_mrg + (size_t)g * C;
      uint32_t n = 0;
      uint64_t thr = 0;
      for (int w = 0; w < kAdcWarps; w++) {
        const uint32_t cw = s_wcnt[w][g];
        const uint64_t* src = s_wbuf + ((size_t)w * kAdcGroupQ + g) * C;
        for (uint32_t i = lane; i < cw; i += 32) mrg[n + i] = src[i];
        __syncwarp();
        n += cw;
        if (n > (uint32_t)(C - a.K)) {
          warp_compact_one<R>(mrg, n, (uint32_t)a.K, thr, n);
          __syncwarp();
        }
      }
      if (n > (uint32_t)a.K) {
        warp_compact_one<R>(mrg, n, (uint32_t)a.K, thr, n);
        __syncwarp();
      } else if (n == (uint32_t)a.K) {
        uint64_t mn = ~0ull;
        for (uint32_t i = lane; i < n; i += 32) mn = mrg[i] < mn ? mrg[i] : mn;
        thr = warp_min_u64(mn);
      }
      const int q = s_q[g];
      const size_t sidx = (size_t)s_p[g] * a.nq + q;
      for (uint32_t i = lane; i < n; i += 32) a.out[sidx * a.K + i] = mrg[i];
      if (lane == 0) {
        a.out_cnt[sidx] = n;
        if (n == (uint32_t)a.K) atomicMax((unsigned long long*)&a.floor[q], (unsigned long long)thr);
      }
    }
  }
}


// ---------------------------------------------------------------------------------------
// IVF-flat list scan: IvfIndex.search without PQ (IvfIndex.java:170-226) scores a probed
// cluster's rows in batches of BATCH_ROWS = 64 through VectorUtil.batchSquaredL2 /
// batchDotProduct (scanPartitionBulk, :244-277).  Inside a batch the rows in groups of four
// take matVecSquaredL2 / matVecDot's arithmetic -- eight lane accumulators (lane j: dims j,
// j + 8, ... below dim & ~7, subtract-then-FMA or FMA), summed as reduce_add8_local, then the
// remaining dims folded in with FMA -- exactly route_tile_kernel's arithmetic; the batch's last
// count % 4 rows go through squareDistance / dotProduct instead (flat_tail_kernel).  Score:
// -d (EUCLIDEAN), dot (DOT_PRODUCT, MAXIMUM_INNER_PRODUCT) or
// (float)(dot / sqrt((double)|q|^2 * (double)|v|^2)) (COSINE, norms by dotProduct).
//
// One CTA takes up to 64 (query, list) pairs of one list: 32-row tiles of the list against the
// group's queries, dims staged 64 at a time (cp.async, double buffer, zero past dim & ~7);
// per-query candidate buffers in shared memory, shrunk to K between tiles; a query's best K
// over earlier lists (its floor) bounds admission, as in the ADC scan.
// ---------------------------------------------------------------------------------------
constexpr int kFlGroup = kRtQ;  // pairs per group (64)

// Rows [n][dim] (stride src_stride, optionally gathered through map) -> [n][Dp], zero padded.
__global__ void pad_rows_kernel(const float* __restrict__ src, int64_t n, int dim, int64_t src_stride,
                                const int32_t* __restrict__ map, int Dp, float* __restrict__ dst) {
  const int64_t total = n * (int64_t)Dp;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / Dp;
    const int d = (int)(i - r * Dp);
    const int64_t s = map ? (int64_t)map[r] : r;
    dst[i] = d < dim ? src[s * src_stride + d] : 0.0f;
  }
}

// dotProduct(v, v) (PanamaVectorUtilSupport.java:204-230) of every padded row; one warp a row.
__global__ void row_norms_kernel(const float* __restrict__ rows, int64_t n, int dim, int Dp, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (w >= n) return;
  const float* v = rows + w * Dp;
  const float d = warp_dot(RowF32{v}, RowF32{v}, dim);
  if (lane == 0) out[w] = d;
}

// The last batch's trailing count % 4 rows of every live pair's list, scored with
// squareDistance / dotProduct (raw: distance or dot); one warp per (pair slot, row).
template <bool kL2>
__global__ void flat_tail_kernel(FlatListArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t slot = w / 3;
  const int t = (int)(w - slot * 3);
  if (slot >= *a.pair_count) return;
  const int32_t pair = a.pairs[slot];
  const int q = pair / a.nprobe;
  const int l = a.lists[pair];
  const int64_t b = a.list_off[l];
  const int n = (int)(a.list_off[l + 1] - b);
  const int last = ((n - 1) / 64) * 64;
  const int r = last + ((n - last) & ~3) + t;
  if (r >= n) return;
  const float* qv = a.queries + (size_t)q * a.Dp;
  const float* x = a.rows + (size_t)(b + r) * a.Dp;
  const float s = kL2 ? warp_sqdist(RowF32{qv}, RowF32{x}, a.dim) : warp_dot(RowF32{qv}, RowF32{x}, a.dim);
  if (lane == 0) a.tail[slot * 3 + t] = s;
}

// Stages dims [k0, k0 + 64) of the group's queries and of rows r0 .. r0 + 31 of the list.
__device__ __forceinline__ void flat_stage(float* s_q, float* s_c, const FlatListArgs& a, const int* s_query,
                                           int npq, const float* rows, int r0, int n, int k0, int limit) {
  for (int i = threadIdx.x; i < (kRtQ + kRtC) * (kRtK / 4); i += 256) {
    const int r = i / (kRtK / 4), v = i % (kRtK / 4);
    const int d = k0 + 4 * v;
    if (r < kRtQ) {
      const bool in = r < npq && d < limit;
      cp_async16(s_q + r * kRtStride + 4 * v, a.queries + (in ? (size_t)s_query[r] * a.Dp + d : 0), in ? 16u : 0u);
    } else {
      const int rc = r - kRtQ;
      const bool in = r0 + rc < n && d < limit;
      cp_async16(s_c + rc * kRtStride + 4 * v, rows + (in ? (size_t)(r0 + rc) * a.Dp + d : 0), in ? 16u : 0u);
    }
  }
  cp_async_commit();
}

// One staged 64-dim chunk into the accumulators of the first NU 16-query slices (the rest of
// the group's 64 slots hold no pair), routing's 8-lane batched arithmetic on packed lane pairs.
template <bool kL2, int NU>
__device__ __forceinline__ void flat_chunk(const float* sq, const float* sc, int tq, int tc, uint64_t (&acc)[4][2][4]) {
#pragma unroll 4
  for (int kk = 0; kk < kRtK; kk += 4) {
    ulonglong2 qv[NU], cv[2];
#pragma unroll
    for (int u = 0; u < NU; u++) qv[u] = *reinterpret_cast<const ulonglong2*>(sq + (tq + 16 * u) * kRtStride + kk);
#pragma unroll
    for (int v = 0; v < 2; v++) cv[v] = *reinterpret_cast<const ulonglong2*>(sc + (tc + 16 * v) * kRtStride + kk);
    const int pb = (kk & 4) >> 1;
#pragma unroll
    for (int u = 0; u < NU; u++)
#pragma unroll
      for (int v = 0; v < 2; v++) {
        if (kL2) {
          const uint64_t d0 = f2_sub(qv[u].x, cv[v].x), d1 = f2_sub(qv[u].y, cv[v].y);
          acc[u][v][pb] = f2_fma(d0, d0, acc[u][v][pb]);
          acc[u][v][pb + 1] = f2_fma(d1, d1, acc[u][v][pb + 1]);
        } else {
          acc[u][v][pb] = f2_fma(qv[u].x, cv[v].x, acc[u][v][pb]);
          acc[u][v][pb + 1] = f2_fma(qv[u].y, cv[v].y, acc[u][v][pb + 1]);
        }
      }
  }
}

template <bool kL2, int R>
__global__ void __launch_bounds__(256, 2) flat_list_kernel(FlatListArgs a) {
  extern __shared__ __align__(16) float s_flat[];
  constexpr int kStage = (kRtQ + kRtC) * kRtStride;
  constexpr int C = 32 * R;  // key slots per query; a tile adds at most 32
  uint64_t* keys = reinterpret_cast<uint64_t*>(s_flat + 2 * kStage);  // [64][C]
  __shared__ int s_query[kFlGroup], s_probe[kFlGroup], s_slot[kFlGroup];
  __shared__ float s_qn[kFlGroup];
  __shared__ uint64_t s_thr[kFlGroup];
  __shared__ uint32_t s_cnt[kFlGroup];
  const int tq = threadIdx.x >> 4, tc = threadIdx.x & 15;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool cosine = a.metric == kCosine;
  __shared__ int s_gi;
  const int ng = a.ngroups[0];
  const int limit = a.dim & ~7;
  for (;;) {
    __syncthreads();  // the previous group is done with every shared buffer (and s_gi)
    if (threadIdx.x == 0) s_gi = atomicAdd(a.ngroups + 1, 1);  // longest lists first
    __syncthreads();
    const int gi = s_gi;
    if (gi >= ng) break;
    const int2 grp = a.groups[gi];
    const int npq = grp.y & 0xFF;
    const int part = grp.y >> 8;  // row part of a list longer than a.rmax rows
    if (threadIdx.x < kFlGroup) {
      const int g = threadIdx.x;
      int q = 0, p = 0;
      uint64_t f = 0;
      if (g < npq) {
        const int32_t pair = a.pairs[grp.x + g];
        q = pair / a.nprobe;
        p = pair - q * a.nprobe;
        f = a.floor ? a.floor[q] : 0ull;
      }
      s_query[g] = q;
      s_probe[g] = p;
      s_slot[g] = grp.x + g;
      s_qn[g] = (g < npq && cosine) ? a.qnorm[q] : 0.0f;
      s_thr[g] = f > 0 ? f - 1 : 0ull;  // keys >= the query's floor stay admissible
      s_cnt[g] = 0;
    }
    __syncthreads();
    const int l = a.lists[(size_t)s_query[0] * a.nprobe + s_probe[0]];
    const int64_t b = a.list_off[l];
    const int n = (int)(a.list_off[l + 1] - b);
    const int last = ((n - 1) / 64) * 64;
    const int tail_begin = last + ((n - last) & ~3);
    const float* rows = a.rows + (size_t)b * a.Dp;
    const int nu = npq > 48 ? 4 : (npq + 15) / 16;  // 16-query slices holding pairs
    // this group's rows: the whole list, or part `part` of rmax rows (a multiple of 64, so that
    // a 32-row tile never straddles two parts and the last 64-row batch lies in the last part)
    const bool parted = a.rmax > 0 && n > a.rmax;
    const int r_lo = parted ? part * a.rmax : 0;
    const int r_hi = parted ? min(n, r_lo + a.rmax) : n;
    for (int r0 = r_lo; r0 < r_hi; r0 += kRtC) {
      uint64_t acc[4][2][4];  // accumulator lanes (2p, 2p + 1) packed in acc[.][.][p]
#pragma unroll
      for (int u = 0; u < 4; u++)
#pragma unroll
        for (int v = 0; v < 2; v++)
#pragma unroll
          for (int p = 0; p < 4; p++) acc[u][v][p] = 0ull;
      if (limit > 0) {
        flat_stage(s_flat, s_flat + kRtQ * kRtStride, a, s_query, npq, rows, r0, n, 0, limit);
        int buf = 0;
        for (int k0 = 0; k0 < limit; k0 += kRtK) {
          if (k0 + kRtK < limit) {
            float* nb = s_flat + (buf ^ 1) * kStage;
            flat_stage(nb, nb + kRtQ * kRtStride, a, s_query, npq, rows, r0, n, k0 + kRtK, limit);
            cp_async_wait<1>();
          } else {
            cp_async_wait<0>();
          }
          __syncthreads();
          const float* sq = s_flat + buf * kStage;
          const float* sc = sq + kRtQ * kRtStride;
          // only the 16-query slices that hold pairs of this group (the same for every thread);
          // the dot-product instances keep all four (the extra variants would spill there)
          if constexpr (kL2) {
            switch (nu) {
              case 1: flat_chunk<kL2, 1>(sq, sc, tq, tc, acc); break;
              case 2: flat_chunk<kL2, 2>(sq, sc, tq, tc, acc); break;
              case 3: flat_chunk<kL2, 3>(sq, sc, tq, tc, acc); break;
              default: flat_chunk<kL2, 4>(sq, sc, tq, tc, acc); break;
            }
          } else {
            flat_chunk<kL2, 4>(sq, sc, tq, tc, acc);
          }
          __syncthreads();  // every warp is done with this buffer before it is refilled
          buf ^= 1;
        }
      }
      // this tile's keys into the per-query buffers
#pragma unroll
      for (int u = 0; u < 4; u++)
#pragma unroll
        for (int v = 0; v < 2; v++) {
          const int g = tq + 16 * u, rr = r0 + tc + 16 * v;
          if (g < npq && rr < n) {
            float s;
            if (rr >= tail_begin) {
              s = a.tail[(size_t)s_slot[g] * 3 + (rr - tail_begin)];
            } else {
              float lanes[8];
#pragma unroll
              for (int p = 0; p < 4; p++) {
                const float2 x = f2_unpack(acc[u][v][p]);
                lanes[2 * p] = x.x;
                lanes[2 * p + 1] = x.y;
              }
              s = reduce_add8_local(lanes);
              const float* qv = a.queries + (size_t)s_query[g] * a.Dp;
              const float* xv = rows + (size_t)rr * a.Dp;
              for (int i = limit; i < a.dim; i++) {
                if (kL2) {
                  const float e = __fsub_rn(qv[i], xv[i]);
                  s = __fmaf_rn(e, e, s);
                } else {
                  s = __fmaf_rn(qv[i], xv[i], s);
                }
              }
            }
            float score;
            if (kL2) {
              score = -s;
            } else if (cosine) {
              score = (float)((double)s / sqrt((double)s_qn[g] * (double)a.rnorm[b + rr]));
            } else {
              score = s;
            }
            const uint64_t key = float_key(score, (uint32_t)a.ordinals[b + rr]);
            if (key > s_thr[g]) keys[(size_t)g * C + atomicAdd(&s_cnt[g], 1u)] = key;
          }
        }
      __syncthreads();
      // buffers that another tile could overflow shrink to their K best
      for (int g = warp; g < npq; g += 8) {
        const uint32_t c = s_cnt[g];
        if (c > (uint32_t)(C - kRtC)) {
          uint64_t t;
          uint32_t nc;
          warp_compact_one<R>(keys + (size_t)g * C, c, (uint32_t)a.K, t, nc);
          if (lane == 0) {
            s_thr[g] = t;
            s_cnt[g] = nc;
          }
        }
      }
      __syncthreads();
    }
    // each query's K best of this list to its (probe, query) slot; its floor rises
    for (int g = warp; g < npq; g += 8) {
      uint32_t c = s_cnt[g];
      uint64_t t = 0;
      uint64_t* kb = keys + (size_t)g * C;
      if (c > (uint32_t)a.K) {
        warp_compact_one<R>(kb, c, (uint32_t)a.K, t, c);
      } else if (c == (uint32_t)a.K) {
        uint64_t mn = ~0ull;
        for (uint32_t i = lane; i < c; i += 32) mn = kb[i] < mn ? kb[i] : mn;
        t = warp_min_u64(mn);
      }
      const int q = s_query[g];
      // a part's K best go to the pair's part slot (merged afterwards); the K-th of a part is a
      // valid floor too (K rows of the list reach it)
      const size_t sidx = parted ? (size_t)s_slot[g] * a.pmax + part : (size_t)s_probe[g] * a.nq + q;
      uint64_t* dst = parted ? a.part_out : a.out;
      for (uint32_t i = lane; i < c; i += 32) dst[sidx * a.K + i] = kb[i];
      if (lane == 0) {
        (parted ? a.part_cnt : a.out_cnt)[sidx] = c;
        if (a.floor && c == (uint32_t)a.K) atomicMax((unsigned long long*)&a.floor[q], (unsigned long long)t);
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// SOAR spill expansion (CentroidIndex.routeWithSpillDistances, CentroidIndex.java:155-187 and
// spillBoundary :213-220).  After the primary probes (ascending distance), with gamma > 0 the
// spill target of each primary within the boundary -- nearest * (1 + gamma) for EUCLIDEAN,
// else the negated (nearest score - |nearest score| * gamma) -- is appended at its own
// distance, unless it is out of range or already listed; the walk stops at the first primary
// beyond the boundary.  Also writes each listed cluster's routing distance (the early exit's
// input).  One thread per query; slots past the query's count hold -1.
// ---------------------------------------------------------------------------------------
__global__ void route_expand_kernel(const int32_t* __restrict__ lists, int nq, int probes,
                                    const float* __restrict__ dist, int nlist, int euclid, float gamma,
                                    const int32_t* __restrict__ spill, int width, int32_t* __restrict__ out_lists,
                                    float* __restrict__ out_dist) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const int32_t* pl = lists + (size_t)q * probes;
  const float* dq = dist + (size_t)q * nlist;
  int32_t* ol = out_lists + (size_t)q * width;
  float* od = out_dist + (size_t)q * width;
  int count = 0;
  for (int r = 0; r < probes; r++) {
    const int32_t l = pl[r];
    ol[count] = l;
    od[count] = l >= 0 ? dq[l] : 0.0f;
    count++;
  }
  if (gamma > 0.0f && spill && probes > 0 && pl[0] >= 0) {
    const float nearest = dq[pl[0]];
    float boundary;
    if (euclid) {
      boundary = __fmul_rn(nearest, __fadd_rn(1.0f, gamma));
    } else {
      const float ns = -nearest;
      boundary = -__fsub_rn(ns, __fmul_rn(fabsf(ns), gamma));
    }
    for (int r = 0; r < probes && count < width; r++) {
      const int32_t l = pl[r];
      if (l < 0 || dq[l] > boundary) break;
      const int32_t sp = spill[l];
      if (sp < 0 || sp >= nlist) continue;
      bool seen = false;
      for (int i = 0; i < count; i++) seen |= ol[i] == sp;
      if (seen) continue;
      ol[count] = sp;
      od[count] = dq[sp];
      count++;
    }
  }
  for (int i = count; i < width; i++) {
    ol[i] = -1;
    od[i] = 0.0f;
  }
}

// BuoyIndex.computeRadii / euclideanDist (BuoyIndex.java:175-183,220-227): the largest
// distance from a cluster's centroid to its rows, each distance a sequential fp32 sum of
// (v - c)^2 (no fused multiply-add) and (float) Math.sqrt of it.  One thread per list-ordered
// row; the maximum by integer atomicMax on the non-negative float bits (radii zeroed).
__global__ void list_radii_kernel(const float* __restrict__ rows, int64_t n, int dim, int Dp,
                                  const int64_t* __restrict__ list_off, int nlist, const float* __restrict__ cent,
                                  float* __restrict__ radii) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  int lo = 0, hi = nlist - 1;  // the list holding row i: the last l with list_off[l] <= i
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (list_off[mid] <= i) lo = mid;
    else hi = mid - 1;
  }
  const float* v = rows + i * Dp;
  const float* c = cent + (size_t)lo * dim;
  float sum = 0.0f;
  for (int d = 0; d < dim; d++) {
    const float e = __fsub_rn(v[d], c[d]);
    sum = __fadd_rn(sum, __fmul_rn(e, e));
  }
  const float r = (float)sqrt((double)sum);
  atomicMax(reinterpret_cast<int*>(radii + lo), __float_as_int(r));
}

// |q - gc| per query: one thread, the sequential sum of squares of PQVectors.cosineScoreFunction
// (PQVectors.java:148-155; gc = 0 without a global centroid).
__global__ void pq_query_norms_kernel(const float* __restrict__ queries, int nq, int dim, const float* __restrict__ gc,
                                      float* __restrict__ out) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const float* v = queries + (size_t)q * dim;
  float s = 0.0f;
  for (int d = 0; d < dim; d++) {
    const float x = __fsub_rn(v[d], gc[d]);
    s = __fadd_rn(s, __fmul_rn(x, x));
  }
  out[q] = (float)sqrt((double)s);
}

// PQVectors.precomputeCentroidNormsSq (PQVectors.java:73-89): one thread per (subspace, centroid).
__global__ void pq_centroid_norms_kernel(int M, int Ks, const int32_t* __restrict__ sub,
                                         const float* __restrict__ codebooks, const int64_t* __restrict__ cb_off,
                                         float* __restrict__ cnorm) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= M * Ks) return;
  const int m = e / Ks, c = e - m * Ks;
  const int size = sub[2 * m];
  const float* cb = codebooks + cb_off[m] + (size_t)c * size;
  float s = 0.0f;
  for (int d = 0; d < size; d++) s = __fadd_rn(s, __fmul_rn(cb[d], cb[d]));
  cnorm[e] = s;
}

// Per row: vecNormSq = sum over subspaces, in order, of centroidNormSq[m][code[m]]
// (PQVectors.java:160-166); one thread per row.
__global__ void pq_row_norms_kernel(const uint8_t* __restrict__ codes, int64_t n, int M, int Mp, int Ks,
                                    const float* __restrict__ cnorm, float* __restrict__ out) {
  const int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= n) return;
  const uint8_t* code = codes + r * Mp;
  float s = 0.0f;
  for (int m = 0; m < M; m++) s = __fadd_rn(s, cnorm[(size_t)m * Ks + code[m]]);
  out[r] = s;
}

// IvfIndex.search's EUCLIDEAN early exit (IvfIndex.java:190-205) over the per-(probe, query)
// results of the list scan (each list's own best K, no floors shared across lists): one warp
// per query walks its listed clusters in route order, keeping the K best keys seen (the
// TopKHeap of k); once it holds K, a cluster whose bound (max(0, (float) sqrt(centroid
// distance) - radius))^2 reaches the K-th best distance ends the walk, and every later cluster
// is skipped with it.  Keys scoring below min_score are not offered (scanPartitionBulk's
// minScore test comes before heap.offer).  Other metrics (no early exit): every listed cluster
// is merged.  The kept keys are written sorted descending.
constexpr int kExitWarps = 8;
constexpr int kExitR = 16;  // 512 key slots per warp >= 2 K (K <= 256)

__global__ void __launch_bounds__(kExitWarps * 32) ivf_early_exit_kernel(
    const uint64_t* __restrict__ out, const uint32_t* __restrict__ out_cnt, int nq, int width, int K,
    const int32_t* __restrict__ lists, const float* __restrict__ ldist, const float* __restrict__ radii, int euclid,
    uint64_t min_key, const uint64_t* __restrict__ harm, const uint32_t* __restrict__ harm_cnt,
    const uint8_t* __restrict__ keyed, uint64_t* __restrict__ keys, uint32_t* __restrict__ kcnt) {
  __shared__ uint64_t s_buf[kExitWarps][32 * kExitR];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = blockIdx.x * kExitWarps + warp;
  if (q >= nq) return;
  uint64_t* buf = s_buf[warp];
  uint32_t n = 0;
  uint64_t worst = 0;  // the K-th best key once n == K
  for (int p = 0; p < width; p++) {
    const int32_t cid = lists[(size_t)q * width + p];
    if (cid < 0) break;
    if (euclid && n == (uint32_t)K) {
      const float worst_score = key_score(worst);
      const float cl2 = (float)sqrt((double)ldist[(size_t)q * width + p]);
      const float lb = __fsub_rn(cl2, radii[cid]);
      if (lb > 0.0f && __fmul_rn(lb, lb) >= -worst_score) break;
    }
    const size_t slot = (size_t)p * nq + q;
    // a list with key dimensions met with a full heap: scanPartitionWithHarmony's results
    const bool harmony = euclid && keyed && keyed[cid] && n == (uint32_t)K;
    const uint32_t c = harmony ? harm_cnt[slot] : out_cnt[slot];
    const uint64_t* src = (harmony ? harm : out) + slot * K;
    for (uint32_t i0 = 0; i0 < c; i0 += 32) {
      const uint32_t i = i0 + lane;
      const uint64_t key = i < c ? src[i] : kEmptyKey;
      const bool keep = i < c && key >= min_key;
      const uint32_t m = __ballot_sync(0xFFFFFFFFu, keep);
      if (keep) buf[n + __popc(m & ((1u << lane) - 1u))] = key;
      n += __popc(m);
    }
    __syncwarp();
    if (n > (uint32_t)K) {
      uint64_t t;
      uint32_t nc;
      warp_compact_one<kExitR>(buf, n, (uint32_t)K, t, nc);
      n = nc;
      worst = t;
    } else if (n == (uint32_t)K) {
      uint64_t mn = ~0ull;
      for (uint32_t i = lane; i < n; i += 32) mn = buf[i] < mn ? buf[i] : mn;
      worst = warp_min_u64(mn);
    }
    __syncwarp();
  }
  // sorted descending (bitonic over the next power of two, empty keys as padding)
  uint32_t p2 = 1;
  while (p2 < n) p2 <<= 1;
  for (uint32_t i = n + lane; i < p2; i += 32) buf[i] = kEmptyKey;
  for (uint32_t size = 2; size <= p2; size <<= 1)
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      __syncwarp();
      for (uint32_t i = lane; i < p2 / 2; i += 32) {
        const uint32_t lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
        const bool desc = (lo & size) == 0;
        const uint64_t x = buf[lo], y = buf[hi];
        if ((x < y) == desc) {
          buf[lo] = y;
          buf[hi] = x;
        }
      }
    }
  __syncwarp();
  for (uint32_t i = lane; i < n; i += 32) keys[(size_t)q * K + i] = buf[i];
  if (lane == 0) kcnt[q] = n;
}

// HARMONY lists (IvfIndex.scanPartitionWithHarmony, IvfIndex.java:279-289): the rows of a keyed
// list scored -squareDistance(query, row) in the reference's order (warp_sqdist), one CTA per
// (query, slot) of a keyed list; each warp scores 32 rows one after another (lane j keeps row j's
// key), offers them to its candidate buffer, and the warps' buffers merge into the K best.  The
// reference first skips rows whose partial distance over the key dimensions reaches the heap's
// worst; such rows' full distances reach it too, so they could not enter the heap (TopKHeap
// admits only better scores) and scoring them changes nothing.
template <int R>
__global__ void __launch_bounds__(256) harmony_list_kernel(HarmonyArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int nwarps = 8, C = 32 * R;
  uint64_t* s_wbuf = reinterpret_cast<uint64_t*>(smem_raw);  // [8][C]
  uint64_t* s_merge = s_wbuf + (size_t)nwarps * C;            // [2][8 K]
  const uint32_t mcap = (uint32_t)(nwarps * a.K);
  uint32_t* s_red = reinterpret_cast<uint32_t*>(s_merge + 2 * (size_t)mcap);
  uint32_t* s_counter = s_red + 32;
  const int64_t pair = blockIdx.x;
  const int q = (int)(pair / a.width), p = (int)(pair % a.width);
  const size_t slot = (size_t)p * a.nq + q;
  const int l = a.lists[(size_t)q * a.width + p];
  if (l < 0 || !a.keyed[l]) {
    if (threadIdx.x == 0) a.out_cnt[slot] = 0;
    return;
  }
  const int64_t b = a.list_off[l], e = a.list_off[l + 1];
  const float* qv = a.queries + (size_t)q * a.Dp;
  WarpStream<R> ws{s_wbuf + (size_t)warp * C, 0u, 0ull};
  for (int64_t r0 = b + (int64_t)warp * 32; r0 < e; r0 += (int64_t)nwarps * 32) {
    uint64_t mine = 0;
    const int nr = (int)((e - r0) < 32 ? (e - r0) : 32);
    for (int j = 0; j < nr; j++) {
      const float d = warp_sqdist(RowF32{qv}, RowF32{a.rows + (size_t)(r0 + j) * a.Dp}, a.dim);
      if (lane == j) mine = float_key(-d, (uint32_t)a.ordinals[r0 + j]);
    }
    ws.offer32(mine, lane < nr, C, a.K);
  }
  __syncwarp();
  if (ws.cnt > (uint32_t)a.K) warp_compact_one<R>(ws.buf, ws.cnt, (uint32_t)a.K, ws.thr, ws.cnt);
  __syncwarp();
  if (lane == 0) s_red[warp] = ws.cnt;
  __syncthreads();
  uint32_t at = 0, total = 0;
  for (int i = 0; i < nwarps; i++) {
    at += i < warp ? s_red[i] : 0u;
    total += s_red[i];
  }
  for (uint32_t i = lane; i < ws.cnt; i += 32) s_merge[at + i] = ws.buf[i];
  __syncthreads();
  const uint32_t n = block_keep_top(s_merge, total, (uint32_t)a.K, s_merge + mcap, s_red, s_counter);
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) a.out[slot * a.K + i] = s_merge[i];
  if (threadIdx.x == 0) a.out_cnt[slot] = n;
}

}  // namespace

cudaError_t launch_route_expand(const int32_t* lists, int nq, int probes, const float* dist, int nlist, int metric,
                                float gamma, const int32_t* spill, int width, int32_t* out_lists, float* out_dist,
                                cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  route_expand_kernel<<<(nq + 127) / 128, 128, 0, st>>>(lists, nq, probes, dist, nlist, metric == kEuclidean ? 1 : 0,
                                                         gamma, spill, width, out_lists, out_dist);
  return cudaGetLastError();
}

cudaError_t launch_list_radii(const float* rows, int64_t n, int dim, int Dp, const int64_t* list_off, int nlist,
                              const float* cent, float* radii, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(radii, 0, sizeof(float) * nlist, st);
  if (e != cudaSuccess || n <= 0) return e;
  list_radii_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rows, n, dim, Dp, list_off, nlist, cent, radii);
  return cudaGetLastError();
}

cudaError_t launch_pq_query_norms(const float* queries, int nq, int dim, const float* gc, float* out,
                                  cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  pq_query_norms_kernel<<<(nq + 127) / 128, 128, 0, st>>>(queries, nq, dim, gc, out);
  return cudaGetLastError();
}

cudaError_t launch_pq_row_norms(const uint8_t* codes, int64_t n, int M, int Mp, int Ks, const int32_t* sub,
                                const float* codebooks, const int64_t* cb_off, float* cnorm_scratch, float* out,
                                cudaStream_t st) {
  pq_centroid_norms_kernel<<<(M * Ks + 255) / 256, 256, 0, st>>>(M, Ks, sub, codebooks, cb_off, cnorm_scratch);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || n <= 0) return e;
  pq_row_norms_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(codes, n, M, Mp, Ks, cnorm_scratch, out);
  return cudaGetLastError();
}

cudaError_t launch_harmony_lists(const HarmonyArgs& a, cudaStream_t st) {
  const int64_t pairs = (int64_t)a.nq * a.width;
  if (pairs <= 0) return cudaSuccess;
  const StreamGeom g = stream_geom(a.K, 32);
  const size_t smem = (size_t)8 * g.C * 8 + (size_t)2 * 8 * a.K * 8 + 33 * 4 + 16;
#define VX_HARM_CASE(RR)                                                                              \
  case RR: {                                                                                          \
    cudaError_t e = cudaFuncSetAttribute(harmony_list_kernel<RR>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                         (int)smem);                                                  \
    if (e != cudaSuccess) return e;                                                                   \
    harmony_list_kernel<RR><<<(unsigned)pairs, 256, smem, st>>>(a);                                   \
    return cudaGetLastError();                                                                        \
  }
  switch (g.R) {
    VX_HARM_CASE(2)
    VX_HARM_CASE(3)
    VX_HARM_CASE(5)
    VX_HARM_CASE(9)
    VX_HARM_CASE(17)
    default: return cudaErrorInvalidValue;
  }
#undef VX_HARM_CASE
}

bool early_exit_supported(int K) { return K >= 1 && 2 * K <= 32 * kExitR; }

cudaError_t launch_ivf_early_exit(const uint64_t* out, const uint32_t* out_cnt, int nq, int width, int K,
                                  const int32_t* lists, const float* ldist, const float* radii, int metric,
                                  float min_score, const uint64_t* harm, const uint32_t* harm_cnt,
                                  const uint8_t* keyed, uint64_t* keys, uint32_t* kcnt, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  if (!early_exit_supported(K)) return cudaErrorInvalidValue;
  // keys scoring >= min_score are those >= (order bits of min_score) << 32; -0.0 == 0.0 as in Java
  const float m = min_score == 0.0f ? -0.0f : min_score;
  const uint64_t min_key = (uint64_t)float_order_bits(m) << 32;
  ivf_early_exit_kernel<<<(nq + kExitWarps - 1) / kExitWarps, kExitWarps * 32, 0, st>>>(
      out, out_cnt, nq, width, K, lists, ldist, radii, metric == kEuclidean ? 1 : 0, min_key, harm, harm_cnt, keyed,
      keys, kcnt);
  return cudaGetLastError();
}

// The tiled routing kernel is used where it applies unless VX_ROUTE_TILED=0.

static bool route_tiled() {
  static const bool v = [] {
    const char* e = getenv("VX_ROUTE_TILED");
    return !(e && *e == '0');
  }();
  return v;
}

static bool route_tile_applies(const float* q, const float* cent, int dim, int nlist) {
  return route_tiled() && dim % kRtK == 0 && (nlist & ~3) > 0 && ((uintptr_t)q & 15u) == 0 &&
         ((uintptr_t)cent & 15u) == 0;
}

int route_launches(const float* queries, int dim, const float* cent, int nlist, int metric) {
  // l2normalize (COSINE), tiled distances, per-row distances for the rest, selection
  const bool tiled = route_tile_applies(metric == kCosine ? nullptr : queries, cent, dim, nlist);
  const bool rest = !tiled || (nlist & 3) != 0;
  return (metric == kCosine ? 1 : 0) + (tiled ? 1 : 0) + (rest ? 1 : 0) + 1;
}

cudaError_t launch_route(const float* queries, int nq, int dim, const float* cent, int nlist,
                         int metric, int nprobe, float* qnorm_scratch, float* dist,
                         int32_t* lists, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  const float* qsrc = queries;
  if (metric == kCosine) {
    l2normalize_kernel<<<(nq * 32 + 255) / 256, 256, 0, st>>>(queries, nq, dim, qnorm_scratch);
    qsrc = qnorm_scratch;
  }
  const int group = nlist & ~3;
  int c_begin = 0;
  cudaError_t e = cudaSuccess;
  if (route_tile_applies(qsrc, cent, dim, nlist)) {
    const dim3 grid((group + kRtC - 1) / kRtC, (nq + kRtQ - 1) / kRtQ);
    const size_t rsmem = (size_t)2 * (kRtQ + kRtC) * kRtStride * sizeof(float);
    auto kern = metric == kEuclidean ? route_tile_kernel<true> : route_tile_kernel<false>;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsmem);
    if (e != cudaSuccess) return e;
    kern<<<grid, 256, rsmem, st>>>(qsrc, nq, dim, cent, group, nlist, dist);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    c_begin = group;
  }
  if (c_begin < nlist) {
    const size_t smem = (size_t)kQG * dim * sizeof(float);
    e = cudaFuncSetAttribute(route_dist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    route_dist_kernel<<<(nq + kQG - 1) / kQG, 256, smem, st>>>(qsrc, nq, dim, cent, nlist, metric, dist, c_begin);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  uint32_t cap = 1;
  while (cap < (uint32_t)nlist) cap <<= 1;
  const size_t smem2 = (size_t)cap * 16 + 33 * 4 + 16;
  e = cudaFuncSetAttribute(route_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem2);
  if (e != cudaSuccess) return e;
  route_select_kernel<<<nq, 256, smem2, st>>>(dist, nlist, nprobe, lists);
  return cudaGetLastError();
}

cudaError_t launch_copy_lists(const int32_t* src, int n, int nlist, int32_t* dst, int32_t* bad, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  copy_lists_kernel<<<(n + 255) / 256, 256, 0, st>>>(src, n, nlist, dst, bad);
  return cudaGetLastError();
}

cudaError_t launch_group_pairs(const int32_t* lists, const int64_t* list_off, int npairs, int nlist,
                               int32_t* counts, int32_t* offsets, int32_t* cursor, int32_t* pairs,
                               cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(counts, 0, sizeof(int32_t) * nlist, st);
  if (e != cudaSuccess) return e;
  if (npairs <= 0) return cudaSuccess;
  pair_hist_kernel<<<(npairs + 255) / 256, 256, 0, st>>>(lists, list_off, npairs, counts);
  pair_scan_kernel<<<1, 1024, 0, st>>>(counts, nlist, offsets, cursor);
  pair_scatter_kernel<<<(npairs + 255) / 256, 256, 0, st>>>(lists, list_off, npairs, cursor, pairs);
  return cudaGetLastError();
}

size_t adc_smem(int M, int Ks, int dim, int R, int K) {
  const int nwarps = 8;
  size_t s = (size_t)M * Ks * 4 + (size_t)dim * 4 + 16;
  s += (size_t)nwarps * 32 * R * 8;
  s += 2ull * nwarps * K * 8;
  s += 33 * 4 + 16;
  return s;
}

cudaError_t launch_adc_scan(const AdcArgs& a, int R, int grid, cudaStream_t st) {
  if (a.npairs <= 0) return cudaSuccess;
  const size_t smem = adc_smem(a.M, a.Ks, a.dim, R, a.K);
#define VX_ADC_CASE(RR)                                                                          \
  case RR: {                                                                                     \
    cudaError_t e = cudaFuncSetAttribute(adc_scan_kernel<RR>,                                    \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e != cudaSuccess) return e;                                                              \
    adc_scan_kernel<RR><<<grid, 256, smem, st>>>(a);                                             \
    return cudaGetLastError();                                                                   \
  }
  switch (R) {
    VX_ADC_CASE(2)
    VX_ADC_CASE(3)
    VX_ADC_CASE(5)
    VX_ADC_CASE(9)
    VX_ADC_CASE(17)
    VX_ADC_CASE(33)
    default: return cudaErrorInvalidValue;
  }
#undef VX_ADC_CASE
}

bool adc_group_supported(int M, int Ks, int dim) {
  return Ks == 256 && M > 0 && M % kMChunk == 0 && dim == 8 * M;
}

cudaError_t launch_make_groups(const int32_t* counts, const int32_t* offsets, const int32_t* order, int nlist,
                               int wmax, int2* groups, int32_t* ngroups, cudaStream_t st, const int64_t* list_off,
                               int rmax) {
  if (wmax < 1 || wmax > 255 || (rmax > 0 && !list_off)) return cudaErrorInvalidValue;
  // ngroups[1] is the dispenser the scan kernels take groups from
  cudaError_t e = cudaMemsetAsync(ngroups + 1, 0, sizeof(int32_t), st);
  if (e != cudaSuccess) return e;
  make_groups_kernel<<<1, 1024, 0, st>>>(counts, offsets, order, nlist, wmax, list_off, rmax, groups, ngroups);
  return cudaGetLastError();
}

// Row parts of one (query, list) pair: the union of its parts' K best (each part at most K keys,
// unsorted; ordinals distinct across parts) cut to the K best and written to the pair's slot of
// out.  One warp per pair position; pairs of single-part lists were written by the scan itself.
// The parts' keys are first packed to the front of the pair's part area (held in registers in
// between), then shrunk in place by warp_compact_one.
template <int R>
__global__ void flat_parts_merge_kernel(FlatListArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t w = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  if (w >= *a.pair_count) return;
  const int32_t pair = a.pairs[w];
  const int l = a.lists[pair];
  const int n = (int)(a.list_off[l + 1] - a.list_off[l]);
  if (!(a.rmax > 0 && n > a.rmax)) return;
  const int parts = (n + a.rmax - 1) / a.rmax;
  uint64_t* base = a.part_out + (size_t)w * a.pmax * a.K;
  const uint32_t* cnt = a.part_cnt + (size_t)w * a.pmax;
  uint64_t e[R];
  uint32_t mine = 0;
#pragma unroll
  for (int r = 0; r < R; r++) {
    const int i = lane + 32 * r;
    const int j = i / a.K, o = i - j * a.K;
    const bool ok = j < parts && o < (int)cnt[j];
    e[r] = ok ? base[i] : kEmptyKey;
    mine += ok ? 1u : 0u;
  }
  uint32_t incl = mine;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, d);
    if (lane >= d) incl += v;
  }
  const uint32_t total = __shfl_sync(0xFFFFFFFFu, incl, 31);
  uint32_t pos = incl - mine;
  __syncwarp();
#pragma unroll
  for (int r = 0; r < R; r++) {
    const int i = lane + 32 * r;
    const int j = i / a.K, o = i - j * a.K;
    if (j < parts && o < (int)cnt[j]) base[pos++] = e[r];
  }
  __syncwarp();
  uint32_t c = total;
  uint64_t t = 0;
  if (c > (uint32_t)a.K) warp_compact_one<R>(base, c, (uint32_t)a.K, t, c);
  const int q = pair / a.nprobe, p = pair - q * a.nprobe;
  const size_t sidx = (size_t)p * a.nq + q;
  for (uint32_t i = lane; i < c; i += 32) a.out[sidx * a.K + i] = base[i];
  if (lane == 0) a.out_cnt[sidx] = c;
}

cudaError_t launch_flat_parts_merge(const FlatListArgs& a, int64_t pair_slots, cudaStream_t st) {
  if (pair_slots <= 0 || a.rmax <= 0 || a.pmax <= 1) return cudaSuccess;
  const int keys = a.pmax * a.K;
  if (keys > kFlatPartKeysMax) return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)((pair_slots * 32 + 255) / 256);
  if (keys <= 32) flat_parts_merge_kernel<1><<<grid, 256, 0, st>>>(a);
  else if (keys <= 64) flat_parts_merge_kernel<2><<<grid, 256, 0, st>>>(a);
  else if (keys <= 128) flat_parts_merge_kernel<4><<<grid, 256, 0, st>>>(a);
  else if (keys <= 256) flat_parts_merge_kernel<8><<<grid, 256, 0, st>>>(a);
  else if (keys <= 512) flat_parts_merge_kernel<16><<<grid, 256, 0, st>>>(a);
  else flat_parts_merge_kernel<32><<<grid, 256, 0, st>>>(a);
  return cudaGetLastError();
}

bool flat_list_supported(int K) { return K >= 1 && K <= 9 * 32 - kRtC; }

cudaError_t launch_pad_rows(const float* src, int64_t n, int dim, int64_t src_stride, const int32_t* map, int Dp,
                            float* dst, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t total = n * (int64_t)Dp;
  const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 32);
  pad_rows_kernel<<<grid, 256, 0, st>>>(src, n, dim, src_stride, map, Dp, dst);
  return cudaGetLastError();
}

cudaError_t launch_row_norms(const float* rows, int64_t n, int dim, int Dp, float* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  row_norms_kernel<<<(unsigned)((n * 32 + 255) / 256), 256, 0, st>>>(rows, n, dim, Dp, out);
  return cudaGetLastError();
}

cudaError_t launch_flat_list(const FlatListArgs& a, int64_t pair_slots, int grid, cudaStream_t st) {
  if (pair_slots <= 0) return cudaSuccess;
  const bool l2 = a.metric == kEuclidean;
  const int64_t warps = pair_slots * 3;
  const unsigned tgrid = (unsigned)((warps * 32 + 255) / 256);
  if (l2) flat_tail_kernel<true><<<tgrid, 256, 0, st>>>(a);
  else flat_tail_kernel<false><<<tgrid, 256, 0, st>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  // key slots per query 32 R >= K + one tile's 32; R = 9 (K up to 256) takes ~200 KB of shared
  // memory, one CTA per SM
  const int R = a.K <= 2 * 32 - kRtC ? 2 : a.K <= 4 * 32 - kRtC ? 4 : 9;
  const size_t smem = (size_t)2 * (kRtQ + kRtC) * kRtStride * sizeof(float) + (size_t)kFlGroup * 32 * R * 8;
  auto kern = l2 ? (R == 2 ? flat_list_kernel<true, 2> : R == 4 ? flat_list_kernel<true, 4> : flat_list_kernel<true, 9>)
                 : (R == 2 ? flat_list_kernel<false, 2> : R == 4 ? flat_list_kernel<false, 4> : flat_list_kernel<false, 9>);
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, 256, smem, st>>>(a);
  return cudaGetLastError();
}

static size_t adc_group_smem(int dim, int R) {
  return (size_t)kMChunk * 256 * 16 + (size_t)kAdcGroupQ * dim * 4 +
         (size_t)(kAdcWarps + 1) * kAdcGroupQ * 32 * R * 8;
}

// R in {2, 3, 5, 9} with 32 R >= 2 K + 1 (each warp buffer and each merge buffer); shared
// memory 64 KB tables + 4 residuals + 9 * 4 buffers of 32 R keys (<= 159 KB at R = 9).
cudaError_t launch_adc_group(const AdcArgs& a, int R, int grid, cudaStream_t st) {
  if (a.npairs <= 0) return cudaSuccess;
  const size_t smem = adc_group_smem(a.dim, R);
  const bool dot = a.metric != kEuclidean;
#define VX_ADCG_CASE(RR)                                                                         \
  case RR: {                                                                                     \
    auto kern = dot ? adc_group_kernel<true, RR> : adc_group_kernel<false, RR>;                 \
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e != cudaSuccess) return e;                                                              \
    kern<<<grid, kAdcThreads, smem, st>>>(a);                                                    \
    return cudaGetLastError();                                                                   \
  }
  switch (R) {
    VX_ADCG_CASE(2)
    VX_ADCG_CASE(3)
    VX_ADCG_CASE(5)
    VX_ADCG_CASE(9)
    default: return cudaErrorInvalidValue;
  }
#undef VX_ADCG_CASE
}

}  // namespace vx
