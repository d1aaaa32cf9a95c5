// bq_scan.cu -- sign-bit binary quantization (BQ) Hamming scan with fused top-K.
//
// Restates, batched over queries, QuantizedFlatScanAdapter.selectApproximateCandidates
// (vectors-db/.../index/QuantizedFlatScanAdapter.java:97-113) over
// BinaryQuantizedVectors.signBitScoreFunction (vectors-quantization/.../
// BinaryQuantizedVectors.java:81-107): h = sum_w popcount(q_w XOR v_w).  Every score
// function of h is strictly decreasing in h for 0 <= h <= dim, so ranking by (h asc, id asc)
// equals ranking by (score desc, id asc); scores are recovered from h at the end.
//
// Layout: the database is row-major, 8*nw_pad bytes per row (the reference's long[] words,
// BinaryQuantizer.java:207-232, zero-padded to nw_pad words).  Each CTA owns a contiguous
// range of rows (a "part") and streams it through shared memory in 128-row tiles; every
// thread owns one query (its words live in registers) and scores each staged row against
// it.  The database is read from HBM once per batch; the binding roof is the integer/popc
// pipe.  These popcount scans serve BQ and BBQ indexes built without the int8 operand of the
// tensor-core scan (gemm_scan.cu), and vx_bq_scan_candidates_noalloc; the file also holds the
// BBQ query preparation and the per-row records both BBQ scans read.
#include "bbq.cuh"
#include "common.cuh"
#include "kernels.h"

namespace vx {

namespace {

constexpr int kBqTile = 128;
constexpr int kBqThreads = 256;

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(sz)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

template <int NW, int R>
__global__ void __launch_bounds__(kBqThreads, 2)
    bq_scan_kernel(const uint64_t* __restrict__ db, int64_t n, const uint64_t* __restrict__ qw,
                   int nq, int64_t rows_per_part, int K, int C, uint64_t* __restrict__ bufs,
                   uint32_t* __restrict__ cnts, uint64_t* __restrict__ thrs) {
  extern __shared__ __align__(16) uint64_t s_tile[];  // [2][kBqTile * NW]
  const int part = blockIdx.x;
  const int64_t r0 = (int64_t)part * rows_per_part;
  int64_t r1 = r0 + rows_per_part;
  if (r1 > n) r1 = n;
  const int64_t nrows = r1 > r0 ? r1 - r0 : 0;
  const int ntiles = (int)((nrows + kBqTile - 1) / kBqTile);
  constexpr int kChunks = kBqTile * NW / 2;  // 16-byte chunks per tile

  auto stage = [&](int t) {
    uint64_t* dst = s_tile + (t & 1) * (kBqTile * NW);
    const int64_t base_row = r0 + (int64_t)t * kBqTile;
    for (int c = threadIdx.x; c < kChunks; c += kBqThreads) {
      int row = c / (NW / 2 > 0 ? NW / 2 : 1);
      bool valid = (base_row + row) < r1;
      const uint64_t* src = valid ? db + (base_row * NW) + (int64_t)c * 2 : db;
      cp_async16(dst + c * 2, src, valid);
    }
  };

  if (ntiles > 0) stage(0);
  cp_async_commit();
  for (int t = 0; t < ntiles; t++) {
    if (t + 1 < ntiles) stage(t + 1);
    cp_async_commit();
    cp_async_wait1();
    __syncthreads();
    const uint64_t* T = s_tile + (t & 1) * (kBqTile * NW);
    const int64_t base_row = r0 + (int64_t)t * kBqTile;
    const int rows = (int)((r1 - base_row) < kBqTile ? (r1 - base_row) : kBqTile);
    for (int qb = 0; qb < nq; qb += kBqThreads) {
      const int q = qb + threadIdx.x;
      const bool active = q < nq;
      uint64_t qr[NW];
#pragma unroll
      for (int w = 0; w < NW; w++) qr[w] = active ? qw[(size_t)q * NW + w] : 0ull;
      const size_t sidx = (size_t)part * nq + (active ? q : 0);
      LaneStream st;
      st.base = bufs + sidx * (size_t)C;
      st.cnt = active ? cnts[sidx] : 0u;
      st.thr = active ? thrs[sidx] : ~0ull;
      for (int rr = 0; rr < rows; rr += 32) {
        const int re = (rr + 32 < rows) ? rr + 32 : rows;
        for (int r = rr; r < re; r++) {
          const uint64_t* row = T + r * NW;
          uint32_t h = 0;
#pragma unroll
          for (int w = 0; w < NW; w++) h += (uint32_t)__popcll(qr[w] ^ row[w]);
          st.offer(make_key(0xFFFFFFFFu - h, (uint32_t)(base_row + r)));
        }
        warp_compact_lanes<R>(st.cnt > (uint32_t)(C - 32), st.base, st.cnt, st.thr, (uint32_t)K);
      }
      if (active) {
        cnts[sidx] = st.cnt;
        thrs[sidx] = st.thr;
      }
    }
    __syncthreads();
  }
  // Leave every stream of this part with at most K keys.
  for (int qb = 0; qb < nq; qb += kBqThreads) {
    const int q = qb + threadIdx.x;
    const bool active = q < nq;
    const size_t sidx = (size_t)part * nq + (active ? q : 0);
    uint64_t* base = bufs + sidx * (size_t)C;
    uint32_t cnt = active ? cnts[sidx] : 0u;
    uint64_t thr = active ? thrs[sidx] : ~0ull;
    warp_compact_lanes<R>(cnt > (uint32_t)K, base, cnt, thr, (uint32_t)K);
    if (active) cnts[sidx] = cnt;
  }
}

template <int NW>
cudaError_t launch_nw(const uint64_t* db, int64_t n, const uint64_t* qw, int nq, int parts,
                      const StreamGeom& g, uint64_t* bufs, uint32_t* cnts, uint64_t* thrs,
                      cudaStream_t st) {
  int64_t rows_per_part = (n + parts - 1) / parts;
  size_t smem = 2ull * kBqTile * NW * sizeof(uint64_t);
#define VX_BQ_CASE(RR)                                                                         \
  case RR: {                                                                                   \
    auto kern = bq_scan_kernel<NW, RR>;                                                        \
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                         (int)smem);                                           \
    if (e != cudaSuccess) return e;                                                            \
    kern<<<parts, kBqThreads, smem, st>>>(db, n, qw, nq, rows_per_part, g.K, g.C, bufs, cnts,   \
                                          thrs);                                               \
    return cudaGetLastError();                                                                 \
  }
  switch (g.R) {
    VX_BQ_CASE(2)
    VX_BQ_CASE(3)
    VX_BQ_CASE(5)
    VX_BQ_CASE(9)
    VX_BQ_CASE(17)
    VX_BQ_CASE(33)
    default: return cudaErrorInvalidValue;
  }
#undef VX_BQ_CASE
}

// Packs fp32 queries into sign-bit words: bit (d & 63) of word (d >> 6) is set iff
// v[d] >= 0 (BinaryQuantizer.packBits / bytesToLongs, BinaryQuantizer.java:207-232).
__global__ void bq_pack_kernel(const float* __restrict__ q, int nq, int dim, int nw_pad,
                               uint64_t* __restrict__ out) {
  int qi = blockIdx.x;
  for (int w = threadIdx.x; w < nw_pad; w += blockDim.x) {
    uint64_t word = 0;
    for (int b = 0; b < 64; b++) {
      int d = w * 64 + b;
      if (d < dim && q[(size_t)qi * dim + d] >= 0.0f) word |= 1ull << b;
    }
    out[(size_t)qi * nw_pad + w] = word;
  }
}


// ---------------------------------------------------------------------------------------
// BBQ (BinaryMode.BBQ): BinaryQuantizedVectors.bbqScoreFunction, computeBbqDot and
// asymmetricDot (vectors-quantization/.../BinaryQuantizedVectors.java:110-275).  Rows are
// centroid-relative sign bits with corrections (|v - c|^2, vl = min(v - c), width = max - min);
// the query is centred, quantised to 4 bits over its own [min, max] and split into 4 bit
// planes.  rawAsymDot = sum_b popcount(bits & plane_b) << b is exact; the score follows the
// Java float expression operation by operation (no fused multiply-add).
// ---------------------------------------------------------------------------------------
// One thread per query: the two sequential passes of bbqScoreFunction's query set-up.
__global__ void bbq_prep_queries_kernel(const float* __restrict__ q, int nq, int dim, const float* __restrict__ cent,
                                        int nw_pad, uint64_t* __restrict__ planes, BbqQuery* __restrict__ info) {
  const int qi = blockIdx.x * blockDim.x + threadIdx.x;
  if (qi >= nq) return;
  const float* v = q + (size_t)qi * dim;
  float nsq = 0.0f, mn = __int_as_float(0x7f800000), mx = __int_as_float(0xff800000);
  for (int d = 0; d < dim; d++) {
    const float c = __fsub_rn(v[d], cent[d]);  // VectorUtil.subInPlace
    nsq = __fadd_rn(nsq, __fmul_rn(c, c));
    if (c < mn) mn = c;
    if (c > mx) mx = c;
  }
  const float width = __fsub_rn(mx, mn);
  const float scale = width > 0.0f ? __fdiv_rn(15.0f, width) : 0.0f;
  int32_t qsum = 0;
  uint64_t* pl = planes + (size_t)qi * 4 * nw_pad;
  for (int w = 0; w < nw_pad; w++) {
    uint64_t b0 = 0, b1 = 0, b2 = 0, b3 = 0;
    for (int j = 0; j < 64; j++) {
      const int d = w * 64 + j;
      if (d >= dim) break;
      const float c = __fsub_rn(v[d], cent[d]);
      // Math.round: nearest, ties toward +infinity; NaN -> 0
      const float t = __fmul_rn(__fsub_rn(c, mn), scale);
      int32_t qv = 0;
      if (t == t) {
        const float f = floorf(t);
        qv = (int32_t)f + ((__fsub_rn(t, f) >= 0.5f) ? 1 : 0);
      }
      qv = qv < 0 ? 0 : (qv > 15 ? 15 : qv);
      qsum += qv;
      const uint64_t bit = 1ull << j;
      if (qv & 1) b0 |= bit;
      if (qv & 2) b1 |= bit;
      if (qv & 4) b2 |= bit;
      if (qv & 8) b3 |= bit;
    }
    pl[w] = b0;
    pl[nw_pad + w] = b1;
    pl[2 * nw_pad + w] = b2;
    pl[3 * nw_pad + w] = b3;
  }
  BbqQuery o;
  o.qmin = mn;
  o.w15 = __fdiv_rn(width, 15.0f);
  o.nsq = nsq;
  o.norm = (float)sqrt((double)nsq);
  o.qsum = qsum;
  info[qi] = o;
}

// Carry-save adder of three words: l holds the bitwise sum, h the carries (weight 2).
__device__ __forceinline__ void csa(uint64_t& h, uint64_t& l, uint64_t a, uint64_t b, uint64_t c) {
  const uint64_t u = a ^ b;
  h = (a & b) | (u & c);
  l = u ^ c;
}

// sum_w popcount(x[w] & p[w]) over 16 words through a Harley-Seal carry-save tree: the words are
// added bitwise into ones / twos / fours / eights / sixteens (cheap logic operations), so five
// popcounts replace sixteen on the slow population-count pipe; the integer is the same.
__device__ __forceinline__ int32_t popc_and16(const uint64_t* x, const uint64_t (&p)[16]) {
  uint64_t ones = 0, twos = 0, fours = 0, eights = 0, sixteens;
  uint64_t twos_a, twos_b, fours_a, fours_b, eights_a, eights_b;
  csa(twos_a, ones, ones, x[0] & p[0], x[1] & p[1]);
  csa(twos_b, ones, ones, x[2] & p[2], x[3] & p[3]);
  csa(fours_a, twos, twos, twos_a, twos_b);
  csa(twos_a, ones, ones, x[4] & p[4], x[5] & p[5]);
  csa(twos_b, ones, ones, x[6] & p[6], x[7] & p[7]);
  csa(fours_b, twos, twos, twos_a, twos_b);
  csa(eights_a, fours, fours, fours_a, fours_b);
  csa(twos_a, ones, ones, x[8] & p[8], x[9] & p[9]);
  csa(twos_b, ones, ones, x[10] & p[10], x[11] & p[11]);
  csa(fours_a, twos, twos, twos_a, twos_b);
  csa(twos_a, ones, ones, x[12] & p[12], x[13] & p[13]);
  csa(twos_b, ones, ones, x[14] & p[14], x[15] & p[15]);
  csa(fours_b, twos, twos, twos_a, twos_b);
  csa(eights_b, fours, fours, fours_a, fours_b);
  csa(sixteens, eights, eights, eights_a, eights_b);
  return 16 * __popcll(sixteens) + 8 * __popcll(eights) + 4 * __popcll(fours) + 2 * __popcll(twos) +
         __popcll(ones);
}

// Score of one (query, row): computeBbqDot then the metric's transform (:155-225).
__device__ __forceinline__ float bbq_score(int metric, const BbqQuery& qi, float4 ri, int32_t raw, int dim) {
  const float dist_c = ri.x, vl = ri.y, width = ri.z;
  const int32_t pop = __float_as_int(ri.w);
  const float approx =
      bbq_approx(qi.qmin, qi.w15, (float)qi.qsum, vl, width, bbq_row_term(vl, width, dim, pop), (float)raw);
  switch (metric) {
    case kEuclidean: return bbq_l2_score(bbq_l2_adj(approx, qi.nsq, dist_c));
    case kCosine: return bbq_cos_score(approx, qi.norm, bbq_vnorm(dist_c));
    case kMaxInnerProduct: return scale_mip(approx);
    default: return bbq_dot_score(approx);
  }
}

template <int NW, int R>
__global__ void __launch_bounds__(kBqThreads, 1)  // the 4 query planes stay in registers
    bbq_scan_kernel(const uint64_t* __restrict__ db, const float4* __restrict__ rowinfo, int64_t n, int dim,
                    int metric, const uint64_t* __restrict__ planes, const BbqQuery* __restrict__ qinfo, int nq,
                    int64_t rows_per_part, int K, int C, uint64_t* __restrict__ bufs, uint32_t* __restrict__ cnts,
                    uint64_t* __restrict__ thrs) {
  extern __shared__ __align__(16) uint64_t s_tile[];  // [2][kBqTile * NW] words, then [2][kBqTile] float4
  float4* s_info = reinterpret_cast<float4*>(s_tile + 2 * kBqTile * NW);
  const int part = blockIdx.x;
  const int64_t r0 = (int64_t)part * rows_per_part;
  int64_t r1 = r0 + rows_per_part;
  if (r1 > n) r1 = n;
  const int64_t nrows = r1 > r0 ? r1 - r0 : 0;
  const int ntiles = (int)((nrows + kBqTile - 1) / kBqTile);
  constexpr int kChunks = kBqTile * NW / 2;

  auto stage = [&](int t) {
    uint64_t* dst = s_tile + (t & 1) * (kBqTile * NW);
    float4* idst = s_info + (t & 1) * kBqTile;
    const int64_t base_row = r0 + (int64_t)t * kBqTile;
    for (int c = threadIdx.x; c < kChunks + kBqTile; c += kBqThreads) {
      if (c < kChunks) {
        const int row = c / (NW / 2);
        const bool valid = (base_row + row) < r1;
        cp_async16(dst + c * 2, valid ? db + base_row * NW + (int64_t)c * 2 : db, valid);
      } else {
        const int row = c - kChunks;
        const bool valid = (base_row + row) < r1;
        cp_async16(idst + row, valid ? rowinfo + base_row + row : rowinfo, valid);
      }
    }
  };

  // Query chunks outermost: a thread keeps its query's planes and stream in registers while the
  // part's rows stream past (re-reading the rows per chunk is cheaper than the planes per tile).
  for (int qb = 0; qb < nq; qb += kBqThreads) {
    const int q = qb + threadIdx.x;
    const bool active = q < nq;
    uint64_t qp[4][NW];
#pragma unroll
    for (int b = 0; b < 4; b++)
#pragma unroll
      for (int w = 0; w < NW; w++) qp[b][w] = active ? planes[((size_t)q * 4 + b) * NW + w] : 0ull;
    const BbqQuery qi = active ? qinfo[q] : BbqQuery{};
    const size_t sidx = (size_t)part * nq + (active ? q : 0);
    LaneStream st;
    st.base = bufs + sidx * (size_t)C;
    st.cnt = 0u;
    st.thr = active ? 0ull : ~0ull;
    __syncthreads();  // the previous chunk is done with both staging buffers
    if (ntiles > 0) stage(0);
    cp_async_commit();
    for (int t = 0; t < ntiles; t++) {
      if (t + 1 < ntiles) stage(t + 1);
      cp_async_commit();
      cp_async_wait1();
      __syncthreads();
      const uint64_t* T = s_tile + (t & 1) * (kBqTile * NW);
      const float4* I = s_info + (t & 1) * kBqTile;
      const int64_t base_row = r0 + (int64_t)t * kBqTile;
      const int rows = (int)((r1 - base_row) < kBqTile ? (r1 - base_row) : kBqTile);
      for (int rr = 0; rr < rows; rr += 32) {
        const int re = (rr + 32 < rows) ? rr + 32 : rows;
        for (int r = rr; r < re; r++) {
          const uint64_t* row = T + r * NW;
          int32_t raw = 0;
#pragma unroll
          for (int b = 0; b < 4; b++) {
            int32_t sb = 0;
            if constexpr (NW == 16) {
              sb = popc_and16(row, qp[b]);
            } else {
#pragma unroll
              for (int w = 0; w < NW; w++) sb += __popcll(row[w] & qp[b][w]);
            }
            raw += sb << b;
          }
          if (active) st.offer(float_key(bbq_score(metric, qi, I[r], raw, dim), (uint32_t)(base_row + r)));
        }
        warp_compact_lanes<R>(st.cnt > (uint32_t)(C - 32), st.base, st.cnt, st.thr, (uint32_t)K);
      }
      __syncthreads();  // every thread is done with this buffer before it is refilled
    }
    warp_compact_lanes<R>(st.cnt > (uint32_t)K, st.base, st.cnt, st.thr, (uint32_t)K);
    if (active) {
      cnts[sidx] = st.cnt;
      thrs[sidx] = st.thr;
    }
  }
}

// Per-row staging record: (|v - c|^2, vl, width, popcount of the bits as int bits).
__global__ void bbq_rowinfo_kernel(const uint64_t* __restrict__ words, int nw, int nw_pad, const float* __restrict__ corr,
                                   int64_t n, float4* __restrict__ out) {
  const int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= n) return;
  int32_t pop = 0;
  for (int w = 0; w < nw; w++) pop += __popcll(words[r * nw_pad + w]);  // BitCounts.popcount
  out[r] = make_float4(corr[r * 3], corr[r * 3 + 1], corr[r * 3 + 2], __int_as_float(pop));
}

// Per-row epilogue record of the int8 tensor-core BBQ scan: (vl, width, vl * D + width * pop,
// |v - c| for COSINE or |v - c|^2 otherwise), from the (|v - c|^2, vl, width, pop) record.
__global__ void bbq_epi_rows_kernel(const float4* __restrict__ info, int64_t n, int dim, int metric,
                                    float4* __restrict__ out) {
  const int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= n) return;
  const float4 i = info[r];
  const float s1 = bbq_row_term(i.y, i.z, dim, __float_as_int(i.w));
  out[r] = make_float4(i.y, i.z, s1, metric == kCosine ? bbq_vnorm(i.x) : i.x);
}

// The 4-bit query codes as int8 (the A operand of rawAsymDot on the tensor cores) from the bit
// planes [nq][4][nw_pad]; one thread per 4 bytes of a row, dims [dim, Dp8) -> 0.
__global__ void bbq_planes_to_i8_kernel(const uint64_t* __restrict__ planes, int nq, int dim, int nw_pad, int Dp8,
                                        int8_t* __restrict__ dst) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int per_row = Dp8 / 4;
  if (t >= (int64_t)nq * per_row) return;
  const int64_t r = t / per_row;
  const int c0 = (int)(t - r * per_row) * 4;
  const uint64_t* pl = planes + r * 4 * nw_pad;
  uint32_t out = 0;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int c = c0 + j;
    uint32_t v = 0;
    if (c < dim) {
      const int w = c >> 6, b = c & 63;
#pragma unroll
      for (int p = 0; p < 4; p++) v |= (uint32_t)((pl[p * nw_pad + w] >> b) & 1ull) << p;
    }
    out |= v << (8 * j);
  }
  reinterpret_cast<uint32_t*>(dst + r * Dp8)[c0 / 4] = out;
}

template <int NW>
cudaError_t launch_bbq_nw(const uint64_t* db, const float4* rowinfo, int64_t n, int dim, int metric,
                          const uint64_t* planes, const BbqQuery* qinfo, int nq, int parts, const StreamGeom& g,
                          uint64_t* bufs, uint32_t* cnts, uint64_t* thrs, cudaStream_t st) {
  const int64_t rows_per_part = (n + parts - 1) / parts;
  const size_t smem = 2ull * kBqTile * NW * sizeof(uint64_t) + 2ull * kBqTile * sizeof(float4);
#define VX_BBQ_CASE(RR)                                                                             \
  case RR: {                                                                                        \
    auto kern = bbq_scan_kernel<NW, RR>;                                                            \
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e != cudaSuccess) return e;                                                                 \
    kern<<<parts, kBqThreads, smem, st>>>(db, rowinfo, n, dim, metric, planes, qinfo, nq, rows_per_part, g.K, g.C, \
                                          bufs, cnts, thrs);                                        \
    return cudaGetLastError();                                                                      \
  }
  switch (g.R) {
    VX_BBQ_CASE(2)
    VX_BBQ_CASE(3)
    VX_BBQ_CASE(5)
    VX_BBQ_CASE(9)
    VX_BBQ_CASE(17)
    VX_BBQ_CASE(33)
    default: return cudaErrorInvalidValue;
  }
#undef VX_BBQ_CASE
}

}  // namespace

int bq_padded_words(int nw) {
  for (int p : {2, 4, 8, 16, 32})
    if (nw <= p) return p;
  return -1;
}

int bq_parts(int64_t n, int num_sms) {
  int64_t p = (int64_t)num_sms * 2;
  int64_t max_parts = (n + kBqTile - 1) / kBqTile;
  if (p > max_parts) p = max_parts;
  return (int)(p < 1 ? 1 : p);
}

cudaError_t launch_bq_scan(const uint64_t* db, int64_t n, int nw_pad, const uint64_t* qw, int nq,
                           int parts, const StreamGeom& g, uint64_t* bufs, uint32_t* cnts,
                           uint64_t* thrs, cudaStream_t st) {
  switch (nw_pad) {
    case 2: return launch_nw<2>(db, n, qw, nq, parts, g, bufs, cnts, thrs, st);
    case 4: return launch_nw<4>(db, n, qw, nq, parts, g, bufs, cnts, thrs, st);
    case 8: return launch_nw<8>(db, n, qw, nq, parts, g, bufs, cnts, thrs, st);
    case 16: return launch_nw<16>(db, n, qw, nq, parts, g, bufs, cnts, thrs, st);
    case 32: return launch_nw<32>(db, n, qw, nq, parts, g, bufs, cnts, thrs, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_bbq_prep_queries(const float* q, int nq, int dim, const float* centroid, int nw_pad,
                                    uint64_t* planes, BbqQuery* info, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  bbq_prep_queries_kernel<<<(nq + 127) / 128, 128, 0, st>>>(q, nq, dim, centroid, nw_pad, planes, info);
  return cudaGetLastError();
}

cudaError_t launch_bbq_rowinfo(const uint64_t* words, int nw, int nw_pad, const float* corr, int64_t n, float4* out,
                               cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  bbq_rowinfo_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(words, nw, nw_pad, corr, n, out);
  return cudaGetLastError();
}

cudaError_t launch_bbq_epi_rows(const float4* info, int64_t n, int dim, int metric, float4* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  bbq_epi_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(info, n, dim, metric, out);
  return cudaGetLastError();
}

cudaError_t launch_bbq_planes_to_i8(const uint64_t* planes, int nq, int dim, int nw_pad, int Dp8, int8_t* dst,
                                    cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  const int64_t total = (int64_t)nq * (Dp8 / 4);
  bbq_planes_to_i8_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(planes, nq, dim, nw_pad, Dp8, dst);
  return cudaGetLastError();
}

bool bbq_supported(int nw_pad) { return nw_pad >= 2 && nw_pad <= 16; }

cudaError_t launch_bbq_scan(const uint64_t* db, const float4* rowinfo, int64_t n, int nw_pad, int dim, int metric,
                            const uint64_t* planes, const BbqQuery* qinfo, int nq, int parts, const StreamGeom& g,
                            uint64_t* bufs, uint32_t* cnts, uint64_t* thrs, cudaStream_t st) {
  switch (nw_pad) {
    case 2: return launch_bbq_nw<2>(db, rowinfo, n, dim, metric, planes, qinfo, nq, parts, g, bufs, cnts, thrs, st);
    case 4: return launch_bbq_nw<4>(db, rowinfo, n, dim, metric, planes, qinfo, nq, parts, g, bufs, cnts, thrs, st);
    case 8: return launch_bbq_nw<8>(db, rowinfo, n, dim, metric, planes, qinfo, nq, parts, g, bufs, cnts, thrs, st);
    case 16: return launch_bbq_nw<16>(db, rowinfo, n, dim, metric, planes, qinfo, nq, parts, g, bufs, cnts, thrs, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_bq_pack_queries(const float* q, int nq, int dim, int nw_pad, uint64_t* out,
                                   cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  bq_pack_kernel<<<nq, 32, 0, st>>>(q, nq, dim, nw_pad, out);
  return cudaGetLastError();
}

StreamGeom stream_geom(int K, int slack) {
  StreamGeom g;
  g.K = K;
  int need = (K + slack + 1 + 31) / 32;
  int R = -1;
  for (int r : {2, 3, 5, 9, 17, 33})
    if (r >= need) {
      R = r;
      break;
    }
  g.R = R;
  g.C = R > 0 ? 32 * R : 0;
  return g;
}

}  // namespace vx
