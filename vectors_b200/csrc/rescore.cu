// rescore.cu -- exact re-scoring of approximate candidates, the completeness test that
// decides whether the approximate pass provably kept every row of the exact top-k, and the
// exact fallback scan used for queries that fail it.
//
// Why this is exact.  The tensor-core pass ranks rows by an approximate key a(x) with a
// proven bound |a(x) - e(x)| <= m_q, where e(x) is the same key computed exactly.  Let A_k be
// the k-th best approximate key.  Every row of the exact top-k has a(x) >= A_k - 2 m_q, so if
// the Kc-th kept candidate is already below A_k - 2 m_q, the Kc candidates contain the whole
// exact top-k and re-scoring them in fp32 (exact.cuh) yields the reference's answer.  Queries
// whose candidate window is too narrow (ties, duplicates, extreme data) are flagged and
// re-run through exact_scan_kernel, which scores every row in fp32.
#include "exact.cuh"
#include "kernels.h"
#include "rescore.h"
#include "select.cuh"

namespace vx {

namespace {

template <class RowT>
__device__ __forceinline__ RowT row_at(const void* base, int64_t id, int64_t stride);
template <>
__device__ __forceinline__ RowF32 row_at<RowF32>(const void* base, int64_t id, int64_t stride) {
  return RowF32{(const float*)base + id * stride};
}
template <>
__device__ __forceinline__ RowF16 row_at<RowF16>(const void* base, int64_t id, int64_t stride) {
  return RowF16{(const __half*)base + id * stride};
}

template <class RowT>
__global__ void __launch_bounds__(256) rescore_kernel(RescoreArgs a) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int q = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t cap = a.cap;
  uint64_t* s_keys = (uint64_t*)smem_raw;
  uint64_t* s_tmp = s_keys + cap;
  uint32_t* s_red = (uint32_t*)(s_tmp + cap);
  uint32_t* s_counter = s_red + 32;
  __shared__ int s_complete;
  __shared__ uint32_t s_nres;

  const uint32_t c = a.cand_cnt[q];
  const uint64_t* cand = a.cand + (size_t)q * a.Kc;
  if (threadIdx.x == 0) {
    bool complete = true;
    if (a.n_rows <= (int64_t)a.Kc) {
      complete = true;  // every row is a candidate
    } else if (a.check_margin && c >= (uint32_t)a.Kc && a.Kc > a.k) {
      const float ak = key_score(cand[a.k - 1]);
      const float alast = key_score(cand[a.Kc - 1]);
      const float m = a.margin ? a.margin[q] : 0.0f;
      complete = alast < ak - 2.0f * m;  // false for NaN keys as well
    } else if (a.check_margin && c >= (uint32_t)a.Kc && a.Kc <= a.k) {
      complete = false;
    }
    s_complete = complete ? 1 : 0;
    s_nres = c;
    if (!complete) {
      int slot = atomicAdd(a.nflag, 1);
      a.flag_list[slot] = q;
    }
  }
  __syncthreads();
  if (!s_complete) return;
  // Candidates are sorted by approximate key.  With a margin, one whose approximate score is
  // below A_k - 2m has an exact key below every one of the k best approximate candidates'
  // exact keys, so only the prefix at or above A_k - 2m needs the exact score.
  if (a.check_margin && c > (uint32_t)a.k && a.n_rows > (int64_t)a.Kc) {
    const float cut = key_score(cand[a.k - 1]) - 2.0f * (a.margin ? a.margin[q] : 0.0f);
    for (uint32_t i = (uint32_t)a.k + threadIdx.x; i < c; i += blockDim.x)
      if (key_score(cand[i]) < cut && !(key_score(cand[i - 1]) < cut)) s_nres = i;  // first below
    __syncthreads();
  }
  const uint32_t nres = s_nres;

  RowF32 qrow{a.queries + (size_t)q * a.dim};
  for (uint32_t i = warp; i < nres; i += blockDim.x / 32) {
    const uint32_t id = key_id(cand[i]);
    RowT x = row_at<RowT>(a.rows, (int64_t)id, a.row_stride);
    const float s = warp_exact_score(a.flavor, a.metric, qrow, x, a.dim);
    if (lane == 0) s_keys[i] = float_key(s, id + a.id_offset);
  }
  __syncthreads();
  uint32_t n = nres;
  if (nres > 256) n = block_keep_top(s_keys, nres, (uint32_t)a.k, s_tmp, s_red, s_counter);
  block_sort_desc(s_keys, n, cap);
  if (n > (uint32_t)a.k) n = (uint32_t)a.k;
  // Fp16QuantizedVectors clamps DOT/COSINE scores at 0: if the cut falls on a clamped score,
  // rows tied at 0 are ranked by ordinal alone, which the approximate key cannot see.
  if (a.check_margin && a.flavor == kFlavorFp16Quantized && a.metric != kEuclidean &&
      a.metric != kMaxInnerProduct && n > 0 && !(key_score(s_keys[n - 1]) > 0.0f)) {
    if (threadIdx.x == 0) {
      int slot = atomicAdd(a.nflag, 1);
      a.flag_list[slot] = q;
    }
    return;
  }
  for (int i = threadIdx.x; i < a.k; i += blockDim.x) {
    const size_t o = (size_t)q * a.k + i;
    if ((uint32_t)i < n) {
      a.out_ids[o] = (int32_t)key_id(s_keys[i]);
      a.out_scores[o] = key_score(s_keys[i]);
    } else {
      a.out_ids[o] = -1;
      a.out_scores[o] = 0.0f;
    }
  }
  if (threadIdx.x == 0) a.out_counts[q] = (int32_t)n;
}

// Exact scan of every row for up to 8 queries (fallback).  Global warp w scores rows
// w, w + W, ...; lane f (< nfq) keeps warp w's candidate stream for query f.
template <class RowT, int R>
__global__ void __launch_bounds__(256) exact_scan_kernel(ExactScanArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t W = (int64_t)gridDim.x * (blockDim.x / 32);
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const bool owner = lane < a.nfq;
  const size_t sidx = (size_t)w * 8 + (owner ? lane : 0);
  LaneStream st;
  st.base = a.bufs + sidx * (size_t)a.C;
  st.cnt = 0;
  st.thr = owner ? 0ull : ~0ull;
  int since = 0;
  for (int64_t r = w; r < a.n; r += W) {
    RowT x = row_at<RowT>(a.rows, r, a.row_stride);
    for (int f = 0; f < a.nfq; f++) {
      RowF32 qrow{a.queries + (size_t)f * a.dim};
      const float s = warp_exact_score(a.flavor, a.metric, qrow, x, a.dim);
      if (lane == f) st.offer(float_key(s, (uint32_t)r));
    }
    if (++since == 32) {
      since = 0;
      warp_compact_lanes<R>(st.cnt > (uint32_t)(a.C - 32), st.base, st.cnt, st.thr, (uint32_t)a.K);
    }
  }
  warp_compact_lanes<R>(st.cnt > (uint32_t)a.K, st.base, st.cnt, st.thr, (uint32_t)a.K);
  if (lane < 8) a.cnts[(size_t)w * 8 + lane] = owner ? st.cnt : 0u;
}

}  // namespace

size_t rescore_smem(int Kc) {
  uint32_t cap = 1;
  while (cap < (uint32_t)Kc) cap <<= 1;
  return (size_t)cap * 16 + 33 * 4 + 16;
}

cudaError_t launch_rescore(RescoreArgs a, bool rows_f16, cudaStream_t st) {
  if (a.nq <= 0) return cudaSuccess;
  uint32_t cap = 1;
  while (cap < (uint32_t)a.Kc) cap <<= 1;
  a.cap = cap;
  size_t smem = rescore_smem(a.Kc);
  if (rows_f16) {
    cudaError_t e = cudaFuncSetAttribute(rescore_kernel<RowF16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    rescore_kernel<RowF16><<<a.nq, 256, smem, st>>>(a);
  } else {
    cudaError_t e = cudaFuncSetAttribute(rescore_kernel<RowF32>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    rescore_kernel<RowF32><<<a.nq, 256, smem, st>>>(a);
  }
  return cudaGetLastError();
}

int exact_scan_warps(int num_sms) { return num_sms * 2 * 8; }

cudaError_t launch_exact_scan(const ExactScanArgs& a, bool rows_f16, int R, int num_sms,
                              cudaStream_t st) {
  const int blocks = num_sms * 2;
#define VX_EX_CASE(RR)                                                             \
  case RR:                                                                         \
    if (rows_f16)                                                                  \
      exact_scan_kernel<RowF16, RR><<<blocks, 256, 0, st>>>(a);                    \
    else                                                                           \
      exact_scan_kernel<RowF32, RR><<<blocks, 256, 0, st>>>(a);                    \
    return cudaGetLastError();
  switch (R) {
    VX_EX_CASE(2)
    VX_EX_CASE(3)
    VX_EX_CASE(5)
    VX_EX_CASE(9)
    VX_EX_CASE(17)
    VX_EX_CASE(33)
    default: return cudaErrorInvalidValue;
  }
#undef VX_EX_CASE
}

}  // namespace vx
