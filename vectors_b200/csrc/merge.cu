// merge.cu -- per-query merge of candidate streams, key -> (id, score) finishing, and the
// cross-shard merge (IndexShards.mergeWithOffsets, vectors-db/.../index/IndexShards.java:168-211).
#include "kernels.h"
#include "select.cuh"

namespace vx {

// Shared-memory key slots of the stream merge: the sort window (a power of two) and at
// least K plus one stream's worth of keys.
__host__ __device__ __forceinline__ uint32_t merge_cap(int C, int K) {
  uint32_t need = (uint32_t)K + (uint32_t)(C > 1024 ? C : 1024);
  return need > 2048u ? need : 2048u;
}

// Each block merges the candidate streams of one query into its K best keys, sorted
// descending.  Stream s of query q holds cnts[s*nq+q] keys at bufs + ((s*nq)+q)*C, where nq
// is the stream stride (queries beyond the grid are padding and are not merged).
//
// Keys below the query's shared floor cannot reach its top K (at least K keys score at or
// above the floor), so only keys >= floor are gathered.  The stream counts of up to 256
// streams are read at once and prefix-summed, and their keys are gathered as one flat
// index range.  The gathered keys are usually a few hundred: they are sorted outright;
// larger sets are first cut to K by the bitwise K-th search.
constexpr int kMergeThreads = 256;
constexpr uint32_t kMergeSortMax = 1024;  // gathered keys sorted without a prior cut

__device__ __forceinline__ uint32_t block_excl_scan_u32(uint32_t v, uint32_t* s_red, uint32_t& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += t;
  }
  __syncthreads();
  if (lane == 31) s_red[warp] = incl;
  __syncthreads();
  uint32_t before = 0;
  total = 0;
  for (int i = 0; i < nw; i++) {
    const uint32_t w = s_red[i];
    before += i < warp ? w : 0u;
    total += w;
  }
  return before + incl - v;
}

__global__ void __launch_bounds__(kMergeThreads) merge_streams_kernel(const uint64_t* __restrict__ bufs,
                                                                      const uint32_t* __restrict__ cnts,
                                                                      int S, int nq, int C, int K,
                                                                      const uint64_t* __restrict__ floor,
                                                                      uint64_t* __restrict__ out_keys,
                                                                      uint32_t* __restrict__ out_cnt) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int q = blockIdx.x;
  const uint32_t cap = merge_cap(C, K);
  uint64_t* s_keys = (uint64_t*)smem_raw;
  uint64_t* s_tmp = s_keys + cap;
  uint32_t* s_red = (uint32_t*)(s_tmp + cap);
  uint32_t* s_counter = s_red + 32;
  __shared__ uint32_t s_n;
  __shared__ uint32_t s_off[kMergeThreads + 1];
  const uint64_t f = floor ? floor[q] : 0ull;
  uint32_t n = 0;
  if (threadIdx.x == 0) s_n = 0;
  for (int s0 = 0; s0 < S; s0 += kMergeThreads) {
    const int ns = min(kMergeThreads, S - s0);
    const uint32_t c = (int)threadIdx.x < ns ? cnts[(size_t)(s0 + threadIdx.x) * nq + q] : 0u;
    uint32_t total;
    const uint32_t excl = block_excl_scan_u32(c, s_red, total);
    s_off[threadIdx.x] = excl;
    if (threadIdx.x == 0) s_off[kMergeThreads] = total;
    __syncthreads();
    for (uint32_t base = 0; base < total;) {
      if (n + min(total - base, 1024u) > cap) {  // rare: cut to K before gathering more
        n = block_keep_top(s_keys, n, (uint32_t)K, s_tmp, s_red, s_counter);
        if (threadIdx.x == 0) s_n = n;
        __syncthreads();
      }
      const uint32_t take = min(total - base, cap - n);
      for (uint32_t i = threadIdx.x; i < take; i += blockDim.x) {
        const uint32_t idx = base + i;
        int lo = 0, hi = ns - 1;  // last stream whose offset <= idx
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (s_off[mid] <= idx) lo = mid; else hi = mid - 1;
        }
        const uint64_t key = bufs[((size_t)(s0 + lo) * nq + q) * (size_t)C + (idx - s_off[lo])];
        if (key >= f) s_keys[atomicAdd(&s_n, 1u)] = key;
      }
      __syncthreads();
      n = s_n;
      base += take;
      __syncthreads();
    }
  }
  if (n > kMergeSortMax) n = block_keep_top(s_keys, n, (uint32_t)K, s_tmp, s_red, s_counter);
  block_sort_desc(s_keys, n, cap);
  const uint32_t kept = n < (uint32_t)K ? n : (uint32_t)K;
  for (uint32_t i = threadIdx.x; i < (uint32_t)K; i += blockDim.x)
    out_keys[(size_t)q * K + i] = (i < kept) ? s_keys[i] : kEmptyKey;
  if (threadIdx.x == 0) out_cnt[q] = kept;
}

size_t merge_streams_smem(int C, int K) { return (size_t)merge_cap(C, K) * 16 + 33 * 4 + 16; }

cudaError_t launch_merge_streams(const uint64_t* bufs, const uint32_t* cnts, int S, int nq,
                                 int stride, int C, int K, uint64_t* out_keys, uint32_t* out_cnt,
                                 cudaStream_t st, const uint64_t* floor) {
  if (nq <= 0) return cudaSuccess;
  size_t smem = merge_streams_smem(C, K);
  cudaError_t e = cudaFuncSetAttribute(merge_streams_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  merge_streams_kernel<<<nq, kMergeThreads, smem, st>>>(bufs, cnts, S, stride, C, K, floor, out_keys, out_cnt);
  return cudaGetLastError();
}

// Admission floors from a probe sweep: probe[q][g] is query q's largest score over the g-th
// group of 32 rows, so the K-th largest group maximum x is reached by K distinct rows and the
// query's K-th best key is at least (bits(x), any id).  One warp per query, bitwise search
// for the K-th largest of the G order-preserving score bits.
__global__ void probe_floor_kernel(const float* __restrict__ probe, int nq, int G, int K,
                                   uint64_t* __restrict__ floor) {
  const int q = (int)((blockIdx.x * (size_t)blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (q >= nq) return;
  const float* row = probe + (size_t)q * G;
  uint32_t t = 0;
  for (int b = 31; b >= 0; b--) {
    const uint32_t cand = t | (1u << b);
    uint32_t c = 0;
    for (int i = lane; i < G; i += 32) c += float_order_bits(row[i]) >= cand ? 1u : 0u;
    c = __reduce_add_sync(0xFFFFFFFFu, c);
    if (c >= (uint32_t)K) t = cand;
  }
  if (lane == 0) floor[q] = (G >= K && t > 0) ? ((uint64_t)t << 32) : 0ull;
}

cudaError_t launch_probe_floor(const float* probe, int nq, int G, int K, uint64_t* floor, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  probe_floor_kernel<<<(nq * 32 + 255) / 256, 256, 0, st>>>(probe, nq, G, K, floor);
  return cudaGetLastError();
}

// Converts sorted keys to the reference's (ordinal, score) output.  kind selects how the
// score is recovered: the key's float bits (exact scores), or a Hamming distance mapped
// through BinaryQuantizedVectors.signBitScoreFunction (BinaryQuantizedVectors.java:88-106).
__global__ void finish_keys_kernel(const uint64_t* __restrict__ keys, const uint32_t* __restrict__ cnt,
                                   int nq, int K, int k_out, int kind, int metric, int dim,
                                   int32_t* __restrict__ ids, float* __restrict__ scores,
                                   int32_t* __restrict__ counts) {
  int q = blockIdx.x;
  int c = (int)cnt[q];
  if (c > k_out) c = k_out;
  __syncthreads();
  for (int i = threadIdx.x; i < k_out; i += blockDim.x) {
    if (i < c) {
      uint64_t key = keys[(size_t)q * K + i];
      ids[(size_t)q * k_out + i] = (int32_t)key_id(key);
      float s;
      if (kind == kFinishHamming) {
        uint32_t h = 0xFFFFFFFFu - key_hi(key);
        s = bq_score_device(metric, (int)h, dim);
      } else if (kind == kFinishNegHamming) {
        s = bq_score_device(metric, (int)(-key_score(key)), dim);
      } else {
        s = key_score(key);
      }
      scores[(size_t)q * k_out + i] = s;
    } else {
      ids[(size_t)q * k_out + i] = -1;
      scores[(size_t)q * k_out + i] = 0.0f;
    }
  }
  if (threadIdx.x == 0) counts[q] = c;
}

// Drops the trailing hits scoring below min_score (results are sorted descending), as
// IvfIndex.pqSearch does with IvfSearchRequest.minScore (IvfIndex.java:592-616).
__global__ void min_score_kernel(const float* __restrict__ scores, int nq, int k, float min_score,
                                 int32_t* __restrict__ counts) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  int c = counts[q];
  while (c > 0 && scores[(size_t)q * k + c - 1] < min_score) c--;
  counts[q] = c;
}

cudaError_t launch_min_score(const float* scores, int nq, int k, float min_score, int32_t* counts,
                             cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  min_score_kernel<<<(nq + 127) / 128, 128, 0, st>>>(scores, nq, k, min_score, counts);
  return cudaGetLastError();
}

// Packs (ordinal, score) outputs into keys (counts may be < K).
__global__ void ids_to_keys_kernel(const int32_t* __restrict__ ids, const int32_t* __restrict__ cnt,
                                   int nq, int K, uint64_t* __restrict__ keys) {
  const int q = blockIdx.x;
  for (int i = threadIdx.x; i < K; i += blockDim.x)
    keys[(size_t)q * K + i] = i < cnt[q] ? make_key(0u, (uint32_t)ids[(size_t)q * K + i]) : kEmptyKey;
}

cudaError_t launch_ids_to_keys(const int32_t* ids, const int32_t* cnt, int nq, int K, uint64_t* keys,
                               cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  ids_to_keys_kernel<<<nq, 128, 0, st>>>(ids, cnt, nq, K, keys);
  return cudaGetLastError();
}

// Gathers rows src[map[i]] (dim floats each) into dst[i].
__global__ void gather_rows_kernel(const float* __restrict__ src, const int32_t* __restrict__ map, int m,
                                  int dim, float* __restrict__ dst) {
  const int i = blockIdx.x;
  if (i >= m) return;
  const float* s = src + (size_t)map[i] * dim;
  for (int d = threadIdx.x; d < dim; d += blockDim.x) dst[(size_t)i * dim + d] = s[d];
}

cudaError_t launch_gather_rows(const float* src, const int32_t* map, int m, int dim, float* dst,
                               cudaStream_t st) {
  if (m <= 0) return cudaSuccess;
  gather_rows_kernel<<<m, 128, 0, st>>>(src, map, m, dim, dst);
  return cudaGetLastError();
}

// Writes per-query results computed for a subset back to their places: row i of the subset
// goes to query map[i].
__global__ void scatter_results_kernel(const int32_t* __restrict__ ids, const float* __restrict__ sc,
                                       const int32_t* __restrict__ cnt, const int32_t* __restrict__ map,
                                       int m, int k, int32_t* __restrict__ out_ids,
                                       float* __restrict__ out_sc, int32_t* __restrict__ out_cnt) {
  const int i = blockIdx.x;
  if (i >= m) return;
  const int q = map[i];
  for (int j = threadIdx.x; j < k; j += blockDim.x) {
    out_ids[(size_t)q * k + j] = ids[(size_t)i * k + j];
    out_sc[(size_t)q * k + j] = sc[(size_t)i * k + j];
  }
  if (threadIdx.x == 0) out_cnt[q] = cnt[i];
}

cudaError_t launch_scatter_results(const int32_t* ids, const float* sc, const int32_t* cnt,
                                   const int32_t* map, int m, int k, int32_t* out_ids, float* out_sc,
                                   int32_t* out_cnt, cudaStream_t st) {
  if (m <= 0) return cudaSuccess;
  scatter_results_kernel<<<m, 128, 0, st>>>(ids, sc, cnt, map, m, k, out_ids, out_sc, out_cnt);
  return cudaGetLastError();
}

cudaError_t launch_finish_keys(const uint64_t* keys, const uint32_t* cnt, int nq, int K, int k_out,
                               int kind, int metric, int dim, int32_t* ids, float* scores,
                               int32_t* counts, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  finish_keys_kernel<<<nq, 128, 0, st>>>(keys, cnt, nq, K, k_out, kind, metric, dim, ids, scores,
                                         counts);
  return cudaGetLastError();
}

// Passes of a candidate search wider than one stream: ceil[q] = the smallest key kept so far
// when the query's previous pass was full (there may be more rows below it), else 0 (none).
__global__ void pass_ceilings_kernel(const uint64_t* __restrict__ keys, const uint32_t* __restrict__ cnt, int nq,
                                     int K, int got, uint64_t* __restrict__ ceil) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  ceil[q] = cnt[q] == (uint32_t)got ? keys[(size_t)q * K + got - 1] : 0ull;
}

// Appends a pass's sorted keys (all below the query's ceiling) after the keys kept so far.
__global__ void pass_append_kernel(uint64_t* __restrict__ keys, uint32_t* __restrict__ cnt, int nq, int K, int got,
                                   const uint64_t* __restrict__ keys2, const uint32_t* __restrict__ cnt2, int K2) {
  const int q = blockIdx.x;
  if (cnt[q] != (uint32_t)got) return;  // the earlier passes already hold every row
  const uint32_t c2 = cnt2[q];
  for (uint32_t i = threadIdx.x; i < c2; i += blockDim.x) keys[(size_t)q * K + got + i] = keys2[(size_t)q * K2 + i];
  __syncthreads();
  if (threadIdx.x == 0) cnt[q] = (uint32_t)got + c2;
}

cudaError_t launch_pass_ceilings(const uint64_t* keys, const uint32_t* cnt, int nq, int K, int got, uint64_t* ceil,
                                 cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  pass_ceilings_kernel<<<(nq + 255) / 256, 256, 0, st>>>(keys, cnt, nq, K, got, ceil);
  return cudaGetLastError();
}

cudaError_t launch_pass_append(uint64_t* keys, uint32_t* cnt, int nq, int K, int got, const uint64_t* keys2,
                               const uint32_t* cnt2, int K2, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  pass_append_kernel<<<nq, 128, 0, st>>>(keys, cnt, nq, K, got, keys2, cnt2, K2);
  return cudaGetLastError();
}

// Row windows: both inputs hold a query's keys in descending order; a window key's ordinal is
// local, and make_key stores 0xFFFFFFFF - id, so key - base carries the ordinal id + base.  The
// windows come in ordinal order, so a later row whose score equals the K-th kept key's ranks
// below it (TopK.select's ordinal tie rule): seed (the K-th key with every id bit set) admits in
// the next window only higher scores (and local ordinal 0 at an equal score, which the next
// merge ranks correctly).  One thread per query.
__global__ void window_merge_kernel(const uint64_t* __restrict__ run, const uint32_t* __restrict__ run_cnt,
                                    const uint64_t* __restrict__ win, const uint32_t* __restrict__ win_cnt, int nq,
                                    int K, uint32_t base, uint64_t* __restrict__ out, uint32_t* __restrict__ out_cnt,
                                    uint64_t* __restrict__ seed) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  const uint32_t cr = run ? min(run_cnt[q], (uint32_t)K) : 0u;
  const uint32_t cw = min(win_cnt[q], (uint32_t)K);
  const uint64_t* r = run + (size_t)q * K;
  const uint64_t* w = win + (size_t)q * K;
  uint64_t* o = out + (size_t)q * K;
  uint32_t i = 0, j = 0, n = 0;
  uint64_t a = cr ? r[0] : kEmptyKey;
  uint64_t b = cw ? w[0] - base : kEmptyKey;
  while (n < (uint32_t)K && (i < cr || j < cw)) {
    if (i < cr && (j >= cw || a > b)) {
      o[n++] = a;
      a = ++i < cr ? r[i] : kEmptyKey;
    } else {
      o[n++] = b;
      b = ++j < cw ? w[j] - base : kEmptyKey;
    }
  }
  for (uint32_t t = n; t < (uint32_t)K; t++) o[t] = kEmptyKey;
  out_cnt[q] = n;
  seed[q] = n == (uint32_t)K ? (o[K - 1] | 0xFFFFFFFFull) : 0ull;
}

cudaError_t launch_window_merge(const uint64_t* run, const uint32_t* run_cnt, const uint64_t* win,
                                const uint32_t* win_cnt, int nq, int K, uint32_t base, uint64_t* out,
                                uint32_t* out_cnt, uint64_t* seed, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  window_merge_kernel<<<(nq + 127) / 128, 128, 0, st>>>(run, run_cnt, win, win_cnt, nq, K, base, out, out_cnt,
                                                        seed);
  return cudaGetLastError();
}

// Cross-shard merge: shard s contributes shard_counts[s*nq+q] (ordinal, score) pairs for
// query q at [(s*nq+q)*kin]; ordinals are shifted by offsets[s].  Output: the k best by
// (score desc, ordinal asc), the canonical order of TopK.select.
__global__ void __launch_bounds__(256) merge_shards_kernel(
    int nshards, const int64_t* __restrict__ offsets, const int32_t* __restrict__ sids,
    const float* __restrict__ ssc, const int32_t* __restrict__ scnt, int kin, int nq, int k,
    uint32_t total_cap, int32_t* __restrict__ ids, float* __restrict__ scores,
    int32_t* __restrict__ counts) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  const int q = blockIdx.x;
  uint64_t* s_keys = (uint64_t*)smem_raw;
  uint64_t* s_tmp = s_keys + total_cap;
  uint32_t* s_red = (uint32_t*)(s_tmp + total_cap);
  uint32_t* s_counter = s_red + 32;
  if (threadIdx.x == 0) *s_counter = 0;
  __syncthreads();
  for (int s = 0; s < nshards; s++) {
    int c = scnt[(size_t)s * nq + q];
    for (int i = threadIdx.x; i < c; i += blockDim.x) {
      size_t at = ((size_t)s * nq + q) * kin + i;
      uint32_t id = (uint32_t)((int64_t)sids[at] + offsets[s]);
      s_keys[atomicAdd(s_counter, 1u)] = float_key(ssc[at], id);
    }
  }
  __syncthreads();
  uint32_t n = *s_counter;
  __syncthreads();
  n = block_keep_top(s_keys, n, (uint32_t)k, s_tmp, s_red, s_counter);
  block_sort_desc(s_keys, n, total_cap);
  for (int i = threadIdx.x; i < k; i += blockDim.x) {
    if ((uint32_t)i < n) {
      ids[(size_t)q * k + i] = (int32_t)key_id(s_keys[i]);
      scores[(size_t)q * k + i] = key_score(s_keys[i]);
    } else {
      ids[(size_t)q * k + i] = -1;
      scores[(size_t)q * k + i] = 0.0f;
    }
  }
  if (threadIdx.x == 0) counts[q] = (int32_t)n;
}

cudaError_t launch_merge_shards(int nshards, const int64_t* offsets, const int32_t* sids,
                                const float* ssc, const int32_t* scnt, int kin, int nq, int k,
                                int32_t* ids, float* scores, int32_t* counts, cudaStream_t st) {
  if (nq <= 0) return cudaSuccess;
  size_t cap = (size_t)nshards * kin;
  uint32_t p = 1;
  while (p < cap) p <<= 1;
  if (p > cap) cap = p;  // bitonic padding room
  size_t smem = cap * 16 + 33 * 4 + 16;
  cudaError_t e = cudaFuncSetAttribute(merge_shards_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  merge_shards_kernel<<<nq, 256, smem, st>>>(nshards, offsets, sids, ssc, scnt, kin, nq, k,
                                             (uint32_t)cap, ids, scores, counts);
  return cudaGetLastError();
}

}  // namespace vx
