// ivfpq.h -- IVF-PQ routing and ADC scan (ivfpq.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace vx {

struct AdcArgs {
  int nq, dim, nprobe, metric;
  int M, Ks, Mp;                 // subspaces, centroids per subspace, padded code bytes per row
  int K;                         // keys kept per (query, list)
  int64_t npairs;                // routed pairs (nq * nprobe)
  const int32_t* pairs;          // pair indices (q * nprobe + p), grouped by list
  const int32_t* pair_count;     // device count of the grouped pairs
  const int32_t* lists;          // [nq][nprobe] routed list ids
  const float* queries;          // [nq][dim]
  const float* cent;             // [nlist][dim]
  const int64_t* list_off;       // [nlist + 1] CSR offsets into codes / ordinals
  const int32_t* ordinals;       // [n] ordinal of each list-ordered row
  const uint8_t* codes;          // [n][Mp] list-ordered PQ codes
  const float* codebooks;        // concatenated, subspace m at cb_off[m]
  const int64_t* cb_off;         // [M]
  const int32_t* sub;            // [M][2] size, offset
  uint64_t* out;                 // [nprobe][nq][K]
  uint32_t* out_cnt;             // [nprobe][nq]
  // grouped scan only (adc_group_kernel)
  const int2* groups;            // (first pair slot, pairs) of up to 4 pairs sharing one list
  int32_t* ngroups;              // [0] device count of groups, [1] the group dispenser
  uint64_t* floor;               // [nq] per-query admission floor shared across lists (zeroed)
  // PQ as a flat quantizer (PQVectors, one list holding every row): tables of (query - global
  // centroid) for every metric, and PQVectors' score of the sum instead of IvfIndex's
  int pq_flat = 0;
  const float* qnorm = nullptr;  // [nq] |query - global centroid| (COSINE)
  const float* rnorm = nullptr;  // [n] per list-ordered row: sum of centroidNormSq[m][code[m]] (COSINE)
};

cudaError_t launch_route(const float* queries, int nq, int dim, const float* cent, int nlist,
                         int metric, int nprobe, float* qnorm_scratch, float* dist,
                         int32_t* lists, cudaStream_t st);
cudaError_t launch_copy_lists(const int32_t* src, int n, int nlist, int32_t* dst, int32_t* bad, cudaStream_t st);
int route_launches(const float* queries, int dim, const float* cent, int nlist, int metric);
// Buckets the (query, probe) pairs by list: only routed pairs (list id >= 0) whose list holds
// rows on this device; offsets[nlist] is the number of such pairs.
cudaError_t launch_group_pairs(const int32_t* lists, const int64_t* list_off, int npairs, int nlist,
                               int32_t* counts, int32_t* offsets, int32_t* cursor, int32_t* pairs,
                               cudaStream_t st);
size_t adc_smem(int M, int Ks, int dim, int R, int K);
cudaError_t launch_adc_scan(const AdcArgs& a, int R, int grid, cudaStream_t st);

// Grouped ADC scan for 8-dimensional subspaces with 256 centroids (M a multiple of 16):
// pairs sharing a list are taken up to four at a time.
constexpr int kAdcGroupQ = 4;
bool adc_group_supported(int M, int Ks, int dim);
// Groups of up to `wmax` (<= 255) consecutive pairs of one list: groups[i] = (first pair slot,
// pairs), lists taken in `order` (null: by id; longest first balances the scans).  With rmax > 0
// a list of more than rmax rows (list_off) gives each pair group once per row part of rmax
// rows: groups[i].y = pairs | part << 8.  ngroups[0] is the count and ngroups[1] the dispenser
// the grouped scans take groups from (zeroed here).
cudaError_t launch_make_groups(const int32_t* counts, const int32_t* offsets, const int32_t* order, int nlist,
                               int wmax, int2* groups, int32_t* ngroups, cudaStream_t st,
                               const int64_t* list_off = nullptr, int rmax = 0);
cudaError_t launch_adc_group(const AdcArgs& a, int R, int grid, cudaStream_t st);

// IVF-flat list scan (IvfIndex.search without PQ): pairs grouped by list, up to 64 per group.
struct FlatListArgs {
  int nq, dim, Dp, nprobe, metric, K;
  const int32_t* pairs;       // pair indices (q * nprobe + p), grouped by list
  const int32_t* pair_count;  // device count of the grouped pairs
  const int2* groups;         // (first pair slot, pairs) of up to 64 pairs sharing one list
  int32_t* ngroups;           // [0] count, [1] dispenser
  const int32_t* lists;       // [nq][nprobe] routed list ids
  const float* queries;       // [nq][Dp] zero-padded copy
  const float* qnorm;         // [nq] dotProduct(q, q) (COSINE)
  const int64_t* list_off;    // [nlist + 1]
  const int32_t* ordinals;    // [n] ordinal of each list-ordered row
  const float* rows;          // [n][Dp] list-ordered rows, zero-padded
  const float* rnorm;         // [n] dotProduct(v, v) of the list-ordered rows (COSINE)
  float* tail;                // [pairs][3] raw scores of each list's last-batch trailing rows
  uint64_t* out;              // [nprobe][nq][K]
  uint32_t* out_cnt;          // [nprobe][nq]
  uint64_t* floor;            // [nq] per-query admission floor across lists (zeroed); null: each
                              // (query, list) keeps its own best K (the early exit's input)
  // Row parts (rmax > 0): a list of more than rmax rows is scanned by one group per part of rmax
  // rows (a multiple of 64), so that no single group bounds the kernel; each part's K best go to
  // part_out [pair position][pmax][K] / part_cnt [pair position][pmax] (pair position: index into
  // pairs) and launch_flat_parts_merge combines the parts into out.
  int rmax, pmax;
  uint64_t* part_out;
  uint32_t* part_cnt;
};
constexpr int kFlatGroup = 64;
// Keys kept per (query, list) that the scan supports: K <= 256.
bool flat_list_supported(int K);
cudaError_t launch_pad_rows(const float* src, int64_t n, int dim, int64_t src_stride, const int32_t* map, int Dp,
                            float* dst, cudaStream_t st);
cudaError_t launch_row_norms(const float* rows, int64_t n, int dim, int Dp, float* out, cudaStream_t st);
// flat_tail_kernel then flat_list_kernel (2 launches)
cudaError_t launch_flat_list(const FlatListArgs& a, int64_t pair_slots, int grid, cudaStream_t st);
// The row parts of every pair whose list has more than one (a.rmax > 0): the K best of the
// parts' keys into out / out_cnt, one warp per pair; pmax * K <= kFlatPartKeysMax.
constexpr int kFlatPartKeysMax = 1024;
cudaError_t launch_flat_parts_merge(const FlatListArgs& a, int64_t pair_slots, cudaStream_t st);

// PQVectors (PQVectors.java:62-89, 148-166): |q - gc| per query (sequential sum of squares,
// (float) Math.sqrt), and per row the sequential sum over subspaces of the centroids' squared
// norms (centroidNormSq, each a sequential sum of squares over the subspace).
cudaError_t launch_pq_query_norms(const float* queries, int nq, int dim, const float* gc, float* out,
                                  cudaStream_t st);
cudaError_t launch_pq_row_norms(const uint8_t* codes, int64_t n, int M, int Mp, int Ks, const int32_t* sub,
                                const float* codebooks, const int64_t* cb_off, float* cnorm_scratch, float* out,
                                cudaStream_t st);

// CentroidIndex.routeWithSpillDistances' SOAR additions: lists [nq][probes] (ascending) and the
// routing distances [nq][nlist] -> out_lists / out_dist [nq][width] (primaries, then spill
// targets when gamma > 0 and spill is set, -1 past the count) with each cluster's distance.
cudaError_t launch_route_expand(const int32_t* lists, int nq, int probes, const float* dist, int nlist, int metric,
                                float gamma, const int32_t* spill, int width, int32_t* out_lists, float* out_dist,
                                cudaStream_t st);
// BuoyIndex.computeRadii over the list-ordered rows [n][Dp] (radii [nlist], overwritten).
cudaError_t launch_list_radii(const float* rows, int64_t n, int dim, int Dp, const int64_t* list_off, int nlist,
                              const float* cent, float* radii, cudaStream_t st);
// The per-(probe, query) list results merged per query in route order, with IvfIndex.search's
// EUCLIDEAN early exit (other metrics: a plain merge); keys [nq][K] sorted descending, kcnt [nq].
// harm / harm_cnt / keyed (nullable): the HARMONY results of lists with key dimensions, taken
// instead of out when the query's heap is full at that list.
bool early_exit_supported(int K);
cudaError_t launch_ivf_early_exit(const uint64_t* out, const uint32_t* out_cnt, int nq, int width, int K,
                                  const int32_t* lists, const float* ldist, const float* radii, int metric,
                                  float min_score, const uint64_t* harm, const uint32_t* harm_cnt,
                                  const uint8_t* keyed, uint64_t* keys, uint32_t* kcnt, cudaStream_t st);
// HARMONY (IvfIndex.scanPartitionWithHarmony): for every (query, slot) whose list is keyed, the K
// best rows by -squareDistance(query, row) in the reference's order -> harm [width][nq][K].
struct HarmonyArgs {
  int nq, width, K, dim, Dp;
  const int32_t* lists;       // [nq][width]
  const uint8_t* keyed;       // [nlist]
  const int64_t* list_off;
  const int32_t* ordinals;    // list-ordered
  const float* rows;          // [n][Dp] list-ordered, zero padded
  const float* queries;       // [nq][Dp] zero padded
  uint64_t* out;              // [width][nq][K]
  uint32_t* out_cnt;          // [width][nq]
};
cudaError_t launch_harmony_lists(const HarmonyArgs& a, cudaStream_t st);

}  // namespace vx
