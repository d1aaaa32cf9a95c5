/*
 * vx_oracle.h -- CPU oracle for the batch distance + top-k scan.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is a plain C++ restatement of the
 * integrallis/vectors Java hot path (FLAT exact search, the SQ8 / FP16 / sign-bit
 * BQ quantized scans and the IVF-PQ ADC list scan).  It exists so that tests,
 * the smoke check and the CPU-baseline leg of the benchmark can check and time
 * the CUDA product path.  Nothing in the product (libvx.so, the Python package)
 * links, loads or calls it.
 *
 * Every function cites the reference file:line it restates (paths relative to
 * the reference project root).  Floating-point evaluation order follows the
 * Java source: no contraction (built with -ffp-contract=off), std::fma only where
 * Java calls Math.fma / FloatVector.fma (vector and scalar FMA both on, the
 * reference default on x86: PanamaConstants.java:189-231), 8-lane (256-bit)
 * species (PanamaConstants.java:47).
 *
 * Parity pinning: the integer paths (byte dot, Hamming, PQ code gathers) and the
 * explicitly sequential float paths (PQ L2 table built from the scalar tail,
 * PQ sequential sum, SQ8 score epilogue, fp16 conversion) are fully determined
 * by the Java source.  The fp32 dot uses an explicit lane order
 * (PanamaVectorUtilSupport.java:1377-1386) and is pinned too.  squareDistance
 * and cosine end in FloatVector.reduceLanes(ADD), whose order the JVM does not
 * define; the oracle uses the same pairwise order as the dot product there
 * ("parity unpinned" at the last bit for those two reductions).
 */
#ifndef VX_ORACLE_H
#define VX_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* SimilarityFunction ordinals (vectors-core/.../SimilarityFunction.java:30-120). */
enum { VO_EUCLIDEAN = 0, VO_DOT_PRODUCT = 1, VO_COSINE = 2, VO_MAXIMUM_INNER_PRODUCT = 3 };

/* Top-k policies: 0 = the reference's bounded min-heap (admits score > root,
 * FlatScanAdapter.java:72-95), 1 = canonical (score desc, id asc; TopK.java:58-116). */
enum { VO_POLICY_REFERENCE_HEAP = 0, VO_POLICY_CANONICAL = 1 };

/* ---- java.util.Random (published LCG algorithm; used by ReservoirSampler and k-means++) ---- */
typedef struct {
  uint64_t seed;
  double next_next_gaussian;
  int32_t have_next_next_gaussian;
} vo_jrandom;
void vo_jrandom_init(vo_jrandom* r, int64_t seed);
int32_t vo_jrandom_next_int(vo_jrandom* r);
int32_t vo_jrandom_next_int_bound(vo_jrandom* r, int32_t bound);
int64_t vo_jrandom_next_long(vo_jrandom* r);
float vo_jrandom_next_float(vo_jrandom* r);
double vo_jrandom_next_double(vo_jrandom* r);
void vo_jrandom_next_bytes(vo_jrandom* r, int8_t* out, int32_t n);

/* ---- seeded synthetic data (SplitMix64 -> uniform doubles -> Box-Muller) ---- */
uint64_t vo_splitmix64_at(uint64_t seed, uint64_t index);
double vo_uniform_at(uint64_t seed, uint64_t index);
double vo_normal_at(uint64_t seed, uint64_t index);
/* Isotropic Gaussian mixture: centres ~ N(0,1)^dim (seed_centres), component ~ U{0..C-1},
 * x = centre + sigma * N(0,1)^dim (seed_points); rows [first_row, first_row + n).
 * normalize != 0 applies l2normalize (PanamaVectorUtilSupport.java:5178-5194). */
void vo_gen_mixture(float* out, int64_t first_row, int64_t n, int32_t dim, int32_t n_centres,
                    float sigma, uint64_t seed_centres, uint64_t seed_points, int32_t normalize,
                    int32_t nthreads);

/* ---- L0 kernels (vectors-core) ---- */
float vo_dot(const float* a, const float* b, int32_t len);
float vo_square_distance(const float* a, const float* b, int32_t len);
float vo_cosine(const float* a, const float* b, int32_t len);
float vo_compare(int32_t metric, const float* a, const float* b, int32_t len);
float vo_scale_mip(float dot);
void vo_l2normalize(float* v, int32_t len);
int32_t vo_byte_dot(const int8_t* a, const int8_t* b, int32_t len);
int32_t vo_byte_square_distance(const int8_t* a, const int8_t* b, int32_t len);
int32_t vo_hamming(const uint64_t* a, const uint64_t* b, int32_t nwords);
void vo_mat_vec_square_l2(const float* query, const float* rows, int32_t nrows, int32_t dim,
                          float* out);
void vo_mat_vec_dot(const float* query, const float* rows, int32_t nrows, int32_t dim, float* out);

/* ---- quantizers (vectors-quantization) ---- */
void vo_sq8_train(const float* data, int64_t n, int32_t dim, float confidence_interval,
                  float* min_q, float* max_q);
/* returns the per-vector correction; dst gets codes 0..127 */
float vo_sq8_encode(float min_q, float max_q, const float* v, int32_t dim, int8_t* dst);
float vo_sq8_score(int32_t metric, float min_q, float max_q, const int8_t* qcodes, float qcorr,
                   const int8_t* vcodes, float vcorr, int32_t dim);
void vo_bq_encode(const float* v, int32_t dim, uint64_t* words);
float vo_bq_score(int32_t metric, int32_t hamming, int32_t dim);
uint16_t vo_f32_to_f16(float f);
float vo_f16_to_f32(uint16_t h);
void vo_pq_subspaces(int32_t dim, int32_t m, int32_t* sizes_offsets /* [m][2] */);
/* ProductQuantizer.train(dataset, m, ks, center=false, trainThreads=1) on up to 25k reservoir rows */
void vo_pq_train(const float* data, int64_t n, int32_t dim, int32_t m, int32_t ks,
                 float* codebooks /* concatenated per subspace: ks * sub_m floats each */);
void vo_pq_encode(const float* v, int32_t dim, int32_t m, int32_t ks, const float* codebooks,
                  uint8_t* code);
void vo_pq_adc_table(const float* q, int32_t dim, int32_t m, int32_t ks, const float* codebooks,
                     int32_t use_dot, float* table /* [m][ks] */);
/* KMeans.train (vectors-core/.../cluster/KMeans.java:54-135) */
void vo_kmeans_train(const float* data, int64_t n, int32_t dim, int32_t k, int32_t max_iter,
                     int64_t seed, float* centroids, int32_t nthreads);
void vo_kmeans_assign(const float* data, int64_t n, int32_t dim, const float* centroids,
                      int32_t k, int32_t* out, int32_t nthreads);

/* batch encoders (Quantizer.encodeAll over n rows) */
void vo_sq8_encode_all(float min_q, float max_q, const float* data, int64_t n, int32_t dim,
                       int8_t* codes, float* corrections, int32_t nthreads);
void vo_bq_encode_all(const float* data, int64_t n, int32_t dim, uint64_t* words, int32_t nthreads);
void vo_fp16_encode_all(const float* data, int64_t n, int32_t dim, uint16_t* codes, int32_t nthreads);
void vo_pq_encode_all(const float* data, int64_t n, int32_t dim, int32_t m, int32_t ks,
                      const float* codebooks, uint8_t* codes, int32_t nthreads);

/* ---- searches: ids/scores are [nq][k] row-major, counts[nq] = valid entries ---- */
void vo_flat_search(const float* db, int64_t n, int32_t dim, int32_t metric, const float* queries,
                    int32_t nq, int32_t k, int32_t policy, int32_t nthreads, int32_t* ids,
                    float* scores, int32_t* counts);
void vo_sq8_search(const int8_t* codes, const float* corrections, int64_t n, int32_t dim,
                   float min_q, float max_q, int32_t metric, const float* queries, int32_t nq,
                   int32_t k, int32_t policy, int32_t nthreads, int32_t* ids, float* scores,
                   int32_t* counts);
float vo_sq_encode(float min_q, float max_q, int32_t max_value, const float* v, int32_t dim, int8_t* dst);
float vo_sq_score(int32_t metric, float min_q, float max_q, int32_t max_value, const int8_t* qc, float qcorr,
                  const int8_t* vc, float vcorr, int32_t dim);
void vo_sq_search(const int8_t* codes, const float* corr, int64_t n, int32_t dim, float min_q, float max_q,
                  int32_t max_value, int32_t metric, const float* queries, int32_t nq, int32_t k, int32_t policy,
                  int32_t nthreads, int32_t* ids, float* scores, int32_t* counts);
void vo_sq_encode_all(float min_q, float max_q, int32_t max_value, const float* data, int64_t n, int32_t dim,
                      int8_t* codes, float* corrections, int32_t nthreads);
void vo_bq_search(const uint64_t* words, int64_t n, int32_t dim, int32_t metric,
                  const float* queries, int32_t nq, int32_t k, int32_t policy, int32_t nthreads,
                  int32_t* ids, float* scores, int32_t* counts);
void vo_bbq_encode_all(const float* data, const float* cent, int64_t n, int32_t dim, uint64_t* words, float* corr,
                       int32_t nthreads);
void vo_bbq_search(const uint64_t* words, const float* corr, const float* cent, int64_t n, int32_t dim,
                   int32_t metric, const float* queries, int32_t nq, int32_t k, int32_t policy, int32_t nthreads,
                   int32_t* ids, float* scores, int32_t* counts);
void vo_fp16_search(const uint16_t* codes, int64_t n, int32_t dim, int32_t metric,
                    const float* queries, int32_t nq, int32_t k, int32_t policy, int32_t nthreads,
                    int32_t* ids, float* scores, int32_t* counts);
/* PQVectors.scoreFunctionFor (PQVectors.java:104-191): the k best rows by the PQ score; codebooks
 * concatenated per subspace (standard sizes), global_centroid NULL when the quantizer has none,
 * codes [n][m]. */
void vo_pq_flat_search(const float* codebooks, const float* global_centroid, const uint8_t* codes, int64_t n,
                       int32_t dim, int32_t m, int32_t ks, int32_t metric, const float* queries, int32_t nq,
                       int32_t k, int32_t policy, int32_t nthreads, int32_t* ids, float* scores, int32_t* counts);
/* QuantizedFlatScanAdapter.search (QuantizedFlatScanAdapter.java:59-95): kind 0=SQ8 1=BQ 2=FP16;
 * qdata/qaux are the kind's codes (and SQ8 corrections / quantiles in qaux[0..1]). */
void vo_quantized_two_pass_search(int32_t kind, const void* qdata, const float* qcorr,
                                  float min_q, float max_q, const float* db, int64_t n,
                                  int32_t dim, int32_t metric, const float* queries, int32_t nq,
                                  int32_t k, float over_query_factor, int32_t policy,
                                  int32_t nthreads, int32_t* ids, float* scores, int32_t* counts);
/* The exact second pass alone (QuantizedFlatScanAdapter.java:79-94): candidates cid[q*stride ..
 * + cnt[q]) re-scored with SimilarityFunction.compare on the fp32 rows, k best kept. */
void vo_rescore_candidates(const float* db, int32_t dim, int32_t metric, const float* queries, int32_t nq,
                           const int32_t* cid, int32_t stride, const int32_t* cnt, int32_t k, int32_t policy,
                           int32_t nthreads, int32_t* ids, float* scores, int32_t* counts);
/* IVF routing (CentroidIndex.routeWithSpillDistances with gamma == 0) */
void vo_route(const float* centroids, int32_t nlist, int32_t dim, int32_t metric,
              const float* queries, int32_t nq, int32_t nprobe, int32_t policy, int32_t nthreads,
              int32_t* list_ids /* [nq][nprobe] */, float* dists);
/* CentroidIndex.routeWithSpillDistances with SOAR spill (gamma > 0): up to 2*nprobe lists per
 * query in list_ids / dists [nq][2*nprobe], their number in counts[nq] */
void vo_route_spill(const float* centroids, int32_t nlist, int32_t dim, int32_t metric,
                    const float* queries, int32_t nq, int32_t nprobe, float gamma,
                    const int32_t* spill_targets, int32_t nthreads, int32_t* list_ids, float* dists,
                    int32_t* counts);
/* IvfIndex.pqSearch (IvfIndex.java:539-619); lists are CSR: list_offsets[nlist+1], list_ordinals */
void vo_ivfpq_search(const float* centroids, int32_t nlist, int32_t dim, const int64_t* list_offsets,
                     const int32_t* list_ordinals, int32_t m, int32_t ks, const float* codebooks,
                     const uint8_t* codes /* [n][m], ordinal order */, int64_t n, int32_t metric,
                     const float* queries, int32_t nq, int32_t k, int32_t nprobe,
                     int32_t rescore_factor, const float* vectors /* for rescore; may be NULL */,
                     int32_t policy, int32_t nthreads, int32_t* ids, float* scores,
                     int32_t* counts);
/* IvfIndex.search without PQ (IvfIndex.java:170-277), every probed cluster scanned */
void vo_ivfflat_search(const float* centroids, int32_t nlist, int32_t dim, const int64_t* list_offsets,
                       const int32_t* list_ordinals, const float* vectors, int64_t n, int32_t metric,
                       const float* queries, int32_t nq, int32_t k, int32_t nprobe, int32_t policy,
                       int32_t nthreads, int32_t* ids, float* scores, int32_t* counts);
/* The same with the reference's EUCLIDEAN triangle-inequality early exit (IvfIndex.java:190-200)
 * against per-cluster radii (BuoyIndex.clusterRadii); other metrics ignore radii. */
/* IvfIndex.pqSearch with gamma > 0: clusters of routeWithSpillDistances, SOAR spill targets
 * (spill_targets[nlist], -1 = none) appended (canonical ranking). */
void vo_ivfpq_search_spill(const float* centroids, int32_t nlist, int32_t dim, const int64_t* list_offsets,
                           const int32_t* list_ordinals, int32_t m, int32_t ks, const float* codebooks,
                           const uint8_t* codes, int64_t n, int32_t metric, const float* queries, int32_t nq,
                           int32_t k, int32_t nprobe, float gamma, const int32_t* spill_targets, int32_t rescore,
                           const float* vectors, int32_t nthreads, int32_t* ids, float* scores, int32_t* counts);
/* IvfIndex.search without PQ in full: SOAR spill routing (gamma > 0), for EUCLIDEAN the early
 * exit against radii (NULL radii: every probed cluster scanned) and the HARMONY scan of partitions
 * with key dimensions (kd_off[nlist + 1] / kd: CSR, NULL: none) (canonical ranking). */
void vo_ivfflat_search_spill(const float* centroids, int32_t nlist, int32_t dim, const int64_t* list_offsets,
                             const int32_t* list_ordinals, const float* vectors, int32_t metric, const float* radii,
                             const float* queries, int32_t nq, int32_t k, int32_t nprobe, float gamma,
                             const int32_t* spill_targets, const int64_t* kd_off, const int32_t* kd,
                             int32_t nthreads, int32_t* ids, float* scores, int32_t* counts);
void vo_ivfflat_search_early_exit(const float* centroids, int32_t nlist, int32_t dim,
                                  const int64_t* list_offsets, const int32_t* list_ordinals,
                                  const float* vectors, int64_t n, int32_t metric, const float* radii,
                                  const float* queries, int32_t nq, int32_t k, int32_t nprobe,
                                  int32_t policy, int32_t nthreads, int32_t* ids, float* scores,
                                  int32_t* counts);
/* BuoyIndex.computeRadii (BuoyIndex.java:175-183): per cluster, the largest
 * (float) sqrt(sum of (v - c)^2) over its members (sequential float sum); 0 for empty lists. */
void vo_ivf_radii(const float* centroids, int32_t nlist, int32_t dim, const int64_t* list_offsets,
                  const int32_t* list_ordinals, const float* vectors, float* radii);
/* IndexShards.mergeWithOffsets (IndexShards.java:168-211); policy 0 = reference partial
 * selection sort (earlier shard wins ties), 1 = canonical. */
void vo_merge_shards(int32_t nshards, const int64_t* offsets, const int32_t* shard_ids,
                     const float* shard_scores, const int32_t* shard_counts, int32_t kin,
                     int32_t nq, int32_t k, int32_t policy, int32_t* ids, float* scores,
                     int32_t* counts);
/* canonical top-k of an arbitrary score list (TopK.select, TopK.java:58-116) */
int32_t vo_topk_select(const float* scores, int32_t n, int32_t k, int32_t* out);

#ifdef __cplusplus
}
#endif
#endif /* VX_ORACLE_H */
