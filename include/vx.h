/*
 * vx.h -- C ABI of libvx.so, the B200 (sm_100a) batch distance + top-k scan behind the
 * integrallis/vectors index SPI.
 *
 * The entry points are what a Java 25 Foreign Function & Memory binding of the reference's
 * IndexSpi backends would call (Linker.nativeLinker().downcallHandle, the pattern of
 * vectors-storage/.../io/MadviseUtil.java:52-58).  Plain pointers and sizes only; every
 * function returns a vx_status and leaves a message for vx_last_error() on failure.
 *
 * Conventions
 *   - Ordinals are int32 (0..n-1), scores are float32 on the reference's scale, results are
 *     ordered by (score desc, ordinal asc), the canonical order of TopK.select
 *     (vectors-core/.../TopK.java:58-116).
 *   - Output arrays are [nq][k] row-major; out_counts[q] valid entries per query (<= k; the
 *     unused tail holds ordinal -1, score 0).
 *   - "host" entry points take host buffers (pinned or pageable) and block until the results
 *     are in them; "_device" entry points take device pointers and a cudaStream_t (as void*)
 *     and return once the work is queued, except where a query needs the exact fallback scan,
 *     which synchronises the stream internally.
 *   - An index is safe for concurrent searches from several host threads; builds and frees
 *     must not overlap searches on the same index (the facade's read/write lock,
 *     FlatScanAdapter.java:31-33).
 */
#ifndef VX_H
#define VX_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VX_ABI_VERSION 1

#if defined(__GNUC__)
#define VX_API __attribute__((visibility("default")))
#else
#define VX_API
#endif

/* Status codes.  The Java shim maps them onto the reference's exceptions. */
typedef enum vx_status {
  VX_OK = 0,
  VX_ERR_INVALID_ARGUMENT = 1, /* IllegalArgumentException (FlatScanAdapter.java:53-62,108-135) */
  VX_ERR_NULL_POINTER = 2,     /* NullPointerException (Objects.requireNonNull) */
  VX_ERR_GPU_UNAVAILABLE = 3,  /* GpuUnavailableException (CuVsBruteForceAdapter.java:67-70) */
  VX_ERR_CUDA = 4,             /* GpuUnavailableException wrapping a native failure (:86-89,117-119) */
  VX_ERR_OUT_OF_MEMORY = 5,
  VX_ERR_UNSUPPORTED = 6,      /* UnsupportedOperationException */
  VX_ERR_DEVICE_TIMEOUT = 7,   /* a bounded device-side wait expired; the context stays usable */
  VX_ERR_FORMAT = 8            /* java.io.IOException: a quantized.bin / graph.bin that does not decode
                                  (QuantizedVectorsCodec.java:131-192) */
} vx_status;

/* SimilarityFunction ordinals (vectors-core/.../SimilarityFunction.java:30-120). */
typedef enum vx_metric {
  VX_EUCLIDEAN = 0,
  VX_DOT_PRODUCT = 1,
  VX_COSINE = 2,
  VX_MAXIMUM_INNER_PRODUCT = 3
} vx_metric;

typedef enum vx_index_kind {
  VX_KIND_FLAT = 0,  /* IndexType.FLAT, QuantizerKind.NONE  -> FlatScanAdapter          */
  VX_KIND_FP16 = 1,  /* QuantizerKind.FP16 -> QuantizedFlatScanAdapter(Fp16QuantizedVectors) */
  VX_KIND_SQ8 = 2,   /* QuantizerKind.SQ8  -> QuantizedFlatScanAdapter(ScalarQuantizedVectors) */
  VX_KIND_BQ = 3,    /* QuantizerKind.BQ (SIGN_BIT) -> QuantizedFlatScanAdapter(BinaryQuantizedVectors) */
  VX_KIND_IVFPQ = 4, /* IndexType.IVF_PQ -> IvfPqAdapter / IvfIndex.pqSearch                 */
  VX_KIND_IVFFLAT = 5, /* IndexType.IVF_FLAT -> IvfFlatAdapter / IvfIndex.search (no PQ)      */
  VX_KIND_SQ4 = 6,     /* QuantizerKind.SQ4 -> QuantizedFlatScanAdapter(ScalarQuantizedVectors INT4) */
  VX_KIND_BBQ = 7,     /* QuantizerKind.BQ, BinaryMode.BBQ -> QuantizedFlatScanAdapter(BinaryQuantizedVectors) */
  VX_KIND_PQ = 8       /* QuantizerKind.PQ -> QuantizedFlatScanAdapter(PQVectors) */
} vx_index_kind;

typedef struct vx_index vx_index;

/* ---- library ------------------------------------------------------------------------ */
VX_API int vx_abi_version(void);
/* Message of the last failed call on this host thread ("" if none). */
VX_API const char* vx_last_error(void);
/* Number of usable CUDA devices; GpuProvider.availability() (vectors-gpu/.../GpuProvider.java). */
VX_API int vx_device_count(int32_t* count);
/* Kernels launched by this library since load (cumulative, all threads). */
VX_API int vx_kernel_launches(int64_t* count);
/* Per-kernel device timing.  When enabled, the library records CUDA events on the launching
 * stream around its main kernels; vx_profile_read waits for them and returns the accumulated
 * device milliseconds and launch count of one slot.  No counterpart in the reference (which
 * reports only SearchResult.searchTimeNanos, vectors-db/.../SearchResult.java:31). */
typedef enum vx_profile_slot {
  VX_PROF_GEMM_SCAN = 0, /* tcgen05 FLAT / FP16 / SQ8 scan */
  VX_PROF_MERGE = 1,     /* per-query candidate merge */
  VX_PROF_RESCORE = 2,   /* exact fp32 re-score */
  VX_PROF_FALLBACK = 3,  /* exact fallback scan */
  VX_PROF_BQ_SCAN = 4,   /* Hamming scan */
  VX_PROF_ADC_SCAN = 5,  /* IVF-PQ table build + ADC list scan */
  VX_PROF_ROUTE = 6,     /* IVF coarse routing */
  VX_PROF_PILOT = 7,     /* pilot sweep that seeds the admission floors of the tcgen05 scan */
  VX_PROF_SLOTS = 8
} vx_profile_slot;
VX_API int vx_profile_enable(int32_t on);
VX_API int vx_profile_read(int32_t slot, double* total_ms, int64_t* launches);
VX_API int vx_profile_reset(void);
/* Test hook: the next vx_* call on this host thread fails with `status` before touching the
 * GPU (host-side fault injection; status 0 clears it). */
VX_API int vx_debug_fail_next(int32_t status);
/* Test hook: one kernel whose only thread waits, with the scan pipeline's bounded wait, on a
 * barrier that nothing completes; after timeout_ms (1..10000) the wait gives up, the kernel
 * records the timeout and returns, and the call returns VX_ERR_DEVICE_TIMEOUT -- the status a
 * scan returns when one of its waits runs out.  The context stays usable.  No counterpart in the
 * reference. */
VX_API int vx_debug_wait_timeout(int32_t device, int32_t timeout_ms);

/* ---- index construction (the handle owns device copies; inputs are not retained) ----- */
/* Input arrays of the build calls may be host or device memory (unified addressing), except
 * the partitions (list_offsets, list_ordinals) of vx_ivfpq_build and vx_ivfflat_build and the
 * codes of vx_ivfpq_build, which are validated or regrouped on the host and must be host memory.
 * FlatScanAdapter.build(float[][] vectors, SimilarityFunction metric)
 * (vectors-db/.../index/FlatScanAdapter.java:42-48).  row_stride in floats (>= dim); use
 * alignUp(dim*4, 64)/4 to read a persistent vectors.bin (MemorySegmentVectors.java:39-45). */
VX_API int vx_flat_build(int32_t device, const float* vectors, int64_t n, int32_t dim, int64_t row_stride,
                  int32_t metric, vx_index** out);
/* Fp16QuantizedVectors (vectors-quantization/.../Fp16QuantizedVectors.java:40-94) wrapped as in
 * QuantizedFlatScanAdapter (vectors-db/.../index/QuantizedFlatScanAdapter.java:34-51).  codes:
 * [n][dim] little-endian binary16 (Fp16Quantizer.encode, Fp16Quantizer.java:72-85).  vectors
 * (fp32, optional) enable the exact rescore of vx_search_batch; NULL keeps codes only. */
VX_API int vx_fp16_build(int32_t device, const uint16_t* codes, int64_t n, int32_t dim, int32_t metric,
                  const float* vectors, int64_t row_stride, vx_index** out);
/* ScalarQuantizedVectors INT8 (ScalarQuantizedVectors.java:40-107): codes [n][dim] in 0..127,
 * per-row corrections, the quantizer's quantiles (ScalarQuantizer.fromQuantiles,
 * ScalarQuantizer.java:144-151). */
VX_API int vx_sq8_build(int32_t device, const int8_t* codes, const float* corrections, int64_t n,
                 int32_t dim, float min_quantile, float max_quantile, int32_t metric,
                 const float* vectors, int64_t row_stride, vx_index** out);
/* ScalarQuantizedVectors INT4 (ScalarQuantizedVectors.java:110-140, ScalarQuantizer.java:285-351):
 * packed codes [n][ceil(dim/2)] (low nibble = even dimension, high nibble = odd), per-row
 * corrections, the quantiles.  Scored as scoreFunctionInt4 does: the codes unpacked one per
 * byte (0..15), the exact int32 dot or squared distance, then the INT8 formulas with
 * maxValue 15. */
VX_API int vx_sq4_build(int32_t device, const uint8_t* packed, const float* corrections, int64_t n,
                        int32_t dim, float min_quantile, float max_quantile, int32_t metric,
                        const float* vectors, int64_t row_stride, vx_index** out);
/* BinaryQuantizedVectors SIGN_BIT (BinaryQuantizedVectors.java:40-107): words [n][ceil(dim/64)]
 * as produced by BinaryQuantizer.packBits + bytesToLongs (BinaryQuantizer.java:207-232).  Scanned
 * on the int8 tensor cores against a +-1 copy of the bits: kept whole (8 bytes per stored bit)
 * within VX_BQ_TENSOR_BYTES, else expanded one row window at a time during each search (scratch
 * of at most VX_BQ_WINDOW_BYTES); with windows off (VX_BQ_WINDOW_BYTES=0) by the popcount scan.
 * Both budgets are read from the environment at each build. */
VX_API int vx_bq_build(int32_t device, const uint64_t* words, int64_t n, int32_t dim, int32_t metric,
                const float* vectors, int64_t row_stride, vx_index** out);
/* BinaryQuantizedVectors BBQ (BinaryQuantizedVectors.java:110-275, BinaryQuantizer.java:199-270):
 * words [n][ceil(dim/64)] of the centroid-relative sign bits, corrections [n][3] =
 * (|v - c|^2, vl, width), the centroid [dim].  Scored as bbqScoreFunction does: the query
 * centred and quantised to 4 bits, rawAsymDot exactly (the 4-bit codes times a 0/1 int8 copy of
 * the bits on the int8 tensor cores: kept whole, 8 bytes of device memory per stored bit, within
 * the VX_BQ_TENSOR_BYTES budget; above it expanded one row window at a time during each search,
 * in scratch of at most VX_BQ_WINDOW_BYTES; with windows off (VX_BQ_WINDOW_BYTES=0), popcounts
 * of the query's 4 bit planes), computeBbqDot and the metric's transform in the Java float order.
 * dim <= 2048 (above 1024 only the tensor scan serves BBQ: windows must be on when the whole
 * operand exceeds VX_BQ_TENSOR_BYTES). */
VX_API int vx_bbq_build(int32_t device, const uint64_t* words, const float* corrections, const float* centroid,
                        int64_t n, int32_t dim, int32_t metric, const float* vectors, int64_t row_stride,
                        vx_index** out);
/* PQVectors (vectors-quantization/.../PQVectors.java:40-191) wrapped as in QuantizedFlatScanAdapter:
 * a ProductQuantizer with m subspaces of ks centroids (ProductQuantizer.fromState), codebooks
 * concatenated per subspace with computeSubspaceSizesAndOffsets' sizes (ProductQuantizer.java:686-700),
 * the global centroid [dim] or NULL, codes [n][m] (host memory).  Scored as scoreFunctionFor does:
 * buildADCTable of the query minus the global centroid, the sequential fp32 sum of the m entries,
 * then the metric's PQVectors transform (COSINE with the centred query norm and the rows' summed
 * centroid norms).  vectors (fp32, optional) enable the exact rescore of vx_search_batch. */
VX_API int vx_pq_build(int32_t device, const float* codebooks, const float* global_centroid, const uint8_t* codes,
                       int64_t n, int32_t dim, int32_t m, int32_t ks, int32_t metric, const float* vectors,
                       int64_t row_stride, vx_index** out);
/* IvfIndex.fromPrebuilt(buoy, partitions, vectors, metric, pq, codes)
 * (vectors-ivf/.../IvfIndex.java:343-351): centroids [nlist][dim]; partitions as CSR
 * (list_offsets[nlist+1], list_ordinals); PQ with m subspaces of ks centroids, codebooks
 * concatenated per subspace (ProductQuantizer.codebooks(), subspace sizes from
 * computeSubspaceSizesAndOffsets, ProductQuantizer.java:686-700), no global centroid; codes
 * [n][m] in ordinal order (IvfIndex.java:59).  nprobe / rescore_factor are the adapter's
 * defaults (IvfPqAdapter.java:84-109); vectors (optional) enable rescore_factor > 1.  The lists
 * may hold a subset of the n coded rows (list_offsets[nlist] <= n): a list-sharded index keeps
 * only its own lists, with global ordinals. */
VX_API int vx_ivfpq_build(int32_t device, const float* centroids, int32_t nlist, int32_t dim,
                   const int64_t* list_offsets, const int32_t* list_ordinals, int32_t m, int32_t ks,
                   const float* codebooks, const uint8_t* codes, int64_t n, int32_t metric,
                   const float* vectors, int32_t nprobe, int32_t rescore_factor, vx_index** out);
/* IvfIndex without PQ (IndexType.IVF_FLAT: IvfFlatAdapter.java:30-150, IvfIndex.search
 * :170-289): centroids and partitions as for vx_ivfpq_build, and the fp32 rows [n] row_stride
 * floats apart (host or device; a mapped vectors.bin with alignUp(dim*4, 64)/4).
 * vx_search_batch follows IvfFlatAdapter.search (searchListSize overrides nprobe,
 * overQueryFactor > 1 widens the probes); vx_ivfpq_search* run IvfIndex.search's flat list scan
 * (their rescore_factor is ignored: the scan is exact) for k <= 256. */
VX_API int vx_ivfflat_build(int32_t device, const float* centroids, int32_t nlist, int32_t dim,
                            const int64_t* list_offsets, const int32_t* list_ordinals, const float* vectors,
                            int64_t n, int64_t row_stride, int32_t metric, int32_t nprobe, vx_index** out);
/* ---- persistent files (host memory; the bytes are not retained) --------------------------
 * quantized.bin as written by QuantizedVectorsCodec.encode and read by .decode
 * (vectors-db/.../storage/QuantizedVectorsCodec.java:91-192): little-endian, header magic 'VQTZ'
 * (FileFormat.java:77), version 1, QuantizerKind ordinal, dimension, vectorCount.  SQ8 / SQ4
 * (:224-296), BQ SIGN_BIT and BBQ (:425-518), FP16 (:194-221) and PQ (:298-420) payloads build the
 * index vx_sq8_build / vx_sq4_build / vx_bq_build / vx_bbq_build / vx_fp16_build / vx_pq_build would;
 * PQ with subspaces other than computeSubspaceSizesAndOffsets', RABITQ, NVQ, TURBOQUANT and
 * EXTENDED_RABITQ return VX_ERR_UNSUPPORTED.  The collection's metric is not stored in the file.  vectors
 * (optional) are the fp32 rows for the two-pass rescore, e.g. a mapped vectors.bin with
 * row_stride = alignUp(dim*4, 64)/4.  Malformed bytes return VX_ERR_FORMAT with the decoder's
 * message. */
VX_API int vx_quantized_bin_info(const uint8_t* bytes, int64_t len, int32_t* kind_ordinal, int32_t* dim,
                                 int64_t* count);
VX_API int vx_quantized_bin_build(int32_t device, const uint8_t* bytes, int64_t len, int32_t metric,
                                  const float* vectors, int64_t row_stride, vx_index** out);
/* graph.bin of an IVF_PQ or IVF_FLAT generation: the bytes of IvfIndex.encode
 * (vectors-ivf/.../IvfIndex.java:354-400; decode :408-442, PQ trailer :450-500) around
 * BuoyIndex.encode (BuoyIndex.java:130-167), big-endian as java.nio.ByteBuffer and
 * java.io.DataOutputStream write them; read by VectorCollectionImpl.openIvfFlatAdapter /
 * openIvfPqAdapter (VectorCollectionImpl.java:684-718).  With a PQ trailer it builds the index
 * vx_ivfpq_build would (vectors, optional, enable rescore_factor > 1 and must number the codes);
 * without one, the index vx_ivfflat_build would from the caller's vectors (required, as
 * IvfIndex.decode takes them).  metric -1 takes the routing metric recorded in the file; another
 * metric must equal it.  PQ with a global centroid or non-standard subspaces returns
 * VX_ERR_UNSUPPORTED; HARMONY key dimensions are read and not used.  vx_ivf_graph_info reports
 * m = 0 and count = the partitioned rows for an IVF-flat file. */
VX_API int vx_ivf_graph_info(const uint8_t* bytes, int64_t len, int32_t* nlist, int32_t* dim, int64_t* count,
                             int32_t* m, int32_t* metric);
VX_API int vx_ivf_graph_build(int32_t device, const uint8_t* bytes, int64_t len, int32_t metric,
                              const float* vectors, int64_t vector_count, int64_t row_stride, int32_t nprobe,
                              int32_t rescore_factor, vx_index** out);
/* The BuoyIndex state an IVF index routes with beyond its centroids (IvfIndex.fromPrebuilt takes
 * a BuoyIndex; vectors-ivf/.../BuoyIndex.java:130-167): radii [nlist], the largest distance from
 * each centroid to a row of its cluster (BuoyIndex.clusterRadii), and SOAR spill targets [nlist]
 * (BuoyIndex.spillTargets, -1 = none).  NULL leaves that part unchanged.  vx_ivfflat_build
 * computes the radii from its partitions as BuoyIndex.computeRadii does (:175-183); graph.bin
 * builds take both from the file.  The IVF-flat EUCLIDEAN search stops early with them as
 * IvfIndex.search does (IvfIndex.java:190-205).  Must not overlap searches on the index. */
VX_API int vx_ivf_set_buoy(vx_index* index, const float* radii, const int32_t* spill_targets);
/* ClusterPartition.keyDimensions of an IVF-flat index's partitions (IvfIndex.build with
 * harmonyKeyDims > 0): key_dim_counts [nlist], the number of key dimensions of each list (0 =
 * none; NULL clears).  A EUCLIDEAN search that reaches such a list with a full heap scores its rows
 * with squareDistance, as scanPartitionWithHarmony does (IvfIndex.java:214-216,279-289); graph.bin
 * builds read the counts from the file.  Must not overlap searches on the index. */
VX_API int vx_ivf_set_key_dims(vx_index* index, const int32_t* key_dim_counts);
/* The adapter's SOAR spill ratio at search time (IvfPqAdapter / IvfFlatAdapter gamma,
 * IvfSearchRequest.gamma >= 0, IvfSearchRequest.java:40; default 0 = no spill).  With gamma > 0
 * and spill targets set, vx_search_batch and vx_ivfpq_search* route with
 * CentroidIndex.routeWithSpillDistances' additions (CentroidIndex.java:155-187).  The routed
 * entry points (vx_ivf_route_device, vx_ivfpq_search_routed_device) route and scan without spill
 * and without the early exit.  Must not overlap searches on the index. */
VX_API int vx_ivf_set_gamma(vx_index* index, float gamma);
/* IndexSpi.size() and the index's shape. */
VX_API int vx_index_info(const vx_index* index, int32_t* kind, int64_t* size, int32_t* dim,
                  int32_t* metric);
/* IndexSpi.close() (IndexSpi.java:157-159). */
VX_API int vx_index_free(vx_index* index);

/* ---- search --------------------------------------------------------------------------- */
/* IndexSpi.searchBatch(float[][] queries, int k, int searchListSize, float overQueryFactor)
 * (IndexSpi.java:127-152; FlatScanAdapter.java:106-175; QuantizedFlatScanAdapter.java:59-95;
 * IvfPqAdapter.java:124-158).  queries: [nq][dim] fp32. */
VX_API int vx_search_batch(vx_index* index, const float* queries, int32_t nq, int32_t dim, int32_t k,
                    int32_t search_list_size, float over_query_factor, int32_t* out_ids,
                    float* out_scores, int32_t* out_counts);
VX_API int vx_search_batch_device(vx_index* index, const float* d_queries, int32_t nq, int32_t dim,
                           int32_t k, int32_t search_list_size, float over_query_factor,
                           int32_t* d_ids, float* d_scores, int32_t* d_counts, void* stream);
/* QuantizedFlatScanAdapter.selectApproximateCandidates (QuantizedFlatScanAdapter.java:97-113):
 * the k best rows by the compressed ScoreFunction (SQ8 / SQ4 / BQ / BBQ / FP16 / PQ scores), no rescore. */
VX_API int vx_scan_candidates(vx_index* index, const float* queries, int32_t nq, int32_t dim, int32_t k,
                       int32_t* out_ids, float* out_scores, int32_t* out_counts);
VX_API int vx_scan_candidates_device(vx_index* index, const float* d_queries, int32_t nq, int32_t dim,
                              int32_t k, int32_t* d_ids, float* d_scores, int32_t* d_counts,
                              void* stream);
/* IvfIndex.search(new IvfSearchRequest(query, k, nprobe, 0f, minScore, rescoreFactor))
 * (IvfIndex.java:170-171,539-619; IvfSearchRequest.java:32-65). */
VX_API int vx_ivfpq_search(vx_index* index, const float* queries, int32_t nq, int32_t dim, int32_t k,
                    int32_t nprobe, int32_t rescore_factor, float min_score, int32_t* out_ids,
                    float* out_scores, int32_t* out_counts);
VX_API int vx_ivfpq_search_device(vx_index* index, const float* d_queries, int32_t nq, int32_t dim,
                           int32_t k, int32_t nprobe, int32_t rescore_factor, float min_score,
                           int32_t* d_ids, float* d_scores, int32_t* d_counts, void* stream);
/* The two halves of vx_ivfpq_search_device, for row-sharded search where every GPU holds the
 * same centroids: CentroidIndex.routeWithSpillDistances with gamma = 0 (CentroidIndex.java:89-211,
 * the routing step of IvfIndex.pqSearch, IvfIndex.java:545-547) writes the min(nprobe, nlist)
 * nearest lists of each query to d_lists [nq][min(nprobe, nlist)], ascending distance, ties by
 * lower list id; the routed search then scans those lists (ids outside [-1, nlist) are
 * rejected with VX_ERR_INVALID_ARGUMENT, -1 means no list).  Routing a slice of the queries on
 * each GPU and exchanging the lists gives the same results as routing everything everywhere. */
VX_API int vx_ivf_route_device(vx_index* index, const float* d_queries, int32_t nq, int32_t dim,
                        int32_t nprobe, int32_t* d_lists, void* stream);
VX_API int vx_ivfpq_search_routed_device(vx_index* index, const float* d_queries, int32_t nq, int32_t dim,
                                  int32_t k, int32_t nprobe, int32_t rescore_factor, float min_score,
                                  const int32_t* d_lists, int32_t* d_ids, float* d_scores,
                                  int32_t* d_counts, void* stream);
/* IvfIndex.search (IvfIndex.java:170-226) on an IVF-flat index split across GPUs by (query,
 * list) pair, in three steps whose results equal vx_ivfpq_search_device's (same lists, same
 * early exit).  Routing: as vx_ivf_route_device, plus each routed list's distance
 * (d_list_dist [nq][min(nprobe, nlist)], the value the early exit's triangle bound reads,
 * IvfIndex.java:198-205).  Scan: the list scan of the slots of d_lists [nq][min(nprobe, nlist)]
 * that hold a list id (-1: a slot another GPU scans) into per-slot results d_pair_keys
 * [min(nprobe, nlist)][nq][min(k, n)] (64-bit keys: order-preserving score bits above
 * 0xFFFFFFFF - ordinal) and d_pair_counts [min(nprobe, nlist)][nq]; the other slots are zeroed,
 * so adding the buffers of GPUs that scanned disjoint slots (an NCCL sum all-reduce) combines
 * them.  Merge: the combined per-slot results taken in route order with the EUCLIDEAN early
 * exit when the index holds BuoyIndex radii (else the k best of all slots), then minScore, into
 * d_ids / d_scores [nq][k] and d_counts [nq].  Not for partitions with HARMONY key dimensions
 * or k above 256 (VX_ERR_UNSUPPORTED); no SOAR spill (gamma is not applied).  The scan takes
 * the whole batch in one pass (its scratch grows with nq); callers split very large batches. */
VX_API int vx_ivf_route_dist_device(vx_index* index, const float* d_queries, int32_t nq, int32_t dim,
                                    int32_t nprobe, int32_t* d_lists, float* d_list_dist, void* stream);
VX_API int vx_ivfflat_scan_pairs_device(vx_index* index, const float* d_queries, int32_t nq, int32_t dim,
                                        int32_t k, int32_t nprobe, const int32_t* d_lists,
                                        uint64_t* d_pair_keys, uint32_t* d_pair_counts, void* stream);
VX_API int vx_ivfflat_merge_pairs_device(vx_index* index, int32_t nq, int32_t k, int32_t nprobe,
                                         const int32_t* d_lists, const float* d_list_dist,
                                         const uint64_t* d_pair_keys, const uint32_t* d_pair_counts,
                                         float min_score, int32_t* d_ids, float* d_scores, int32_t* d_counts,
                                         void* stream);

/* No counterpart in the reference.  The sign-bit BQ candidate scan of vx_scan_candidates_device
 * for callers that must not allocate device memory while searching (a host that reserves its
 * whole device budget up front and accounts every byte, or a latency-critical loop where an
 * allocation would block on the allocator or synchronise the device).  Its scratch is a
 * file-scope 64 MiB device array; no cudaMalloc, cudaFree or pool allocation happens in the
 * call.  With CUDA's default lazy module loading the array is placed on a device by the first
 * vx_bq_build there (which looks it up with cudaGetSymbolAddress), not when the library is
 * loaded, and stays until the process exits; with CUDA_MODULE_LOADING=EAGER every context
 * holds it from load.  If that placement failed, the call returns VX_ERR_OUT_OF_MEMORY.
 * All calls on a device share the array: calls that overlap on the GPU race and must be
 * serialised by the caller.  Batches needing more than 64 MiB of scratch are rejected with
 * VX_ERR_INVALID_ARGUMENT and a message giving the largest batch that fits for the index and
 * k (about 175 queries at k = 100 on a large index; split the batch).  Queries and outputs are
 * device buffers. */
VX_API int vx_bq_scan_candidates_noalloc(vx_index* index, const float* d_queries, int32_t nq,
                                         int32_t dim, int32_t k, int32_t* d_ids, float* d_scores,
                                         int32_t* d_counts, void* stream);

/* ---- shards ---------------------------------------------------------------------------- */
/* IndexShards.mergeWithOffsets (vectors-db/.../index/IndexShards.java:168-211): shard s holds
 * shard_counts[s*nq+q] (ordinal, score) pairs of query q at [(s*nq+q)*kin]; ordinals are
 * shifted by offsets[s]; result: the k best by (score desc, ordinal asc).  Device buffers. */
VX_API int vx_merge_shards_device(int32_t device, int32_t nshards, const int64_t* d_offsets,
                           const int32_t* d_shard_ids, const float* d_shard_scores,
                           const int32_t* d_shard_counts, int32_t kin, int32_t nq, int32_t k,
                           int32_t* d_ids, float* d_scores, int32_t* d_counts, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* VX_H */
