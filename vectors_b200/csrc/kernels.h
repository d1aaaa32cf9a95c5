// kernels.h -- launch entry points of the scan kernels (internal to libvx.so).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace vx {

// SimilarityFunction ordinals (vectors-core/.../SimilarityFunction.java:30-120).
enum Metric : int { kEuclidean = 0, kDotProduct = 1, kCosine = 2, kMaxInnerProduct = 3 };

enum FinishKind : int {
  kFinishFloatKey = 0,    // key high word = order bits of the reference score
  kFinishHamming = 1,     // key high word = 0xFFFFFFFF - Hamming distance
  kFinishNegHamming = 2,  // key high word = order bits of -(Hamming distance) (tensor BQ scan)
};

// Which reference score an exact re-score reproduces (exact.cuh).
enum ScoreFlavor : int { kFlavorFlat = 0, kFlavorFp16Quantized = 1, kFlavorIvfRaw = 2 };

// SimilarityFunction.scaleMaxInnerProductScore (SimilarityFunction.java:155-161).
__host__ __device__ __forceinline__ float scale_mip(float dot) {
#ifdef __CUDA_ARCH__
  return dot >= 0.0f ? __fadd_rn(dot, 1.0f) : __fdiv_rn(1.0f, __fsub_rn(1.0f, dot));
#else
  return dot >= 0.0f ? dot + 1.0f : 1.0f / (1.0f - dot);
#endif
}

// BinaryQuantizedVectors.signBitScoreFunction (BinaryQuantizedVectors.java:88-106).
__host__ __device__ __forceinline__ float bq_score_device(int metric, int h, int dim) {
#ifdef __CUDA_ARCH__
  switch (metric) {
    case kEuclidean: return __fdiv_rn(1.0f, __fadd_rn(1.0f, __fmul_rn(4.0f, (float)h)));
    case kMaxInnerProduct: return scale_mip(__fdiv_rn((float)(dim - 2 * h), (float)dim));
    default: return __fsub_rn(1.0f, __fdiv_rn((float)h, (float)dim));
  }
#else
  switch (metric) {
    case kEuclidean: return 1.0f / (1.0f + 4.0f * (float)h);
    case kMaxInnerProduct: return scale_mip((float)(dim - 2 * h) / (float)dim);
    default: return 1.0f - (float)h / (float)dim;
  }
#endif
}

// Candidate-stream geometry shared by the scan kernels: a stream keeps up to K keys in a
// buffer of C = 32*R slots; at most `slack` keys are appended between two compaction checks.
struct StreamGeom {
  int K;      // keys each stream must keep
  int R;      // registers per lane used by the warp compaction (C = 32 * R)
  int C;      // buffer slots per stream
};
StreamGeom stream_geom(int K, int slack);

// ---- merge.cu
cudaError_t launch_merge_streams(const uint64_t* bufs, const uint32_t* cnts, int S, int nq,
                                 int stride, int C, int K, uint64_t* out_keys, uint32_t* out_cnt,
                                 cudaStream_t st, const uint64_t* floor = nullptr);
cudaError_t launch_probe_floor(const float* probe, int nq, int G, int K, uint64_t* floor, cudaStream_t st);
cudaError_t launch_ids_to_keys(const int32_t* ids, const int32_t* cnt, int nq, int K, uint64_t* keys,
                               cudaStream_t st);
cudaError_t launch_gather_rows(const float* src, const int32_t* map, int m, int dim, float* dst,
                               cudaStream_t st);
cudaError_t launch_scatter_results(const int32_t* ids, const float* sc, const int32_t* cnt,
                                   const int32_t* map, int m, int k, int32_t* out_ids, float* out_sc,
                                   int32_t* out_cnt, cudaStream_t st);
cudaError_t launch_min_score(const float* scores, int nq, int k, float min_score, int32_t* counts,
                             cudaStream_t st);
cudaError_t launch_finish_keys(const uint64_t* keys, const uint32_t* cnt, int nq, int K, int k_out,
                               int kind, int metric, int dim, int32_t* ids, float* scores,
                               int32_t* counts, cudaStream_t st);
// Candidate searches wider than one stream, pass by pass (merge.cu).
cudaError_t launch_pass_ceilings(const uint64_t* keys, const uint32_t* cnt, int nq, int K, int got, uint64_t* ceil,
                                 cudaStream_t st);
cudaError_t launch_pass_append(uint64_t* keys, uint32_t* cnt, int nq, int K, int got, const uint64_t* keys2,
                               const uint32_t* cnt2, int K2, cudaStream_t st);
// Row windows of a BQ / BBQ scan (merge.cu): the best K keys so far (run: global ordinals;
// null on the first window) merged with one window's sorted keys (ordinals local to the window,
// shifted by base) into out; seed[q] = the next window's admission floor.
cudaError_t launch_window_merge(const uint64_t* run, const uint32_t* run_cnt, const uint64_t* win,
                                const uint32_t* win_cnt, int nq, int K, uint32_t base, uint64_t* out,
                                uint32_t* out_cnt, uint64_t* seed, cudaStream_t st);
cudaError_t launch_merge_shards(int nshards, const int64_t* offsets, const int32_t* sids,
                                const float* ssc, const int32_t* scnt, int kin, int nq, int k,
                                int32_t* ids, float* scores, int32_t* counts, cudaStream_t st);

// ---- bq_scan.cu : sign-bit Hamming scan (BinaryQuantizedVectors.java:81-107)
// db: [n][nw_pad] 64-bit words; qw: [nq][nw_pad]; writes S = parts streams per query.
int bq_padded_words(int nw);
int bq_parts(int64_t n, int num_sms);
cudaError_t launch_bq_scan(const uint64_t* db, int64_t n, int nw_pad, const uint64_t* qw, int nq,
                           int parts, const StreamGeom& g, uint64_t* bufs, uint32_t* cnts,
                           uint64_t* thrs, cudaStream_t st);
cudaError_t launch_bq_pack_queries(const float* q, int nq, int dim, int nw_pad, uint64_t* out,
                                   cudaStream_t st);

// BBQ (BinaryQuantizedVectors.java:110-275): per-query terms of bbqScoreFunction, 4 bit planes
// [nq][4][nw_pad] of the 4-bit query; per-row (|v - c|^2, vl, width, popcount) records.
struct BbqQuery {
  float qmin, w15, nsq, norm;  // queryMin, queryWidth / 15, queryNormSq, queryNorm
  int32_t qsum, pad0, pad1, pad2;
};
bool bbq_supported(int nw_pad);  // up to 1024 dimensions
cudaError_t launch_bbq_prep_queries(const float* q, int nq, int dim, const float* centroid, int nw_pad,
                                    uint64_t* planes, BbqQuery* info, cudaStream_t st);
cudaError_t launch_bbq_rowinfo(const uint64_t* words, int nw, int nw_pad, const float* corr, int64_t n, float4* out,
                               cudaStream_t st);
// int8 tensor-core BBQ scan (gemm_scan.cu, kEpiBbq*): per-row (vl, width, vl * D + width * pop,
// |v - c| (COSINE) or |v - c|^2) records, and the 4-bit query codes as int8 rows of Dp8 bytes.
cudaError_t launch_bbq_epi_rows(const float4* info, int64_t n, int dim, int metric, float4* out, cudaStream_t st);
cudaError_t launch_bbq_planes_to_i8(const uint64_t* planes, int nq, int dim, int nw_pad, int Dp8, int8_t* dst,
                                    cudaStream_t st);
cudaError_t launch_bbq_scan(const uint64_t* db, const float4* rowinfo, int64_t n, int nw_pad, int dim, int metric,
                            const uint64_t* planes, const BbqQuery* qinfo, int nq, int parts, const StreamGeom& g,
                            uint64_t* bufs, uint32_t* cnts, uint64_t* thrs, cudaStream_t st);

}  // namespace vx
