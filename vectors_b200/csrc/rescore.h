// rescore.h -- exact fp32 re-scoring of candidates and the exact fallback scan.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace vx {

struct RescoreArgs {
  int nq, dim, k, Kc;
  int flavor, metric;           // ScoreFlavor, Metric
  const float* queries;         // [nq][dim] fp32, as the caller passed them
  const void* rows;             // fp32 or fp16 rows
  int64_t row_stride;           // elements between rows
  const uint64_t* cand;         // [nq][Kc] approximate keys, sorted descending
  const uint32_t* cand_cnt;     // [nq]
  int check_margin;             // 1: apply the completeness test; 0: candidates are final
  const float* margin;          // [nq] bound on |approximate - exact| in key units
  uint32_t id_offset;
  int64_t n_rows;               // rows in the index (all rows are candidates when <= Kc)
  int32_t* out_ids;             // [nq][k]
  float* out_scores;            // [nq][k]
  int32_t* out_counts;          // [nq]
  int32_t* nflag;               // number of queries that failed the test
  int32_t* flag_list;           // their indices
  uint32_t cap;                 // set by the launcher
};

struct ExactScanArgs {
  int nfq, dim, K, C;           // queries (<= 8), dimension, keys per stream, stream slots
  int flavor, metric;
  const float* queries;         // [nfq][dim]
  const void* rows;
  int64_t row_stride, n;
  uint64_t* bufs;               // [warps][8][C]
  uint32_t* cnts;               // [warps][8]
};

cudaError_t launch_rescore(RescoreArgs a, bool rows_f16, cudaStream_t st);
int exact_scan_warps(int num_sms);
cudaError_t launch_exact_scan(const ExactScanArgs& a, bool rows_f16, int R, int num_sms,
                              cudaStream_t st);

}  // namespace vx
