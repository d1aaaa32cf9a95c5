// gemm_scan.h -- interface of the tcgen05 query x database scan (gemm_scan.cu).
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "kernels.h"

namespace vx {

// Epilogue modes: how a TMEM accumulator value becomes a ranking score.
enum EpiMode : int {
  kEpiF16Plain = 0,   // approximate cosine of unit rows: s = acc
  kEpiF16Scaled = 1,  // approximate dot / |q|: s = acc * |x|
  kEpiF16L2 = 2,      // approximate |q|^2 - |q - x|^2: s = 2|q||x| acc - |x|^2
  kEpiSq8Dot = 3,     // ScalarQuantizedVectors DOT/COSINE score (exact)
  kEpiSq8Mip = 4,     // ScalarQuantizedVectors MAXIMUM_INNER_PRODUCT score (exact)
  kEpiSq8L2 = 5,      // ScalarQuantizedVectors EUCLIDEAN score (exact)
  kEpiBqHamming = 6,  // sign-bit BQ on +-1 int8 operands: h = (D - dot) / 2, ranked by -h (exact)
  // BBQ on 0/1 row bits x 4-bit query codes: the int32 accumulator is rawAsymDot exactly; the
  // epilogue applies computeBbqDot and the metric's transform (bbq.cuh), bit-exact
  kEpiBbqDot = 7,     // DOT_PRODUCT
  kEpiBbqMip = 8,     // MAXIMUM_INNER_PRODUCT
  kEpiBbqL2 = 9,      // EUCLIDEAN
  kEpiBbqCos = 10,    // COSINE
};

__host__ __device__ constexpr bool epi_is_bbq(int mode) { return mode >= kEpiBbqDot && mode <= kEpiBbqCos; }

struct EpiParams {
  const float* xnorm;   // [n] row scale: |x| for unit rows, 1 for stored fp16 rows
  const float* rowsq;   // [n] |x|^2 (F16 L2 mode)
  const float* qscale;  // [nq] |q| (F16 L2) or the query correction (SQ8 dot / mip)
  const float* vcorr;   // [n] SQ8 per-row corrections
  const int32_t* qsq;   // [nq] SQ8 sum of squared query codes
  const int32_t* vsq;   // [n] SQ8 sum of squared row codes
  float cm;             // SQ8 constMultiplier = alpha^2
  int32_t bits;         // BQ dimension D (bits per vector)
  const float4* bbq_rows;   // [n] BBQ (vl, width, vl * D + width * pop, |v - c| or |v - c|^2)
  const BbqQuery* bbq_q;    // [nq] BBQ per-query terms
};

struct ScanArgs {
  int64_t n;          // database rows
  int nq;             // queries (rows of the A operand beyond nq are zero padding)
  int num_mblocks;    // ceil(nq / queries per block): 256 for the 2-CTA variant, 128 otherwise
  int kchunks;        // padded row bytes / 128
  int64_t ntiles;     // ceil(n / 256)
  int K;              // keys kept per stream
  int C;              // stream buffer slots (32 * R)
  uint64_t* bufs;     // [units][Qp][C], Qp = num_mblocks * queries per block
  uint32_t* cnts;     // [units][Qp]   (zeroed before launch)
  uint64_t* thrs;     // [units][Qp]   (zeroed before launch)
  int m_major;        // 1: deal (query-block, row-tile) pairs query-block-major (one unit per block)
  uint64_t* floor;    // [nq] shared admission floors (nullable): any stream holding K keys
                      // publishes its K-th key; every stream admits only keys >= floor
  // Pooled floors (nullable top1): every stream tracks its two best admitted keys; a stream
  // whose j-th best key x (j = pool_j in {1, 2}) is matched by the j-th best keys of at least
  // pool_g streams of the same query (pool_g * pool_j >= K) raises that query's floor to x:
  // the streams cover disjoint rows, so at least K rows score >= x.
  uint64_t* top1;     // [units][Qp] best admitted key per stream (zeroed before launch)
  uint64_t* top2;     // [units][Qp] second best admitted key per stream (zeroed before launch)
  int pool_j;
  int pool_g;
  // Probe mode (nullable): the epilogue writes each query's largest score of every 32-row
  // group to probe[q][row / 32] (probe_groups per query) and keeps no candidate streams.
  float* probe;
  int probe_groups;
  // Exclusive upper bound on the keys a stream admits, per query (nullable): a later pass of a
  // search keeping more candidates than one stream holds takes the next keys below the last
  // pass's smallest (no pilot sweep then: its group maxima ignore the bound).
  const uint64_t* ceil = nullptr;
  // Epilogue warps per CTA: 4 (one per TMEM lane quarter, every column of a tile) or 8 (two per
  // lane quarter, each half of the columns, each with its own candidate streams: units * 2
  // streams per query).  stages: depth of the TMA ring (set by the launcher).
  int epi_warps = 4;
  int stages = 0;
  int32_t* err;       // device error word
  uint64_t timeout_ns;
  EpiParams epi;
};

// A work unit is a 2-CTA cluster (two_sm) or one CTA; each unit owns one candidate stream per
// query.  The query operand's tensor map has a 128-row box in both variants; the database
// operand's box is 128 rows with two_sm and 256 rows without.
constexpr int gemm_scan_query_block(bool two_sm) { return two_sm ? 256 : 128; }
constexpr int gemm_scan_db_box(bool two_sm) { return two_sm ? 128 : 256; }
int gemm_scan_units(int64_t ntiles, int num_mblocks, int num_sms, bool two_sm);
int gemm_scan_stream_R(int K);
// Whether the 8-epilogue-warp build exists for this mode and stream size: fp16 scans with
// R = 17 (544-key streams), where the per-tile top-K work outweighs the smaller ring and the
// 168-register cap of a 320-thread block.
bool gemm_scan_epi8(int mode, int R);
// One bounded wait that nothing completes (the scan's give-up path alone): err gets kDevWaitTimeout.
cudaError_t launch_wait_probe(uint64_t timeout_ns, int32_t* err, cudaStream_t st);
cudaError_t launch_gemm_scan(int mode, const CUtensorMap& tmA, const CUtensorMap& tmB,
                             const ScanArgs& a, int units, int R, bool two_sm, cudaStream_t st);

}  // namespace vx
