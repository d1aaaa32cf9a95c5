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
};

struct EpiParams {
  const float* xnorm;   // [n] row scale: |x| for unit rows, 1 for stored fp16 rows
  const float* rowsq;   // [n] |x|^2 (F16 L2 mode)
  const float* qscale;  // [nq] |q| (F16 L2) or the query correction (SQ8 dot / mip)
  const float* vcorr;   // [n] SQ8 per-row corrections
  const int32_t* qsq;   // [nq] SQ8 sum of squared query codes
  const int32_t* vsq;   // [n] SQ8 sum of squared row codes
  float cm;             // SQ8 constMultiplier = alpha^2
};

struct ScanArgs {
  int64_t n;          // database rows
  int nq;             // queries (rows of the A operand beyond nq are zero padding)
  int num_mblocks;    // ceil(nq / 128)
  int kchunks;        // padded row bytes / 128
  int64_t ntiles;     // ceil(n / 256)
  int K;              // keys kept per stream
  int C;              // stream buffer slots (32 * R)
  uint64_t* bufs;     // [grid][num_mblocks*128][C]
  uint32_t* cnts;     // [grid][num_mblocks*128]   (zeroed before launch)
  uint64_t* thrs;     // [grid][num_mblocks*128]   (zeroed before launch)
  int m_major;        // 1: deal (query-block, row-tile) pairs query-block-major (one CTA per block)
  uint64_t* floor;    // [nq] shared admission floors (nullable): any stream holding K keys
                      // publishes its K-th key; every stream admits only keys >= floor
  int32_t* err;       // device error word
  uint64_t timeout_ns;
  EpiParams epi;
};

int gemm_scan_grid(int64_t ntiles, int num_mblocks, int num_sms);
int gemm_scan_stream_R(int K);
cudaError_t launch_gemm_scan(int mode, const CUtensorMap& tmA, const CUtensorMap& tmB,
                             const ScanArgs& a, int grid, int R, cudaStream_t st);

}  // namespace vx
