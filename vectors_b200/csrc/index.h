// index.h -- the device-resident state behind a vx_index handle (internal to libvx.so).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>
#include <vector>

struct vx_index {
  int kind = 0;
  int device = 0;
  int metric = 0;
  int64_t n = 0;
  int dim = 0;
  int num_sms = 148;
  // fp32 rows (FLAT; optional for the quantized kinds), row stride = dim
  float* rows32 = nullptr;
  // fp16 GEMM operand [n][Dp]: unit rows (FLAT) or the stored fp16 rows (FP16)
  __half* rows16 = nullptr;
  int Dp = 0;
  float* rowscale = nullptr;  // |x| (unit rows) or 1 (fp16 rows)
  float* rowsq = nullptr;     // |x|^2
  float* max_norm = nullptr;  // device scalar
  float* max_err = nullptr;   // device scalar: max over rows of |fp16(x/|x|) - x/|x||
  CUtensorMap tm_rows;
  bool has_tm_rows = false;
  // SQ8
  int8_t* codes8 = nullptr;
  int Dp8 = 0;
  float* vcorr = nullptr;
  int32_t* vsq = nullptr;
  float min_q = 0, max_q = 0;
  int sq_max = 127;  // ScalarBits.maxValue(): 127 SQ8, 15 SQ4 (codes unpacked one per byte)
  CUtensorMap tm_codes8;
  // BQ
  uint64_t* words = nullptr;
  int nw_pad = 0;
  // BBQ: the quantizer's centroid, per-row (|v - c|^2, vl, width, popcount) records
  float* bbq_centroid = nullptr;
  float4* bbq_rows = nullptr;
  // BBQ on the int8 tensor-core scan (with codes8 = the 0/1 bits): per-row epilogue records
  // (vl, width, vl * D + width * pop, |v - c| for COSINE or |v - c|^2)
  float4* bbq_epi = nullptr;
  // BQ / BBQ above the int8 operand's budget: the tensor-core scan expands the bits of one row
  // window at a time (codes8 stays null)
  bool bq_windows = false;
  // IVF-PQ
  float* cent = nullptr;
  int nlist = 0;
  int64_t* list_off = nullptr;
  int32_t* list_order = nullptr;  // list ids by row count, longest first (ties by id)
  int64_t max_list_rows = 0;      // rows of the longest list
  int32_t* ordinals = nullptr;
  uint8_t* pq_codes = nullptr;
  int M = 0, Ks = 0, Mp = 0;
  float* codebooks = nullptr;
  int64_t* cb_off = nullptr;
  int32_t* sub = nullptr;
  int nprobe = 1, rescore = 1;
  // PQ as a flat quantizer: each row's sum of centroidNormSq over its codes (COSINE)
  float* pq_rnorm = nullptr;
  // BuoyIndex state (IVF-PQ and IVF-flat): cluster radii (the EUCLIDEAN early exit of the flat
  // list scan), SOAR spill targets (null: none) and the adapter's search-time gamma
  float* radii = nullptr;
  int32_t* spill = nullptr;
  float gamma = 0.0f;
  // IVF-flat partitions built with HARMONY key dimensions (nullable): scanned with
  // squareDistance once a query's heap is full (EUCLIDEAN)
  uint8_t* keyed = nullptr;
  // IVF-flat: list-ordered rows zero-padded to Dp floats, their dotProduct(v, v) (COSINE)
  float* flat_rows = nullptr;
  float* flat_norms = nullptr;
  int Dp_flat = 0;
  std::vector<void*> owned;
  // exact-search view of a quantized index (built on first use)
  vx_index* flat = nullptr;
  std::mutex lazy_mu;
};

