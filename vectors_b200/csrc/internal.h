// internal.h -- library-internal entry points shared between translation units of libvx.so
// (hidden: the library is built with -fvisibility=hidden and these carry no VX_API).
#pragma once
#include <cstdint>

#include "../../include/vx.h"

namespace vx {

// Records `msg` for vx_last_error() and returns `status` (vx_api.cu).
int record_failure(int status, const char* msg);

// Runs an entry point's body as every vx_* call does: host-side injected failures first, then
// CUDA and host-allocation failures mapped to a status (vx_api.cu).
int run_guarded(int (*body)(void*), void* ctx);

// Places the no-allocation scan's static scratch on `device` (the current device) and caches
// its address; called by vx_bq_build (noalloc.cu).
void noalloc_prepare(int device);

// vx_ivfpq_build with the full-precision rows `row_stride` floats apart (vx_api.cu).
int ivfpq_build_strided(int32_t device, const float* centroids, int32_t nlist, int32_t dim,
                        const int64_t* list_offsets, const int32_t* list_ordinals, int32_t m, int32_t ks,
                        const float* codebooks, const uint8_t* codes, int64_t n, int32_t metric,
                        const float* vectors, int64_t row_stride, int32_t nprobe, int32_t rescore_factor,
                        vx_index** out);

// ScalarQuantizedVectors index with codes one per byte, maxValue 127 (SQ8) or 15 (SQ4) (vx_api.cu).
int sq_build(int32_t device, const int8_t* codes, const float* corrections, int64_t n, int32_t dim,
             float min_quantile, float max_quantile, int max_value, int32_t metric, const float* vectors,
             int64_t row_stride, vx_index** out);

}  // namespace vx
