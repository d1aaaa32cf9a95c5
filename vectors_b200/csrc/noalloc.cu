// noalloc.cu -- a BQ (sign-bit Hamming) candidate scan that allocates no device memory.
//
// Who needs it.  Some callers must not allocate device memory on their search path: a
// serving process that reserves its whole device budget at start-up and accounts every byte
// (for example a JVM host that sizes native memory up front and treats a later cudaMalloc as
// a budget breach), or a latency-critical query loop where cudaMalloc / cudaFree, or growing a
// stream-ordered pool, would block on the allocator or synchronise the device.  For them,
// vx_bq_scan_candidates_noalloc runs the same kernels as vx_scan_candidates_device on a BQ
// index, but takes its scratch (packed query words, per-CTA candidate buffers, merge output)
// from one statically sized array instead of allocating it.
//
// The array.  g_noalloc_scratch is a file-scope __device__ array of kNoAllocScratchBytes
// (64 MiB).  CUDA loads this file's module lazily by default (CUDA_MODULE_LOADING=LAZY), so the
// array is placed on a device when its address is first looked up, not when libvx.so is
// loaded; with CUDA_MODULE_LOADING=EAGER every context pays the 64 MiB at load instead.  The
// look-up happens in vx_bq_build (and so in a BQ quantized.bin build), on the index's device:
// every BQ index's build reserves the array there, once per device, and the array stays until
// the process exits.  In host code the array's name is only a host-side stand-in, so the build
// takes its device address with cudaGetSymbolAddress (with that device current) and caches it;
// the scan itself never looks it up and so never loads a module.  All calls on a device share
// the array and it keeps the previous call's contents: the counters that must start at zero are
// cleared on every call, and calls that overlap on the GPU (several host threads or streams at
// once) race on it and must be serialised by the caller.  Batches whose scratch would not fit
// are rejected with VX_ERR_INVALID_ARGUMENT and a message giving the largest batch that fits.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/vx.h"
#include "common.cuh"
#include "index.h"
#include "internal.h"
#include "kernels.h"

namespace vx {
namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};
cudaError_t g_noalloc_err[kMaxDevices] = {};

}  // namespace

void add_launches(int n);  // vx_api.cu: vx_kernel_launches counter

void noalloc_prepare(int device) {
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (device < 0 || device >= kMaxDevices || g_noalloc_ptr[device]) return;
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e == cudaSuccess && p) {
    g_noalloc_ptr[device] = p;
  } else {
    g_noalloc_err[device] = e == cudaSuccess ? cudaErrorInvalidSymbol : e;
    cudaGetLastError();  // the failed look-up must not fail the caller's next CUDA call
  }
}

namespace {

int noalloc_fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return record_failure(status, buf);
}

// Device address of this device's copy of the array, as the BQ build on that device cached it.
int scratch_address(int device, unsigned char** out) {
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (device < 0 || device >= kMaxDevices)
    return noalloc_fail(VX_ERR_INVALID_ARGUMENT, "device %d out of range", device);
  if (!g_noalloc_ptr[device])
    return noalloc_fail(VX_ERR_OUT_OF_MEMORY,
                        "the no-allocation scratch could not be placed on device %d when the BQ index "
                        "was built: %s",
                        device, cudaGetErrorString(g_noalloc_err[device]));
  *out = (unsigned char*)g_noalloc_ptr[device];
  return VX_OK;
}

size_t align_up(size_t v) { return (v + 255) & ~(size_t)255; }

struct NoAllocArgs {
  vx_index* ix;
  const float* d_queries;
  int32_t nq, dim, k;
  int32_t* d_ids;
  float* d_scores;
  int32_t* d_counts;
  void* stream;
};

int noalloc_scan(void* ctx) {
  const NoAllocArgs& a = *(const NoAllocArgs*)ctx;
  vx_index* ix = a.ix;
  const int32_t nq = a.nq, dim = a.dim, k = a.k;
  if (!ix || !a.d_queries || !a.d_ids || !a.d_scores || !a.d_counts)
    return noalloc_fail(VX_ERR_NULL_POINTER, "index, queries and output buffers must not be null");
  if (ix->kind != VX_KIND_BQ) return noalloc_fail(VX_ERR_UNSUPPORTED, "not a BQ index");
  if (nq <= 0) return noalloc_fail(VX_ERR_INVALID_ARGUMENT, "queries must not be empty");
  if (k <= 0) return noalloc_fail(VX_ERR_INVALID_ARGUMENT, "k must be positive: %d", k);
  if (ix->n > 0 && dim != ix->dim)
    return noalloc_fail(VX_ERR_INVALID_ARGUMENT, "Query dimension %d does not match index dimension %d",
                        dim, ix->dim);
  cudaStream_t st = (cudaStream_t)a.stream;
  cudaError_t e = cudaSetDevice(ix->device);
  if (e != cudaSuccess) return noalloc_fail(VX_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
  if (ix->n == 0) {
    if (cudaMemsetAsync(a.d_counts, 0, (size_t)nq * 4, st) != cudaSuccess ||
        cudaMemsetAsync(a.d_ids, 0xFF, (size_t)nq * k * 4, st) != cudaSuccess ||
        cudaMemsetAsync(a.d_scores, 0, (size_t)nq * k * 4, st) != cudaSuccess)
      return noalloc_fail(VX_ERR_CUDA, "cudaMemsetAsync failed");
    return VX_OK;
  }
  const int K = (int)(k < ix->n ? k : ix->n);
  const StreamGeom g = stream_geom(K, 32);
  if (g.R < 0) return noalloc_fail(VX_ERR_UNSUPPORTED, "k=%d is larger than this build supports", k);
  const int parts = bq_parts(ix->n, ix->num_sms);
  // scratch layout: packed queries | stream buffers | counts | thresholds | merged keys | counts
  const size_t b_qw = align_up((size_t)nq * ix->nw_pad * 8);
  const size_t b_bufs = align_up((size_t)parts * nq * g.C * 8);
  const size_t b_cnts = align_up((size_t)parts * nq * 4);
  const size_t b_thrs = align_up((size_t)parts * nq * 8);
  const size_t b_keys = align_up((size_t)nq * K * 8);
  const size_t b_kcnt = align_up((size_t)nq * 4);
  const size_t need = b_qw + b_bufs + b_cnts + b_thrs + b_keys + b_kcnt;
  if (need > kNoAllocScratchBytes) {
    // per-query bytes of the six regions; each region's 256-byte rounding costs at most 255
    const size_t per_q = (size_t)ix->nw_pad * 8 + (size_t)parts * g.C * 8 + (size_t)parts * 12 +
                         (size_t)K * 8 + 4;
    const size_t fit = (kNoAllocScratchBytes - 6 * 256) / per_q;
    return noalloc_fail(VX_ERR_INVALID_ARGUMENT,
                        "nq=%d, k=%d needs %zu bytes of scratch; the no-allocation scan has %zu bytes, "
                        "so at most %zu queries fit per call for this index and k (split the batch)",
                        nq, k, need, kNoAllocScratchBytes, fit);
  }
  unsigned char* base = nullptr;
  if (int s = scratch_address(ix->device, &base)) return s;
  uint64_t* qw = (uint64_t*)base;
  uint64_t* bufs = (uint64_t*)(base + b_qw);
  uint32_t* cnts = (uint32_t*)(base + b_qw + b_bufs);
  uint64_t* thrs = (uint64_t*)(base + b_qw + b_bufs + b_cnts);
  uint64_t* keys = (uint64_t*)(base + b_qw + b_bufs + b_cnts + b_thrs);
  uint32_t* kcnt = (uint32_t*)(base + b_qw + b_bufs + b_cnts + b_thrs + b_keys);
  // counters and thresholds must start at zero; the array keeps the previous call's data
  if (cudaMemsetAsync(cnts, 0, (size_t)parts * nq * 4, st) != cudaSuccess ||
      cudaMemsetAsync(thrs, 0, (size_t)parts * nq * 8, st) != cudaSuccess)
    return noalloc_fail(VX_ERR_CUDA, "cudaMemsetAsync failed");
  if ((e = launch_bq_pack_queries(a.d_queries, nq, dim, ix->nw_pad, qw, st)) != cudaSuccess ||
      (e = launch_bq_scan(ix->words, ix->n, ix->nw_pad, qw, nq, parts, g, bufs, cnts, thrs, st)) != cudaSuccess ||
      (e = launch_merge_streams(bufs, cnts, parts, nq, nq, g.C, K, keys, kcnt, st)) != cudaSuccess ||
      (e = launch_finish_keys(keys, kcnt, nq, K, k, kFinishHamming, ix->metric, dim, a.d_ids, a.d_scores,
                              a.d_counts, st)) != cudaSuccess)
    return noalloc_fail(VX_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e));
  add_launches(4);
  return VX_OK;
}

}  // namespace
}  // namespace vx

using namespace vx;

extern "C" int vx_bq_scan_candidates_noalloc(vx_index* ix, const float* d_queries, int32_t nq,
                                             int32_t dim, int32_t k, int32_t* d_ids,
                                             float* d_scores, int32_t* d_counts, void* stream) {
  NoAllocArgs a{ix, d_queries, nq, dim, k, d_ids, d_scores, d_counts, stream};
  return run_guarded(noalloc_scan, &a);
}
