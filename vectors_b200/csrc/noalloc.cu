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
// (64 MiB); every GPU that loads libvx.so holds one copy until the process exits.  In host
// code its name is only a host-side stand-in, so the first call on each device looks up its
// device address with cudaGetSymbolAddress (with that device current) and caches it; make
// that first call before any stream capture.  All calls on a device share the array and it
// keeps the previous call's contents: the counters that must start at zero are cleared on
// every call, and calls that overlap on the GPU (several host threads or streams at once)
// race on it and must be serialised by the caller.  Batches whose scratch would not fit are
// rejected with VX_ERR_INVALID_ARGUMENT and a message giving the limit.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/vx.h"
#include "common.cuh"
#include "index.h"
#include "kernels.h"

namespace vx {
namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

}  // namespace

int record_failure(int status, const char* msg);  // vx_api.cu: sets vx_last_error()
void add_launches(int n);                          // vx_api.cu: vx_kernel_launches counter

namespace {

int noalloc_fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return record_failure(status, buf);
}

// Device address of this device's copy of the array (looked up once per device).
int scratch_address(int device, unsigned char** out) {
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (device < 0 || device >= kMaxDevices)
    return noalloc_fail(VX_ERR_INVALID_ARGUMENT, "device %d out of range", device);
  if (!g_noalloc_ptr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return noalloc_fail(VX_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed on device %d: %s", device,
                          cudaGetErrorString(e));
    g_noalloc_ptr[device] = p;
  }
  *out = (unsigned char*)g_noalloc_ptr[device];
  return VX_OK;
}

size_t align_up(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace
}  // namespace vx

using namespace vx;

extern "C" int vx_bq_scan_candidates_noalloc(vx_index* ix, const float* d_queries, int32_t nq,
                                             int32_t dim, int32_t k, int32_t* d_ids,
                                             float* d_scores, int32_t* d_counts, void* stream) {
  if (!ix || !d_queries || !d_ids || !d_scores || !d_counts)
    return noalloc_fail(VX_ERR_NULL_POINTER, "index, queries and output buffers must not be null");
  if (ix->kind != VX_KIND_BQ) return noalloc_fail(VX_ERR_UNSUPPORTED, "not a BQ index");
  if (nq <= 0) return noalloc_fail(VX_ERR_INVALID_ARGUMENT, "queries must not be empty");
  if (k <= 0) return noalloc_fail(VX_ERR_INVALID_ARGUMENT, "k must be positive: %d", k);
  if (ix->n > 0 && dim != ix->dim)
    return noalloc_fail(VX_ERR_INVALID_ARGUMENT, "Query dimension %d does not match index dimension %d",
                        dim, ix->dim);
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaSetDevice(ix->device);
  if (e != cudaSuccess) return noalloc_fail(VX_ERR_CUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
  if (ix->n == 0) {
    if (cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, st) != cudaSuccess ||
        cudaMemsetAsync(d_ids, 0xFF, (size_t)nq * k * 4, st) != cudaSuccess ||
        cudaMemsetAsync(d_scores, 0, (size_t)nq * k * 4, st) != cudaSuccess)
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
  if (need > kNoAllocScratchBytes)
    return noalloc_fail(VX_ERR_INVALID_ARGUMENT,
                        "nq=%d, k=%d needs %zu bytes of scratch; the no-allocation scan has %zu bytes "
                        "(split the batch)",
                        nq, k, need, kNoAllocScratchBytes);
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
  if ((e = launch_bq_pack_queries(d_queries, nq, dim, ix->nw_pad, qw, st)) != cudaSuccess ||
      (e = launch_bq_scan(ix->words, ix->n, ix->nw_pad, qw, nq, parts, g, bufs, cnts, thrs, st)) != cudaSuccess ||
      (e = launch_merge_streams(bufs, cnts, parts, nq, nq, g.C, K, keys, kcnt, st)) != cudaSuccess ||
      (e = launch_finish_keys(keys, kcnt, nq, K, k, kFinishHamming, ix->metric, dim, d_ids, d_scores,
                              d_counts, st)) != cudaSuccess)
    return noalloc_fail(VX_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e));
  add_launches(4);
  return VX_OK;
}
