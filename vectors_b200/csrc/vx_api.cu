// vx_api.cu -- the C ABI of libvx.so (include/vx.h): index handles, device copies, query
// chunking and the search pipelines built from the scan kernels.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/vx.h"
#include "common.cuh"
#include "gemm_scan.h"
#include "internal.h"
#include "ivfpq.h"
#include "kernels.h"
#include "prep.h"
#include "rescore.h"

namespace vx {
namespace {

thread_local std::string g_last_error;
thread_local int32_t g_fail_next = 0;
std::atomic<int64_t> g_launches{0};

int fail(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return status;
}

struct CudaFail {
  int status;
};

#define VX_CUDA(expr)                                                                       \
  do {                                                                                      \
    cudaError_t _e = (expr);                                                                \
    if (_e != cudaSuccess) {                                                                \
      int _s = (_e == cudaErrorMemoryAllocation) ? VX_ERR_OUT_OF_MEMORY : VX_ERR_CUDA;      \
      fail(_s, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, __LINE__); \
      throw CudaFail{_s};                                                                   \
    }                                                                                       \
  } while (0)

#define VX_LAUNCH(n, expr)          \
  do {                              \
    g_launches.fetch_add(n);        \
    VX_CUDA(expr);                  \
  } while (0)

// Optional per-kernel device timing: CUDA events recorded on the launching stream around a
// launch, drained by vx_profile_read.
struct ProfRec {
  int slot;
  cudaEvent_t a, b;
};
std::mutex g_prof_mu;
std::vector<ProfRec> g_prof;
std::atomic<bool> g_prof_on{false};
double g_prof_ms[VX_PROF_SLOTS] = {0};
int64_t g_prof_n[VX_PROF_SLOTS] = {0};

#define VX_TIMED(slot, st, n, expr)                                  \
  do {                                                               \
    cudaEvent_t _a = nullptr, _b = nullptr;                          \
    const bool _on = g_prof_on.load();                               \
    if (_on) {                                                       \
      VX_CUDA(cudaEventCreate(&_a));                                 \
      VX_CUDA(cudaEventCreate(&_b));                                 \
      VX_CUDA(cudaEventRecord(_a, st));                              \
    }                                                                \
    VX_LAUNCH(n, expr);                                              \
    if (_on) {                                                       \
      VX_CUDA(cudaEventRecord(_b, st));                              \
      std::lock_guard<std::mutex> _g(g_prof_mu);                     \
      g_prof.push_back(ProfRec{slot, _a, _b});                       \
    }                                                                \
  } while (0)

bool take_injected(int* st) {
  if (g_fail_next != 0) {
    *st = fail(g_fail_next, "injected failure (vx_debug_fail_next)");
    g_fail_next = 0;
    return true;
  }
  return false;
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// ------------------------------------------------------------------ driver entry points
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

// 2-D K-major operand [rows][row_bytes] with a (128-byte x box_rows) box, 128-byte swizzle.
void make_tmap(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes,
               int64_t inner_elems, int64_t rows, int box_rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) {
    fail(VX_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
    throw CudaFail{VX_ERR_CUDA};
  }
  cuuint64_t dims[2] = {(cuuint64_t)inner_elems, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(inner_elems * elem_bytes)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / elem_bytes), (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dt, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    fail(VX_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    throw CudaFail{VX_ERR_CUDA};
  }
}

// ------------------------------------------------------------------ scratch
// Stream-ordered device allocations released (stream-ordered) at scope exit.
struct Scratch {
  cudaStream_t st;
  std::vector<void*> ptrs;
  explicit Scratch(cudaStream_t s) : st(s) {}
  template <class T>
  T* alloc(size_t count) {
    void* p = nullptr;
    size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    VX_CUDA(cudaMallocAsync(&p, bytes, st));
    ptrs.push_back(p);
    return (T*)p;
  }
  ~Scratch() {
    for (void* p : ptrs) cudaFreeAsync(p, st);
  }
};

size_t scratch_budget() {
  const char* e = getenv("VX_SCRATCH_BYTES");
  if (e && *e) return (size_t)strtoull(e, nullptr, 10);
  return (size_t)6 << 30;
}

uint64_t wait_timeout_ns() {
  const char* e = getenv("VX_WAIT_TIMEOUT_MS");
  if (e && *e) return (uint64_t)strtoull(e, nullptr, 10) * 1000000ull;
  return 1500ull * 1000000ull;  // 1.5 s per wait
}

// The pilot sweep before each scan is on unless VX_SCAN_PILOT=0.
bool use_pilot() {
  static const bool v = [] {
    const char* e = getenv("VX_SCAN_PILOT");
    return !(e && *e == '0');
  }();
  return v;
}

// Epilogue warps of the tcgen05 scan: 8 (two per TMEM lane quarter, each half of a tile's
// columns) where that build exists -- fp16 scans with 544-key streams (the FP16 k = 100 scan:
// 15 % faster than 4) -- else 4.  VX_EPI_WARPS=4 picks 4 there too.
int epi_warps_for(int mode, int K) {
  static const int forced = [] {
    const char* e = getenv("VX_EPI_WARPS");
    return (e && (*e == '4' || *e == '8')) ? *e - '0' : 0;
  }();
  if (!gemm_scan_epi8(mode, gemm_scan_stream_R(K))) return 4;
  return forced ? forced : 8;
}

// Pooled admission floors (ScanArgs::top1) unless VX_SCAN_POOL=0.
bool use_pool() {
  static const bool v = [] {
    const char* e = getenv("VX_SCAN_POOL");
    return !(e && *e == '0');
  }();
  return v;
}

// BQ indexes also keep a +-1 int8 copy of the bits (8x the storage) for the tensor-core
// Hamming scan while it fits VX_BQ_TENSOR_BYTES (default 64 GiB), read at each build.
uint64_t bq_tensor_budget() {
  const char* e = getenv("VX_BQ_TENSOR_BYTES");
  return (e && *e) ? (uint64_t)strtoull(e, nullptr, 10) : (uint64_t)64 << 30;
}

// BQ / BBQ indexes above that budget keep only their bits (and BBQ's 16-byte epilogue records)
// and expand one window of rows at a time to the int8 operand, in a search-time scratch buffer of
// at most VX_BQ_WINDOW_BYTES (default 4 GiB; 0 leaves such indexes on the popcount scans), read at
// each build (whether windows are used) and search (their size).
uint64_t bq_window_bytes() {
  const char* e = getenv("VX_BQ_WINDOW_BYTES");
  return (e && *e) ? (uint64_t)strtoull(e, nullptr, 10) : (uint64_t)4 << 30;
}

// Rows per window: whole 256-row tiles within the window budget (at least one tile).
int64_t bq_window_rows(int64_t n, int Dp8) {
  int64_t w = (int64_t)(bq_window_bytes() / (uint64_t)Dp8) / 256 * 256;
  w = std::max<int64_t>(w, 256);
  return std::min<int64_t>(w, n);
}

// IVF-PQ scans use the grouped ADC kernel where the shape allows unless VX_ADC_GROUPED=0.
bool use_adc_group() {
  static const bool v = [] {
    const char* e = getenv("VX_ADC_GROUPED");
    return !(e && *e == '0');
  }();
  return v;
}

// The tcgen05 scan runs on 2-CTA clusters unless VX_GEMM_1SM=1 selects the 1-CTA variant
// (read once per process: index tensor maps are built for the variant in use).
bool gemm_two_sm() {
  static const bool v = [] {
    const char* e = getenv("VX_GEMM_1SM");
    return !(e && *e && *e != '0');
  }();
  return v;
}

}  // namespace

// Shared with noalloc.cu (internal to the library, not exported).
int record_failure(int status, const char* msg) { return fail(status, "%s", msg); }
void add_launches(int n) { g_launches.fetch_add(n); }

}  // namespace vx

using namespace vx;

#include "index.h"

namespace vx {
namespace {

template <class T>
T* dev_alloc(vx_index* ix, size_t count) {
  void* p = nullptr;
  VX_CUDA(cudaMalloc(&p, std::max<size_t>(count * sizeof(T), 16)));
  ix->owned.push_back(p);
  return (T*)p;
}

// A build's temporary device buffer, released when it leaves scope (the error path included).
template <class T>
struct DevTemp {
  T* p = nullptr;
  explicit DevTemp(size_t count) {
    void* q = nullptr;
    VX_CUDA(cudaMalloc(&q, std::max<size_t>(count * sizeof(T), 16)));
    p = (T*)q;
  }
  ~DevTemp() {
    if (p) cudaFree(p);
  }
  DevTemp(const DevTemp&) = delete;
  DevTemp& operator=(const DevTemp&) = delete;
};

void free_index(vx_index* ix) {
  if (!ix) return;
  cudaSetDevice(ix->device);
  cudaDeviceSynchronize();
  if (ix->flat) free_index(ix->flat);
  for (void* p : ix->owned) cudaFree(p);
  delete ix;
}

int check_device(int device, int* nsms) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0)
    return fail(VX_ERR_GPU_UNAVAILABLE, "no CUDA device available (%s)",
                e == cudaSuccess ? "0 devices" : cudaGetErrorString(e));
  if (device < 0 || device >= count)
    return fail(VX_ERR_INVALID_ARGUMENT, "device %d out of range [0, %d)", device, count);
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
    return fail(VX_ERR_GPU_UNAVAILABLE, "cannot query device %d", device);
  if (prop.major != 10)
    return fail(VX_ERR_GPU_UNAVAILABLE, "device %d is sm_%d%d; this library is built for sm_100a",
                device, prop.major, prop.minor);
  if (cudaSetDevice(device) != cudaSuccess)
    return fail(VX_ERR_GPU_UNAVAILABLE, "cannot select device %d", device);
  *nsms = prop.multiProcessorCount;
  // Keep the per-search scratch cached in the device's stream-ordered pool between calls
  // (the default threshold returns it to the driver at every synchronisation).
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
    uint64_t keep = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
  }
  return VX_OK;
}

int check_metric(int metric) {
  if (metric < 0 || metric > 3) return fail(VX_ERR_INVALID_ARGUMENT, "unknown metric %d", metric);
  return VX_OK;
}

// Uploads host rows (stride >= dim floats) as a dense [n][dim] device array.
float* upload_rows32(vx_index* ix, const float* host, int64_t n, int dim, int64_t stride) {
  float* d = dev_alloc<float>(ix, (size_t)n * dim);
  if (n > 0)
    VX_CUDA(cudaMemcpy2D(d, (size_t)dim * 4, host, (size_t)stride * 4, (size_t)dim * 4, (size_t)n,
                         cudaMemcpyDefault));
  return d;
}

// IVF list ids ordered by row count, longest first (ties by id): grouped scans hand out the
// groups of long lists first, so the last groups to finish are short.
int32_t* upload_list_order(vx_index* ix, const int64_t* list_offsets, int nlist) {
  std::vector<int32_t> order(nlist);
  for (int l = 0; l < nlist; l++) order[l] = l;
  ix->max_list_rows = 0;
  for (int l = 0; l < nlist; l++) ix->max_list_rows = std::max(ix->max_list_rows, list_offsets[l + 1] - list_offsets[l]);
  std::stable_sort(order.begin(), order.end(), [&](int32_t x, int32_t y) {
    return list_offsets[x + 1] - list_offsets[x] > list_offsets[y + 1] - list_offsets[y];
  });
  int32_t* d = dev_alloc<int32_t>(ix, (size_t)nlist);
  VX_CUDA(cudaMemcpy(d, order.data(), (size_t)nlist * 4, cudaMemcpyHostToDevice));
  return d;
}

// fp16 unit-row GEMM operand from the fp32 rows.
void build_unit_f16(vx_index* ix) {
  ix->Dp = (int)round_up(ix->dim, 64);
  ix->rows16 = dev_alloc<__half>(ix, (size_t)std::max<int64_t>(ix->n, 1) * ix->Dp);
  ix->rowscale = dev_alloc<float>(ix, (size_t)std::max<int64_t>(ix->n, 1));
  ix->rowsq = dev_alloc<float>(ix, (size_t)std::max<int64_t>(ix->n, 1));
  ix->max_norm = dev_alloc<float>(ix, 1);
  ix->max_err = dev_alloc<float>(ix, 1);
  VX_CUDA(cudaMemset(ix->max_norm, 0, 4));
  VX_CUDA(cudaMemset(ix->max_err, 0, 4));
  VX_LAUNCH(1, launch_rows_to_f16(ix->rows32, ix->n, ix->dim, ix->dim, ix->Dp, true, ix->rows16,
                                  ix->rowscale, ix->rowsq, ix->max_norm, 0, nullptr, ix->max_err));
  if (ix->n > 0) {
    make_tmap(&ix->tm_rows, ix->rows16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ix->Dp, ix->n,
             gemm_scan_db_box(gemm_two_sm()));
    ix->has_tm_rows = true;
  }
  VX_CUDA(cudaDeviceSynchronize());
}

template <class F>
int guarded(F&& f) {
  int st;
  if (take_injected(&st)) return st;
  try {
    return f();
  } catch (const CudaFail& e) {
    return e.status;
  } catch (const std::bad_alloc&) {
    return fail(VX_ERR_OUT_OF_MEMORY, "host allocation failed");
  }
}

}  // namespace

int run_guarded(int (*body)(void*), void* ctx) {
  return guarded([&]() -> int { return body(ctx); });
}

namespace {

int check_device_error(int32_t* d_err, cudaStream_t st) {
  int32_t h = 0;
  VX_CUDA(cudaMemcpyAsync(&h, d_err, 4, cudaMemcpyDeviceToHost, st));
  VX_CUDA(cudaStreamSynchronize(st));
  if (h == kDevWaitTimeout)
    return fail(VX_ERR_DEVICE_TIMEOUT, "a device-side wait exceeded its time budget");
  if (h != 0) return fail(VX_ERR_CUDA, "device error %d", h);
  return VX_OK;
}

// ------------------------------------------------------------------ exact fallback
// Scores every row exactly for the queries in `list` (device indices into q) and writes
// their results in place.
void exact_fallback(vx_index* ix, const float* dq, int nq_chunk, int dim, int k, int flavor,
                    const void* rows, bool rows_f16, int64_t stride, const int32_t* h_list,
                    int nflag, int32_t* d_ids, float* d_scores, int32_t* d_counts,
                    cudaStream_t st) {
  Scratch S(st);
  const StreamGeom g = stream_geom(k, 32);
  const int W = exact_scan_warps(ix->num_sms);
  float* fq = S.alloc<float>((size_t)8 * dim);
  uint64_t* bufs = S.alloc<uint64_t>((size_t)W * 8 * g.C);
  uint32_t* cnts = S.alloc<uint32_t>((size_t)W * 8);
  uint64_t* keys = S.alloc<uint64_t>((size_t)8 * k);
  uint32_t* kc = S.alloc<uint32_t>(8);
  int32_t* tids = S.alloc<int32_t>((size_t)8 * k);
  float* tsc = S.alloc<float>((size_t)8 * k);
  int32_t* tcnt = S.alloc<int32_t>(8);
  for (int f0 = 0; f0 < nflag; f0 += 8) {
    const int nf = std::min(8, nflag - f0);
    for (int i = 0; i < nf; i++)
      VX_CUDA(cudaMemcpyAsync(fq + (size_t)i * dim, dq + (size_t)h_list[f0 + i] * dim,
                              (size_t)dim * 4, cudaMemcpyDeviceToDevice, st));
    ExactScanArgs a;
    a.nfq = nf;
    a.dim = dim;
    a.K = g.K;
    a.C = g.C;
    a.flavor = flavor;
    a.metric = ix->metric;
    a.queries = fq;
    a.rows = rows;
    a.row_stride = stride;
    a.n = ix->n;
    a.bufs = bufs;
    a.cnts = cnts;
    VX_TIMED(VX_PROF_FALLBACK, st, 1, launch_exact_scan(a, rows_f16, g.R, ix->num_sms, st));
    VX_LAUNCH(1, launch_merge_streams(bufs, cnts, W, nf, 8, g.C, k, keys, kc, st));
    VX_LAUNCH(1, launch_finish_keys(keys, kc, nf, k, k, kFinishFloatKey, ix->metric, dim, tids, tsc,
                                    tcnt, st));
    for (int i = 0; i < nf; i++) {
      const int q = h_list[f0 + i];
      VX_CUDA(cudaMemcpyAsync(d_ids + (size_t)q * k, tids + (size_t)i * k, (size_t)k * 4,
                              cudaMemcpyDeviceToDevice, st));
      VX_CUDA(cudaMemcpyAsync(d_scores + (size_t)q * k, tsc + (size_t)i * k, (size_t)k * 4,
                              cudaMemcpyDeviceToDevice, st));
      VX_CUDA(cudaMemcpyAsync(d_counts + q, tcnt + i, 4, cudaMemcpyDeviceToDevice, st));
    }
  }
  VX_CUDA(cudaStreamSynchronize(st));
}

constexpr int kMaxCandidates = 1000;  // largest window the R=33 stream geometry holds
constexpr int kStreamKeysMax = 1023;  // keys one candidate stream keeps (R = 33)
constexpr int kQuantizedKeysMax = 8 * kStreamKeysMax;  // quantized candidates per query, in passes

int candidate_width(int k, int64_t n) {
  // Approximate candidates per query in the first pass: enough headroom above k for the
  // completeness test to pass on typical data.  Queries that fail it are re-run with
  // kMaxCandidates, and only queries failing that too take the exact fallback scan.
  int64_t kc = std::max<int64_t>(128, round_up(2 * (int64_t)k + 32, 32));
  kc = std::min<int64_t>(kc, kMaxCandidates);
  if (n < kc) kc = std::max<int64_t>(n, 1);
  return (int)kc;
}

// Runs the tcgen05 scan for one query chunk and merges each query's streams into its K best
// keys.  A probe sweep over the first kPilotRows rows (the same kernel keeping no streams,
// only each query's maximum per 32-row group) seeds every query's admission floor with the
// K-th largest group maximum; during the main scan, full streams publish their K-th keys and
// pooled floors rise further, so rows below them are never buffered.  The merge then ignores
// keys under the final floor.
constexpr int64_t kPilotRows = 32768;

cudaError_t launch_probe_sweep(int mode, const CUtensorMap& tmq, const CUtensorMap& tmrows, const ScanArgs& p,
                               int units, int R, bool two_sm, uint64_t* floor, int K, cudaStream_t st) {
  cudaError_t e = launch_gemm_scan(mode, tmq, tmrows, p, units, R, two_sm, st);
  if (e == cudaSuccess) e = launch_probe_floor(p.probe, p.nq, p.probe_groups, K, floor, st);
  return e;
}

// seed (nullable, device [Qp]): initial admission floors known from earlier row windows; the
// probe sweep is skipped then.
void scan_and_merge(int mode, const CUtensorMap& tmq, const CUtensorMap& tmrows, ScanArgs a,
                    int units, int R, int Qp, uint64_t* floor, uint64_t* tops, float* probe,
                    uint64_t* cand, uint32_t* cand_cnt, cudaStream_t st, const uint64_t* seed = nullptr) {
  const bool two_sm = gemm_two_sm();
  if (seed) {
    VX_CUDA(cudaMemcpyAsync(floor, seed, (size_t)Qp * 8, cudaMemcpyDeviceToDevice, st));
  } else {
    VX_CUDA(cudaMemsetAsync(floor, 0, (size_t)Qp * 8, st));
  }
  a.floor = floor;
  a.m_major = 0;
  a.probe = nullptr;
  a.probe_groups = 0;
  // Pooled floors need K <= 2 * (streams per query); each stream then contributes its best
  // (pool_j = 1) or second best (pool_j = 2) key.
  // candidate streams per query: one per unit and epilogue half (8 epilogue warps: two)
  const int streams = units * (a.epi_warps / 4);
  a.top1 = a.top2 = nullptr;
  a.pool_j = a.K <= streams ? 1 : (a.K <= 2 * streams ? 2 : 0);
  a.pool_g = a.pool_j ? (a.K + a.pool_j - 1) / a.pool_j : 0;
  if (a.pool_j && tops && use_pool()) {
    a.top1 = tops;
    a.top2 = tops + (size_t)streams * Qp;
    VX_CUDA(cudaMemsetAsync(tops, 0, (size_t)2 * streams * Qp * 8, st));
  }
  if (probe && !seed && !a.ceil && a.n > 2 * kPilotRows && a.K <= kPilotRows / 32 && use_pilot()) {
    // probe sweep over the first kPilotRows rows: group maxima only, then the floors
    ScanArgs p = a;
    p.n = kPilotRows;
    p.ntiles = kPilotRows / 256;
    p.top1 = p.top2 = nullptr;
    p.floor = nullptr;
    p.probe = probe;
    p.probe_groups = (int)(kPilotRows / 32);
    const int punits = (int)std::min<int64_t>((int64_t)p.ntiles * a.num_mblocks, units);
    VX_TIMED(VX_PROF_PILOT, st, 2, launch_probe_sweep(mode, tmq, tmrows, p, punits, R, two_sm, floor, a.K, st));
  }
  VX_CUDA(cudaMemsetAsync(a.cnts, 0, (size_t)streams * Qp * 4, st));
  VX_CUDA(cudaMemsetAsync(a.thrs, 0, (size_t)streams * Qp * 8, st));
  VX_TIMED(VX_PROF_GEMM_SCAN, st, 1, launch_gemm_scan(mode, tmq, tmrows, a, units, R, two_sm, st));
  VX_TIMED(VX_PROF_MERGE, st, 1,
           launch_merge_streams(a.bufs, a.cnts, streams, a.nq, Qp, a.C, a.K, cand, cand_cnt, st, floor));
}

// One approximate pass with Kc candidates per query followed by the exact re-score; queries
// whose candidate window fails the completeness test are appended to *flagged (indices into
// dq) and their outputs are left for a later pass.
int gemm_exact_pass(vx_index* ix, const float* dq, int nq, int k, int Kc, int32_t* d_ids,
                    float* d_scores, int32_t* d_counts, cudaStream_t st,
                    std::vector<int32_t>* flagged) {
  const bool f16_kind = ix->kind == VX_KIND_FP16;
  const int flavor = f16_kind ? kFlavorFp16Quantized : kFlavorFlat;
  const void* rows = f16_kind ? (const void*)ix->rows16 : (const void*)ix->rows32;
  const int64_t stride = f16_kind ? ix->Dp : ix->dim;
  const int dim = ix->dim;
  const int R = gemm_scan_stream_R(Kc);
  if (R < 0) return fail(VX_ERR_UNSUPPORTED, "k=%d is larger than this build supports", k);
  const int C = 32 * R;
  const int64_t ntiles = (ix->n + 255) / 256;
  int mode;
  if (ix->metric == VX_EUCLIDEAN)
    mode = kEpiF16L2;
  else if (f16_kind || ix->metric == VX_COSINE)
    mode = kEpiF16Plain;
  else
    mode = kEpiF16Scaled;
  // query chunk sized by the scratch budget
  const bool two_sm = gemm_two_sm();
  const int QB = gemm_scan_query_block(two_sm);
  const int EW = epi_warps_for(mode, Kc);
  const int U0 = gemm_scan_units(ntiles, 1 << 20, ix->num_sms, two_sm) * (EW / 4);  // streams per query
  int64_t qch = (int64_t)(scratch_budget() / ((size_t)U0 * (C * 8 + 12)));
  qch = std::max<int64_t>(QB, qch / QB * QB);
  // Buffers are sized once for the largest chunk and reused, so repeated calls draw blocks
  // of one size from the stream-ordered pool.
  const int qmax = (int)std::min<int64_t>(qch, std::max(nq, 1));
  const int QpMax = (qmax + QB - 1) / QB * QB;
  const int unitsMax = gemm_scan_units(ntiles, QpMax / QB, ix->num_sms, two_sm) * (EW / 4);  // streams
  const int nchunks = (int)((nq + qch - 1) / qch);
  Scratch S(st);
  int32_t* d_err = S.alloc<int32_t>(1);
  __half* qh = S.alloc<__half>((size_t)QpMax * ix->Dp);
  float* qnorm = S.alloc<float>(QpMax);
  float* qerr = S.alloc<float>(QpMax);
  float* margin = S.alloc<float>(QpMax);
  uint64_t* bufs = S.alloc<uint64_t>((size_t)unitsMax * QpMax * C);
  uint32_t* cnts = S.alloc<uint32_t>((size_t)unitsMax * QpMax);
  uint64_t* thrs = S.alloc<uint64_t>((size_t)unitsMax * QpMax);
  uint64_t* floor = S.alloc<uint64_t>(QpMax);
  uint64_t* tops = S.alloc<uint64_t>((size_t)2 * unitsMax * QpMax);
  float* probe = S.alloc<float>((size_t)QpMax * (kPilotRows / 32));
  uint64_t* cand = S.alloc<uint64_t>((size_t)qmax * Kc);
  uint32_t* cand_cnt = S.alloc<uint32_t>(qmax);
  int32_t* nflag = S.alloc<int32_t>(std::max(nchunks, 1));
  int32_t* flag_list = S.alloc<int32_t>(std::max(nq, 1));
  VX_CUDA(cudaMemsetAsync(d_err, 0, 4, st));
  VX_CUDA(cudaMemsetAsync(nflag, 0, (size_t)std::max(nchunks, 1) * 4, st));
  for (int c = 0; c < nchunks; c++) {
    const int q0 = (int)(c * qch);
    const int qc = (int)std::min<int64_t>(qch, nq - q0);
    const int mblocks = (qc + QB - 1) / QB;
    const int Qp = mblocks * QB;
    const int units = gemm_scan_units(ntiles, mblocks, ix->num_sms, two_sm);
    const float* dqc = dq + (size_t)q0 * dim;
    VX_CUDA(cudaMemsetAsync(qh + (size_t)qc * ix->Dp, 0, (size_t)(Qp - qc) * ix->Dp * 2, st));
    VX_LAUNCH(1, launch_rows_to_f16(dqc, qc, dim, dim, ix->Dp, true, qh, qnorm, nullptr, nullptr, st,
                                    qerr, nullptr));
    VX_LAUNCH(1, launch_margin(qnorm, qerr, qc, dim, ix->metric,
                               f16_kind ? kOperandExactRows : kOperandUnitRows, ix->max_norm,
                               f16_kind ? ix->max_norm : ix->max_err, margin, st));
    CUtensorMap tmq;
    make_tmap(&tmq, qh, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ix->Dp, Qp, 128);
    ScanArgs a;
    a.n = ix->n;
    a.nq = qc;
    a.num_mblocks = mblocks;
    a.kchunks = ix->Dp / 64;
    a.ntiles = ntiles;
    a.K = Kc;
    a.C = C;
    a.bufs = bufs;
    a.cnts = cnts;
    a.thrs = thrs;
    a.err = d_err;
    a.timeout_ns = wait_timeout_ns();
    a.epi_warps = EW;
    a.epi.xnorm = ix->rowscale;
    a.epi.rowsq = ix->rowsq;
    a.epi.qscale = qnorm;
    a.epi.vcorr = nullptr;
    a.epi.qsq = nullptr;
    a.epi.vsq = nullptr;
    a.epi.cm = 0.0f;
    a.epi.bits = 0;
    scan_and_merge(mode, tmq, ix->tm_rows, a, units, R, Qp, floor, tops, probe, cand, cand_cnt, st);
    RescoreArgs r;
    r.nq = qc;
    r.dim = dim;
    r.k = k;
    r.Kc = Kc;
    r.flavor = flavor;
    r.metric = ix->metric;
    r.queries = dqc;
    r.rows = rows;
    r.row_stride = stride;
    r.cand = cand;
    r.cand_cnt = cand_cnt;
    r.check_margin = 1;
    r.margin = margin;
    r.id_offset = 0;
    r.n_rows = ix->n;
    r.out_ids = d_ids + (size_t)q0 * k;
    r.out_scores = d_scores + (size_t)q0 * k;
    r.out_counts = d_counts + q0;
    r.nflag = nflag + c;
    r.flag_list = flag_list + q0;
    VX_TIMED(VX_PROF_RESCORE, st, 1, launch_rescore(r, f16_kind, st));
  }
  int st_err = check_device_error(d_err, st);
  if (st_err != VX_OK) return st_err;
  std::vector<int32_t> h_nflag(std::max(nchunks, 1), 0);
  VX_CUDA(cudaMemcpyAsync(h_nflag.data(), nflag, (size_t)nchunks * 4, cudaMemcpyDeviceToHost, st));
  VX_CUDA(cudaStreamSynchronize(st));
  for (int c = 0; c < nchunks; c++) {
    if (h_nflag[c] <= 0) continue;
    const int q0 = (int)(c * qch);
    std::vector<int32_t> h_list(h_nflag[c]);
    VX_CUDA(cudaMemcpyAsync(h_list.data(), flag_list + q0, (size_t)h_nflag[c] * 4, cudaMemcpyDeviceToHost, st));
    VX_CUDA(cudaStreamSynchronize(st));
    for (int32_t f : h_list) flagged->push_back(q0 + f);
  }
  return VX_OK;
}

// FLAT / FP16: fp16 tcgen05 approximate pass + exact fp32 re-score, a wider second pass for
// the queries whose window was too narrow, and the exact scan for any still unresolved.
int search_gemm_exact(vx_index* ix, const float* dq, int nq, int k, int32_t* d_ids,
                      float* d_scores, int32_t* d_counts, cudaStream_t st) {
  const bool f16_kind = ix->kind == VX_KIND_FP16;
  const int flavor = f16_kind ? kFlavorFp16Quantized : kFlavorFlat;
  const void* rows = f16_kind ? (const void*)ix->rows16 : (const void*)ix->rows32;
  const int64_t stride = f16_kind ? ix->Dp : ix->dim;
  const int dim = ix->dim;
  const int Kc1 = candidate_width(k, ix->n);
  std::vector<int32_t> f1;
  int rc = gemm_exact_pass(ix, dq, nq, k, Kc1, d_ids, d_scores, d_counts, st, &f1);
  if (rc != VX_OK || f1.empty()) return rc;
  std::vector<int32_t> rest;
  const int Kc2 = (int)std::min<int64_t>(kMaxCandidates, std::max<int64_t>(ix->n, 1));
  if (Kc2 > Kc1 && Kc2 > k) {
    const int F = (int)f1.size();
    Scratch S(st);
    int32_t* map = S.alloc<int32_t>(F);
    float* sub = S.alloc<float>((size_t)F * dim);
    int32_t* ti = S.alloc<int32_t>((size_t)F * k);
    float* ts = S.alloc<float>((size_t)F * k);
    int32_t* tc = S.alloc<int32_t>(F);
    VX_CUDA(cudaMemcpyAsync(map, f1.data(), (size_t)F * 4, cudaMemcpyHostToDevice, st));
    VX_LAUNCH(1, launch_gather_rows(dq, map, F, dim, sub, st));
    std::vector<int32_t> f2;
    rc = gemm_exact_pass(ix, sub, F, k, Kc2, ti, ts, tc, st, &f2);
    if (rc != VX_OK) return rc;
    VX_LAUNCH(1, launch_scatter_results(ti, ts, tc, map, F, k, d_ids, d_scores, d_counts, st));
    for (int32_t i : f2) rest.push_back(f1[i]);
    VX_CUDA(cudaStreamSynchronize(st));
  } else {
    rest = f1;
  }
  if (!rest.empty())
    exact_fallback(ix, dq, nq, dim, k, flavor, rows, f16_kind, stride, rest.data(), (int)rest.size(),
                   d_ids, d_scores, d_counts, st);
  return VX_OK;
}

// SQ8 / SQ4 / BQ / BBQ: exact quantized scores; K best per query (optionally re-scored in fp32).
// The int8 tensor-core scan serves every kind: over the whole int8 operand (codes8) where the
// index keeps one, else (BQ / BBQ above VX_BQ_TENSOR_BYTES) over row windows expanded from the
// bits at search time.  With windows switched off (VX_BQ_WINDOW_BYTES=0) such indexes take the
// popcount scans.
int search_quantized_scan(vx_index* ix, const float* dq, int nq, int K, int k_out, bool rescore,
                          int32_t* d_ids, float* d_scores, int32_t* d_counts, cudaStream_t st) {
  const int dim = ix->dim;
  Scratch S(st);
  int32_t* d_err = S.alloc<int32_t>(1);
  VX_CUDA(cudaMemsetAsync(d_err, 0, 4, st));
  if (ix->kind == VX_KIND_SQ8 || ix->kind == VX_KIND_SQ4 ||
      ((ix->kind == VX_KIND_BQ || ix->kind == VX_KIND_BBQ) && (ix->codes8 || ix->bq_windows))) {
    const bool bq = ix->kind == VX_KIND_BQ;    // +-1 operands, Hamming epilogue
    const bool bbq = ix->kind == VX_KIND_BBQ;  // 0/1 rows x 4-bit query codes, BBQ epilogue
    // More candidates than one stream keeps (kStreamKeysMax) are taken in passes: each later
    // pass admits only keys below the previous pass's smallest, so the passes' sorted keys
    // concatenate into the K best.
    if (K > kQuantizedKeysMax)
      return fail(VX_ERR_UNSUPPORTED, "%d candidates per query is more than the %d this build keeps", K,
                  kQuantizedKeysMax);
    const int KP = std::min(K, kStreamKeysMax);  // keys per pass
    const int R = gemm_scan_stream_R(KP);
    if (R < 0) return fail(VX_ERR_UNSUPPORTED, "k=%d is larger than this build supports", K);
    const int C = 32 * R;
    const int64_t ntiles = (ix->n + 255) / 256;
    const bool two_sm = gemm_two_sm();
    const int QB = gemm_scan_query_block(two_sm);
    const int mode = bq ? kEpiBqHamming
                     : bbq ? (ix->metric == VX_EUCLIDEAN ? kEpiBbqL2
                              : ix->metric == VX_MAXIMUM_INNER_PRODUCT ? kEpiBbqMip
                              : ix->metric == VX_COSINE ? kEpiBbqCos
                                                        : kEpiBbqDot)
                     : ix->metric == VX_EUCLIDEAN ? kEpiSq8L2
                     : ix->metric == VX_MAXIMUM_INNER_PRODUCT ? kEpiSq8Mip
                                                              : kEpiSq8Dot;
    const Sq8Consts kc =
        (bq || bbq) ? Sq8Consts{0.f, 0.f, 0.f, 0.f, 0.f} : sq8_consts(ix->min_q, ix->max_q, ix->sq_max);
    const int EW = epi_warps_for(mode, KP);
    const int U0 = gemm_scan_units(ntiles, 1 << 20, ix->num_sms, two_sm) * (EW / 4);  // streams per query
    int64_t qch = (int64_t)(scratch_budget() / ((size_t)U0 * (C * 8 + 12)));
    qch = std::max<int64_t>(QB, qch / QB * QB);
    // sized once for the largest chunk and reused by every chunk
    const int qmax = (int)std::min<int64_t>(qch, std::max(nq, 1));
    const int QpMax = (qmax + QB - 1) / QB * QB;
    const int unitsMax = gemm_scan_units(ntiles, QpMax / QB, ix->num_sms, two_sm) * (EW / 4);  // streams
    int8_t* qcodes = S.alloc<int8_t>((size_t)QpMax * ix->Dp8);
    float* qcorr = S.alloc<float>(QpMax);
    int32_t* qsq = S.alloc<int32_t>(QpMax);
    uint64_t* qplanes = bbq ? S.alloc<uint64_t>((size_t)qmax * 4 * ix->nw_pad) : nullptr;
    BbqQuery* qinfo = bbq ? S.alloc<BbqQuery>(QpMax) : nullptr;
    uint64_t* bufs = S.alloc<uint64_t>((size_t)unitsMax * QpMax * C);
    uint32_t* cnts = S.alloc<uint32_t>((size_t)unitsMax * QpMax);
    uint64_t* thrs = S.alloc<uint64_t>((size_t)unitsMax * QpMax);
    uint64_t* floor = S.alloc<uint64_t>(QpMax);
    uint64_t* tops = S.alloc<uint64_t>((size_t)2 * unitsMax * QpMax);
    float* probe = S.alloc<float>((size_t)QpMax * (kPilotRows / 32));
    uint64_t* keys = S.alloc<uint64_t>((size_t)qmax * K);
    uint32_t* kcnt = S.alloc<uint32_t>(qmax);
    uint64_t* keys2 = K > KP ? S.alloc<uint64_t>((size_t)qmax * KP) : nullptr;  // one later pass
    uint32_t* kcnt2 = K > KP ? S.alloc<uint32_t>(qmax) : nullptr;
    uint64_t* ceil = K > KP ? S.alloc<uint64_t>(QpMax) : nullptr;
    int32_t* nflag = S.alloc<int32_t>(1);
    int32_t* flag_list = S.alloc<int32_t>(qmax);
    // row windows: the int8 operand of win_rows rows, one window's keys, the other half of the
    // running keys' double buffer, the floors carried between windows
    const bool windowed = ix->bq_windows && !ix->codes8;
    const int64_t win_rows = windowed ? bq_window_rows(ix->n, ix->Dp8) : 0;
    int8_t* win8 = windowed ? S.alloc<int8_t>((size_t)win_rows * ix->Dp8) : nullptr;
    uint64_t* wkeys = windowed ? S.alloc<uint64_t>((size_t)qmax * K) : nullptr;
    uint32_t* wcnt = windowed ? S.alloc<uint32_t>(qmax) : nullptr;
    uint64_t* keys_alt = windowed ? S.alloc<uint64_t>((size_t)qmax * K) : nullptr;
    uint32_t* kcnt_alt = windowed ? S.alloc<uint32_t>(qmax) : nullptr;
    uint64_t* wseed = windowed ? S.alloc<uint64_t>(QpMax) : nullptr;
    for (int q0 = 0; q0 < nq; q0 += (int)qch) {
      const int qc = (int)std::min<int64_t>(qch, nq - q0);
      const int mblocks = (qc + QB - 1) / QB;
      const int Qp = mblocks * QB;
      const float* dqc = dq + (size_t)q0 * dim;
      VX_CUDA(cudaMemsetAsync(qcodes + (size_t)qc * ix->Dp8, 0, (size_t)(Qp - qc) * ix->Dp8, st));
      if (bq) {
        VX_LAUNCH(1, launch_bq_queries_to_i8(dqc, qc, dim, ix->Dp8, qcodes, st));
      } else if (bbq) {
        VX_LAUNCH(1, launch_bbq_prep_queries(dqc, qc, dim, ix->bbq_centroid, ix->nw_pad, qplanes, qinfo, st));
        VX_LAUNCH(1, launch_bbq_planes_to_i8(qplanes, qc, dim, ix->nw_pad, ix->Dp8, qcodes, st));
      } else {
        VX_LAUNCH(1, launch_sq8_encode_queries(dqc, qc, dim, ix->Dp8, kc, qcodes, qcorr, qsq, st));
      }
      CUtensorMap tmq;
      make_tmap(&tmq, qcodes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ix->Dp8, Qp, 128);
      ScanArgs a;
      a.n = ix->n;
      a.nq = qc;
      a.num_mblocks = mblocks;
      a.kchunks = ix->Dp8 / 128;
      a.ntiles = ntiles;
      a.K = KP;
      a.C = C;
      a.bufs = bufs;
      a.cnts = cnts;
      a.thrs = thrs;
      a.err = d_err;
      a.timeout_ns = wait_timeout_ns();
      a.epi_warps = EW;
      a.epi.xnorm = nullptr;
      a.epi.rowsq = nullptr;
      a.epi.qscale = qcorr;
      a.epi.vcorr = ix->vcorr;
      a.epi.qsq = qsq;
      a.epi.vsq = ix->vsq;
      a.epi.cm = kc.cm;
      a.epi.bits = dim;
      a.epi.bbq_rows = ix->bbq_epi;
      a.epi.bbq_q = qinfo;
      // The K best keys of rows [0, rows) of the int8 operand behind tmrows into out: one scan,
      // or (K wider than a stream) a first pass into a KP-wide buffer, re-strided to K, then
      // passes below the ceilings.  seed: admission floors from earlier row windows (nullable).
      auto select = [&](const CUtensorMap& tmrows, int64_t rows, const float4* epi_rows, const uint64_t* seed,
                        uint64_t* out, uint32_t* out_cnt) {
        ScanArgs w = a;
        w.n = rows;
        w.ntiles = (rows + 255) / 256;
        w.epi.bbq_rows = epi_rows;
        const int wunits = gemm_scan_units(w.ntiles, mblocks, ix->num_sms, two_sm);
        if (K == KP) {
          scan_and_merge(mode, tmq, tmrows, w, wunits, R, Qp, floor, tops, probe, out, out_cnt, st, seed);
          return;
        }
        scan_and_merge(mode, tmq, tmrows, w, wunits, R, Qp, floor, tops, probe, keys2, kcnt2, st, seed);
        VX_CUDA(cudaMemcpy2DAsync(out, (size_t)K * 8, keys2, (size_t)KP * 8, (size_t)KP * 8, qc,
                                  cudaMemcpyDeviceToDevice, st));
        VX_CUDA(cudaMemcpyAsync(out_cnt, kcnt2, (size_t)qc * 4, cudaMemcpyDeviceToDevice, st));
        for (int got = KP; got < K; got += KP) {
          const int K2 = std::min(KP, K - got);
          VX_CUDA(cudaMemsetAsync(ceil, 0, (size_t)Qp * 8, st));
          VX_LAUNCH(1, launch_pass_ceilings(out, out_cnt, qc, K, got, ceil, st));
          ScanArgs b = w;
          b.K = K2;
          b.ceil = ceil;
          scan_and_merge(mode, tmq, tmrows, b, wunits, R, Qp, floor, tops, probe, keys2, kcnt2, st, seed);
          VX_LAUNCH(1, launch_pass_append(out, out_cnt, qc, K, got, keys2, kcnt2, K2, st));
        }
      };
      if (!windowed) {
        select(ix->tm_codes8, ix->n, ix->bbq_epi, nullptr, keys, kcnt);
      } else {
        // Row windows (BQ / BBQ above VX_BQ_TENSOR_BYTES): each window's bits are expanded to
        // the int8 operand in a scratch buffer, scanned, and merged into the running K best;
        // every window after the first admits only keys above the K-th best of those before.
        const int nwin = (int)((ix->n + win_rows - 1) / win_rows);
        VX_CUDA(cudaMemsetAsync(wseed, 0, (size_t)QpMax * 8, st));
        const uint64_t* run = nullptr;
        const uint32_t* run_cnt = nullptr;
        for (int wi = 0; wi < nwin; wi++) {
          const int64_t b0 = (int64_t)wi * win_rows;
          const int64_t rows = std::min<int64_t>(win_rows, ix->n - b0);
          VX_LAUNCH(1, launch_bq_words_to_i8(ix->words + (size_t)b0 * ix->nw_pad, rows, ix->nw_pad, dim, ix->Dp8,
                                             win8, st, bbq));
          CUtensorMap tmw;
          make_tmap(&tmw, win8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ix->Dp8, rows, gemm_scan_db_box(two_sm));
          select(tmw, rows, bbq ? ix->bbq_epi + b0 : nullptr, wi ? wseed : nullptr, wkeys, wcnt);
          // alternate buffers so that the last window's merge lands in keys
          const bool to_keys = (nwin - 1 - wi) % 2 == 0;
          uint64_t* dst = to_keys ? keys : keys_alt;
          uint32_t* dst_cnt = to_keys ? kcnt : kcnt_alt;
          VX_LAUNCH(1, launch_window_merge(run, run_cnt, wkeys, wcnt, qc, K, (uint32_t)b0, dst, dst_cnt, wseed, st));
          run = dst;
          run_cnt = dst_cnt;
        }
      }
      if (rescore) {
        RescoreArgs r{};
        r.nq = qc;
        r.dim = dim;
        r.k = k_out;
        r.Kc = K;
        r.flavor = kFlavorFlat;
        r.metric = ix->metric;
        r.queries = dqc;
        r.rows = ix->rows32;
        r.row_stride = dim;
        r.cand = keys;
        r.cand_cnt = kcnt;
        r.check_margin = 0;
        r.n_rows = ix->n;
        r.out_ids = d_ids + (size_t)q0 * k_out;
        r.out_scores = d_scores + (size_t)q0 * k_out;
        r.out_counts = d_counts + q0;
        r.nflag = nflag;
        r.flag_list = flag_list;
        VX_LAUNCH(1, launch_rescore(r, false, st));
      } else {
        VX_LAUNCH(1, launch_finish_keys(keys, kcnt, qc, K, k_out, bq ? kFinishNegHamming : kFinishFloatKey,
                                        ix->metric, dim,
                                        d_ids + (size_t)q0 * k_out, d_scores + (size_t)q0 * k_out,
                                        d_counts + q0, st));
      }
    }
  } else {  // BQ
    const StreamGeom g = stream_geom(K, 32);
    if (g.R < 0) return fail(VX_ERR_UNSUPPORTED, "k=%d is larger than this build supports", K);
    const int parts = bq_parts(ix->n, ix->num_sms);
    int64_t qch = (int64_t)(scratch_budget() / ((size_t)parts * (g.C * 8 + 12)));
    qch = std::max<int64_t>(256, qch / 256 * 256);
    // sized once for the largest chunk and reused by every chunk
    const int qmax = (int)std::min<int64_t>(qch, std::max(nq, 1));
    const bool bbq = ix->kind == VX_KIND_BBQ;
    uint64_t* qw = S.alloc<uint64_t>((size_t)qmax * ix->nw_pad * (bbq ? 4 : 1));
    BbqQuery* qinfo = bbq ? S.alloc<BbqQuery>(qmax) : nullptr;
    uint64_t* bufs = S.alloc<uint64_t>((size_t)parts * qmax * g.C);
    uint32_t* cnts = S.alloc<uint32_t>((size_t)parts * qmax);
    uint64_t* thrs = S.alloc<uint64_t>((size_t)parts * qmax);
    uint64_t* keys = S.alloc<uint64_t>((size_t)qmax * K);
    uint32_t* kcnt = S.alloc<uint32_t>(qmax);
    int32_t* nflag = S.alloc<int32_t>(1);
    int32_t* flag_list = S.alloc<int32_t>(qmax);
    for (int q0 = 0; q0 < nq; q0 += (int)qch) {
      const int qc = (int)std::min<int64_t>(qch, nq - q0);
      const float* dqc = dq + (size_t)q0 * dim;
      VX_CUDA(cudaMemsetAsync(cnts, 0, (size_t)parts * qc * 4, st));
      VX_CUDA(cudaMemsetAsync(thrs, 0, (size_t)parts * qc * 8, st));
      if (bbq) {
        VX_LAUNCH(1, launch_bbq_prep_queries(dqc, qc, dim, ix->bbq_centroid, ix->nw_pad, qw, qinfo, st));
        VX_TIMED(VX_PROF_BQ_SCAN, st, 1,
                 launch_bbq_scan(ix->words, ix->bbq_rows, ix->n, ix->nw_pad, dim, ix->metric, qw, qinfo, qc, parts, g,
                                 bufs, cnts, thrs, st));
      } else {
        VX_LAUNCH(1, launch_bq_pack_queries(dqc, qc, dim, ix->nw_pad, qw, st));
        VX_TIMED(VX_PROF_BQ_SCAN, st, 1,
                 launch_bq_scan(ix->words, ix->n, ix->nw_pad, qw, qc, parts, g, bufs, cnts, thrs, st));
      }
      VX_LAUNCH(1, launch_merge_streams(bufs, cnts, parts, qc, qc, g.C, K, keys, kcnt, st));
      if (rescore) {
        RescoreArgs r{};
        r.nq = qc;
        r.dim = dim;
        r.k = k_out;
        r.Kc = K;
        r.flavor = kFlavorFlat;
        r.metric = ix->metric;
        r.queries = dqc;
        r.rows = ix->rows32;
        r.row_stride = dim;
        r.cand = keys;
        r.cand_cnt = kcnt;
        r.check_margin = 0;
        r.n_rows = ix->n;
        r.out_ids = d_ids + (size_t)q0 * k_out;
        r.out_scores = d_scores + (size_t)q0 * k_out;
        r.out_counts = d_counts + q0;
        r.nflag = nflag;
        r.flag_list = flag_list;
        VX_LAUNCH(1, launch_rescore(r, false, st));
      } else {
        VX_LAUNCH(1, launch_finish_keys(keys, kcnt, qc, K, k_out, bbq ? kFinishFloatKey : kFinishHamming, ix->metric, dim,
                                        d_ids + (size_t)q0 * k_out, d_scores + (size_t)q0 * k_out,
                                        d_counts + q0, st));
      }
    }
  }
  return check_device_error(d_err, st);
}

// IVF-PQ: IvfIndex.pqSearch.
// IVF-flat: IvfIndex.search without PQ (IvfIndex.java:170-226).  Routing as for IVF-PQ, then
// the (query, list) pairs grouped by list (up to 64 per group) through the flat list scan, the
// per-list best K merged per query.
// heap_k (>= k) is the size of the reference's TopKHeap, k the hits returned: they differ when
// IvfFlatAdapter widens a search (candidateK = ceil(k * overQueryFactor)) and trims it to k,
// which changes where the EUCLIDEAN early exit stops.
constexpr int64_t kFlatPartRows = 1024;              // rows per part of a long list (a multiple of 64)
constexpr size_t kFlatPartBytes = (size_t)512 << 20;  // cap on the parts' key buffer of one chunk

// The IVF-flat list scan of one chunk's (query, slot) pairs: out [width][qc][K] keys and out_cnt
// [width][qc] per slot (lists [qc][width]; -1: no list).  qfloor (nullable, zeroed here): each
// query's K-th best key over the lists scanned so far, which bounds admission in its later
// lists -- null where every list's own K best are needed (the EUCLIDEAN early exit).  Returns
// the zero-padded queries [qc][Dp] (the HARMONY scan reads them too).
float* ivfflat_scan(vx_index* ix, const float* dqc, int qc, int width, int K, const int32_t* lists, uint64_t* qfloor,
                    uint64_t* out, uint32_t* out_cnt, Scratch& T, cudaStream_t st) {
  const int dim = ix->dim, Dp = ix->Dp_flat;
  int32_t* counts = T.alloc<int32_t>(ix->nlist);
  int32_t* offsets = T.alloc<int32_t>(ix->nlist + 1);
  int32_t* cursor = T.alloc<int32_t>(ix->nlist);
  int32_t* pairs = T.alloc<int32_t>((size_t)qc * width);
  float* qpad = T.alloc<float>((size_t)qc * Dp);
  float* qnorm = T.alloc<float>(qc);
  float* tail = T.alloc<float>((size_t)qc * width * 3);
  // Lists longer than kFlatPartRows rows are scanned in row parts (one group per part), so that
  // the longest list does not bound the kernel; the parts' results take pmax * K keys per pair
  // slot, kept within kFlatPartBytes (fewer, longer parts when that would be exceeded).
  const size_t slots = (size_t)qc * width;
  int rmax = 0, pmax = 1;
  if (ix->max_list_rows > kFlatPartRows) {
    const int64_t cap = std::max<int64_t>(
        1, std::min<int64_t>((int64_t)(kFlatPartBytes / (slots * (size_t)K * 8 + 1)), kFlatPartKeysMax / K));
    int64_t r = kFlatPartRows;
    while ((ix->max_list_rows + r - 1) / r > cap) r *= 2;
    if ((ix->max_list_rows + r - 1) / r > 1) {
      rmax = (int)r;
      pmax = (int)((ix->max_list_rows + r - 1) / r);
    }
  }
  const int64_t maxg = ((int64_t)qc * width / kFlatGroup + ix->nlist + 1) * pmax;
  int2* groups = T.alloc<int2>((size_t)maxg);
  int32_t* ngroups = T.alloc<int32_t>(2);  // count, dispenser
  uint64_t* part_out = pmax > 1 ? T.alloc<uint64_t>(slots * pmax * K) : nullptr;
  uint32_t* part_cnt = pmax > 1 ? T.alloc<uint32_t>(slots * pmax) : nullptr;
  VX_LAUNCH(1, launch_pad_rows(dqc, qc, dim, dim, nullptr, Dp, qpad, st));
  if (ix->metric == VX_COSINE) VX_LAUNCH(1, launch_row_norms(qpad, qc, dim, Dp, qnorm, st));
  VX_LAUNCH(3, launch_group_pairs(lists, ix->list_off, qc * width, ix->nlist, counts, offsets, cursor, pairs, st));
  VX_CUDA(cudaMemsetAsync(out_cnt, 0, (size_t)width * qc * 4, st));
  if (part_cnt) VX_CUDA(cudaMemsetAsync(part_cnt, 0, slots * pmax * 4, st));
  if (qfloor) VX_CUDA(cudaMemsetAsync(qfloor, 0, (size_t)qc * 8, st));
  VX_LAUNCH(1, launch_make_groups(counts, offsets, ix->list_order, ix->nlist, kFlatGroup, groups, ngroups, st,
                                  ix->list_off, rmax));
  FlatListArgs a{};
  a.nq = qc;
  a.dim = dim;
  a.Dp = Dp;
  a.nprobe = width;
  a.metric = ix->metric;
  a.K = K;
  a.pairs = pairs;
  a.pair_count = offsets + ix->nlist;
  a.groups = groups;
  a.ngroups = ngroups;
  a.lists = lists;
  a.queries = qpad;
  a.qnorm = qnorm;
  a.list_off = ix->list_off;
  a.ordinals = ix->ordinals;
  a.rows = ix->flat_rows;
  a.rnorm = ix->flat_norms;
  a.tail = tail;
  a.out = out;
  a.out_cnt = out_cnt;
  a.floor = qfloor;
  a.rmax = rmax;
  a.pmax = pmax;
  a.part_out = part_out;
  a.part_cnt = part_cnt;
  VX_TIMED(VX_PROF_ADC_SCAN, st, 2, launch_flat_list(a, (int64_t)qc * width, ix->num_sms * 2, st));
  if (pmax > 1) VX_LAUNCH(1, launch_flat_parts_merge(a, (int64_t)qc * width, st));
  return qpad;
}

int search_ivfflat(vx_index* ix, const float* dq, int nq, int k, int heap_k, int nprobe, float min_score,
                   int32_t* d_ids, float* d_scores, int32_t* d_counts, cudaStream_t st, const int32_t* given_lists) {
  const int dim = ix->dim, Dp = ix->Dp_flat;
  const int probes = std::min(nprobe, ix->nlist);
  const int K = (int)std::max<int64_t>(1, std::min<int64_t>(std::max(k, heap_k), ix->n));
  if (!flat_list_supported(K)) return fail(VX_ERR_UNSUPPORTED, "k = %d is larger than the IVF-flat scan keeps (256)", K);
  // Routed here (not given): SOAR spill targets widen each query's list to 2 * probes slots,
  // and EUCLIDEAN takes the reference's early exit over the per-list results in route order.
  const bool spill = !given_lists && ix->spill && ix->gamma > 0.0f;
  const bool early_exit = !given_lists && ix->metric == VX_EUCLIDEAN && ix->radii;
  const int width = spill ? 2 * probes : probes;
  const size_t per_q = (size_t)ix->nlist * 4 + (size_t)Dp * 4 + (size_t)width * (K * 8 + 8 + 12 + 8) + 64;
  const int64_t qch = std::max<int64_t>(64, (int64_t)(scratch_budget() / per_q));
  Scratch S(st);
  int32_t* d_bad = S.alloc<int32_t>(1);
  VX_CUDA(cudaMemsetAsync(d_bad, 0, 4, st));
  for (int q0 = 0; q0 < nq; q0 += (int)qch) {
    const int qc = (int)std::min<int64_t>(qch, nq - q0);
    Scratch T(st);
    const float* dqc = dq + (size_t)q0 * dim;
    float* qn = T.alloc<float>((size_t)qc * dim);
    float* dist = T.alloc<float>((size_t)qc * ix->nlist);
    int32_t* routed = T.alloc<int32_t>((size_t)qc * probes);
    int32_t* lists = routed;
    float* ldist = nullptr;
    uint64_t* out = T.alloc<uint64_t>((size_t)width * qc * K);
    uint32_t* out_cnt = T.alloc<uint32_t>((size_t)width * qc);
    uint64_t* keys = T.alloc<uint64_t>((size_t)qc * K);
    uint32_t* kcnt = T.alloc<uint32_t>(qc);
    uint64_t* qfloor = early_exit ? nullptr : T.alloc<uint64_t>(qc);
    const bool harmony = early_exit && ix->keyed;
    uint64_t* harm = harmony ? T.alloc<uint64_t>((size_t)width * qc * K) : nullptr;
    uint32_t* harm_cnt = harmony ? T.alloc<uint32_t>((size_t)width * qc) : nullptr;
    if (given_lists) {
      VX_LAUNCH(1, launch_copy_lists(given_lists + (size_t)q0 * probes, qc * probes, ix->nlist, lists, d_bad, st));
    } else {
      VX_TIMED(VX_PROF_ROUTE, st, route_launches(dqc, dim, ix->cent, ix->nlist, ix->metric),
               launch_route(dqc, qc, dim, ix->cent, ix->nlist, ix->metric, probes, qn, dist, routed, st));
      if (spill || early_exit) {
        lists = T.alloc<int32_t>((size_t)qc * width);
        ldist = T.alloc<float>((size_t)qc * width);
        VX_LAUNCH(1, launch_route_expand(routed, qc, probes, dist, ix->nlist, ix->metric, spill ? ix->gamma : 0.0f,
                                         spill ? ix->spill : nullptr, width, lists, ldist, st));
      }
    }
    float* qpad = ivfflat_scan(ix, dqc, qc, width, K, lists, qfloor, out, out_cnt, T, st);
    if (harmony) {
      HarmonyArgs h{};
      h.nq = qc;
      h.width = width;
      h.K = K;
      h.dim = dim;
      h.Dp = Dp;
      h.lists = lists;
      h.keyed = ix->keyed;
      h.list_off = ix->list_off;
      h.ordinals = ix->ordinals;
      h.rows = ix->flat_rows;
      h.queries = qpad;
      h.out = harm;
      h.out_cnt = harm_cnt;
      VX_TIMED(VX_PROF_ADC_SCAN, st, 1, launch_harmony_lists(h, st));
    }
    if (early_exit) {
      VX_TIMED(VX_PROF_MERGE, st, 1,
               launch_ivf_early_exit(out, out_cnt, qc, width, K, lists, ldist, ix->radii, ix->metric, min_score, harm,
                                     harm_cnt, ix->keyed, keys, kcnt, st));
    } else {
      VX_TIMED(VX_PROF_MERGE, st, 1, launch_merge_streams(out, out_cnt, width, qc, qc, K, K, keys, kcnt, st));
    }
    int32_t* oi = d_ids + (size_t)q0 * k;
    float* os = d_scores + (size_t)q0 * k;
    int32_t* oc = d_counts + q0;
    VX_LAUNCH(1, launch_finish_keys(keys, kcnt, qc, K, k, kFinishFloatKey, ix->metric, dim, oi, os, oc, st));
    VX_LAUNCH(1, launch_min_score(os, qc, k, min_score, oc, st));
  }
  if (given_lists) {
    int32_t h_bad = 0;
    VX_CUDA(cudaMemcpyAsync(&h_bad, d_bad, 4, cudaMemcpyDeviceToHost, st));
    VX_CUDA(cudaStreamSynchronize(st));
    if (h_bad) return fail(VX_ERR_INVALID_ARGUMENT, "%d routed list ids are outside [-1, nlist)", h_bad);
  }
  return VX_OK;
}

// IVF-flat split across GPUs by (query, list) pair: the scan of the pairs a rank owns (every
// query's slots in lists [nq][width], -1 for the slots of other ranks) into per-slot results,
// and the merge of all ranks' per-slot results (summed: each slot's keys come from one rank, the
// others hold zeros) in route order with the reference's early exit.  Together they give
// search_ivfflat's results for the same routed lists and distances.
int ivfflat_scan_pairs(vx_index* ix, const float* dq, int nq, int K, int width, const int32_t* lists,
                       uint64_t* pair_keys, uint32_t* pair_counts, cudaStream_t st) {
  const bool early_exit = ix->metric == VX_EUCLIDEAN && ix->radii;
  Scratch T(st);
  int32_t* checked = T.alloc<int32_t>((size_t)nq * width);
  int32_t* d_bad = T.alloc<int32_t>(1);
  VX_CUDA(cudaMemsetAsync(d_bad, 0, 4, st));
  VX_LAUNCH(1, launch_copy_lists(lists, nq * width, ix->nlist, checked, d_bad, st));
  uint64_t* qfloor = early_exit ? nullptr : T.alloc<uint64_t>(nq);
  VX_CUDA(cudaMemsetAsync(pair_keys, 0, (size_t)width * nq * K * 8, st));
  ivfflat_scan(ix, dq, nq, width, K, checked, qfloor, pair_keys, pair_counts, T, st);
  int32_t h_bad = 0;
  VX_CUDA(cudaMemcpyAsync(&h_bad, d_bad, 4, cudaMemcpyDeviceToHost, st));
  VX_CUDA(cudaStreamSynchronize(st));
  if (h_bad) return fail(VX_ERR_INVALID_ARGUMENT, "%d routed list ids are outside [-1, nlist)", h_bad);
  return VX_OK;
}

int ivfflat_merge_pairs(vx_index* ix, int nq, int k, int K, int width, const int32_t* lists, const float* ldist,
                        const uint64_t* pair_keys, const uint32_t* pair_counts, float min_score, int32_t* d_ids,
                        float* d_scores, int32_t* d_counts, cudaStream_t st) {
  Scratch T(st);
  uint64_t* keys = T.alloc<uint64_t>((size_t)nq * K);
  uint32_t* kcnt = T.alloc<uint32_t>(nq);
  if (ix->metric == VX_EUCLIDEAN && ix->radii) {
    VX_TIMED(VX_PROF_MERGE, st, 1,
             launch_ivf_early_exit(pair_keys, pair_counts, nq, width, K, lists, ldist, ix->radii, ix->metric,
                                   min_score, nullptr, nullptr, nullptr, keys, kcnt, st));
  } else {
    VX_TIMED(VX_PROF_MERGE, st, 1, launch_merge_streams(pair_keys, pair_counts, width, nq, nq, K, K, keys, kcnt, st));
  }
  VX_LAUNCH(1, launch_finish_keys(keys, kcnt, nq, K, k, kFinishFloatKey, ix->metric, ix->dim, d_ids, d_scores,
                                  d_counts, st));
  VX_LAUNCH(1, launch_min_score(d_scores, nq, k, min_score, d_counts, st));
  return VX_OK;
}

// Routing with each routed list's distance (the early exit's bound needs it): lists and
// distances [nq][min(nprobe, nlist)], nearest first, no SOAR spill.
int route_ivf_dist(vx_index* ix, const float* dq, int nq, int nprobe, int32_t* d_lists, float* d_dist,
                   cudaStream_t st) {
  const int dim = ix->dim;
  const int probes = std::min(nprobe, ix->nlist);
  const size_t per_q = (size_t)ix->nlist * 4 + (size_t)dim * 4 + (size_t)probes * 4 + 64;
  const int64_t qch = std::max<int64_t>(64, (int64_t)(scratch_budget() / per_q));
  for (int q0 = 0; q0 < nq; q0 += (int)qch) {
    const int qc = (int)std::min<int64_t>(qch, nq - q0);
    Scratch T(st);
    const float* dqc = dq + (size_t)q0 * dim;
    float* qn = T.alloc<float>((size_t)qc * dim);
    float* dist = T.alloc<float>((size_t)qc * ix->nlist);
    int32_t* routed = T.alloc<int32_t>((size_t)qc * probes);
    VX_TIMED(VX_PROF_ROUTE, st, route_launches(dqc, dim, ix->cent, ix->nlist, ix->metric),
             launch_route(dqc, qc, dim, ix->cent, ix->nlist, ix->metric, probes, qn, dist, routed, st));
    VX_LAUNCH(1, launch_route_expand(routed, qc, probes, dist, ix->nlist, ix->metric, 0.0f, nullptr, probes,
                                     d_lists + (size_t)q0 * probes, d_dist + (size_t)q0 * probes, st));
  }
  return VX_OK;
}

int search_ivfpq(vx_index* ix, const float* dq, int nq, int k, int nprobe, int rescore,
                 float min_score, int32_t* d_ids, float* d_scores, int32_t* d_counts,
                 cudaStream_t st, const int32_t* given_lists = nullptr) {
  if (ix->kind == VX_KIND_IVFFLAT)  // IvfIndex.search takes the flat scan when there is no PQ
    return search_ivfflat(ix, dq, nq, k, k, nprobe, min_score, d_ids, d_scores, d_counts, st, given_lists);
  const int dim = ix->dim;
  const int probes = std::min(nprobe, ix->nlist);
  int64_t wide = std::min<int64_t>((int64_t)k * rescore, ix->n);
  if (wide < 1) wide = 1;
  const int K = (int)wide;
  const StreamGeom g = stream_geom(K, 32);
  if (g.R < 0) return fail(VX_ERR_UNSUPPORTED, "k * rescoreFactor = %d is larger than supported", K);
  if (rescore > 1 && !ix->rows32)
    return fail(VX_ERR_UNSUPPORTED, "rescoreFactor > 1 needs the full-precision vectors at build");
  // Routed here (not given): SOAR spill targets widen each query's list to 2 * probes slots.
  const bool spill = !given_lists && ix->spill && ix->gamma > 0.0f;
  const int width = spill ? 2 * probes : probes;
  // chunk queries: distances [qc][nlist] + outputs [width][qc][K]
  const size_t per_q = (size_t)ix->nlist * 4 + (size_t)width * (K * 8 + 8 + 12) + 64;
  int64_t qch = std::max<int64_t>(64, (int64_t)(scratch_budget() / per_q));
  Scratch S(st);
  int32_t* d_bad = S.alloc<int32_t>(1);
  VX_CUDA(cudaMemsetAsync(d_bad, 0, 4, st));
  for (int q0 = 0; q0 < nq; q0 += (int)qch) {
    const int qc = (int)std::min<int64_t>(qch, nq - q0);
    Scratch T(st);
    const float* dqc = dq + (size_t)q0 * dim;
    float* qn = T.alloc<float>((size_t)qc * dim);
    float* dist = T.alloc<float>((size_t)qc * ix->nlist);
    int32_t* routed = T.alloc<int32_t>((size_t)qc * probes);
    int32_t* lists = routed;
    int32_t* counts = T.alloc<int32_t>(ix->nlist);
    int32_t* offsets = T.alloc<int32_t>(ix->nlist + 1);
    int32_t* cursor = T.alloc<int32_t>(ix->nlist);
    int32_t* pairs = T.alloc<int32_t>((size_t)qc * width);
    uint64_t* out = T.alloc<uint64_t>((size_t)width * qc * K);
    uint32_t* out_cnt = T.alloc<uint32_t>((size_t)width * qc);
    uint64_t* keys = T.alloc<uint64_t>((size_t)qc * K);
    uint32_t* kcnt = T.alloc<uint32_t>(qc);
    if (given_lists) {
      // routed beforehand (possibly by another rank): checked copy, ids outside the index -> -1
      VX_LAUNCH(1, launch_copy_lists(given_lists + (size_t)q0 * probes, qc * probes, ix->nlist, lists, d_bad, st));
    } else {
      VX_TIMED(VX_PROF_ROUTE, st, route_launches(dqc, dim, ix->cent, ix->nlist, ix->metric),
               launch_route(dqc, qc, dim, ix->cent, ix->nlist, ix->metric, probes, qn, dist, routed, st));
      if (spill) {
        lists = T.alloc<int32_t>((size_t)qc * width);
        float* ldist = T.alloc<float>((size_t)qc * width);
        VX_LAUNCH(1, launch_route_expand(routed, qc, probes, dist, ix->nlist, ix->metric, ix->gamma, ix->spill, width,
                                         lists, ldist, st));
      }
    }
    VX_LAUNCH(3, launch_group_pairs(lists, ix->list_off, qc * width, ix->nlist, counts, offsets, cursor, pairs, st));
    VX_CUDA(cudaMemsetAsync(out_cnt, 0, (size_t)width * qc * 4, st));
    AdcArgs a;
    a.nq = qc;
    a.dim = dim;
    a.nprobe = width;
    a.metric = ix->metric;
    a.M = ix->M;
    a.Ks = ix->Ks;
    a.Mp = ix->Mp;
    a.K = K;
    a.npairs = (int64_t)qc * width;
    a.pairs = pairs;
    a.pair_count = offsets + ix->nlist;
    a.lists = lists;
    a.queries = dqc;
    a.cent = ix->cent;
    a.list_off = ix->list_off;
    a.ordinals = ix->ordinals;
    a.codes = ix->pq_codes;
    a.codebooks = ix->codebooks;
    a.cb_off = ix->cb_off;
    a.sub = ix->sub;
    a.out = out;
    a.out_cnt = out_cnt;
    a.groups = nullptr;
    a.ngroups = nullptr;
    a.floor = nullptr;
    const int grid = ix->num_sms * 2;
    const StreamGeom gg = stream_geom(K, std::max(32, K));  // group buffers hold >= 2K keys
    if (use_adc_group() && adc_group_supported(ix->M, ix->Ks, dim) && gg.R > 0 && gg.R <= 9) {
      const int64_t maxg = (int64_t)qc * width / kAdcGroupQ + ix->nlist + 1;
      int2* groups = T.alloc<int2>((size_t)maxg);
      int32_t* ngroups = T.alloc<int32_t>(2);  // count, dispenser
      uint64_t* qfloor = T.alloc<uint64_t>(qc);
      VX_CUDA(cudaMemsetAsync(qfloor, 0, (size_t)qc * 8, st));
      VX_LAUNCH(1, launch_make_groups(counts, offsets, ix->list_order, ix->nlist, kAdcGroupQ, groups, ngroups, st));
      a.groups = groups;
      a.ngroups = ngroups;
      a.floor = qfloor;
      VX_TIMED(VX_PROF_ADC_SCAN, st, 1, launch_adc_group(a, gg.R, grid, st));
    } else {
      VX_TIMED(VX_PROF_ADC_SCAN, st, 1, launch_adc_scan(a, g.R, grid, st));
    }
    VX_TIMED(VX_PROF_MERGE, st, 1, launch_merge_streams(out, out_cnt, width, qc, qc, K, K, keys, kcnt, st));
    int32_t* oi = d_ids + (size_t)q0 * k;
    float* os = d_scores + (size_t)q0 * k;
    int32_t* oc = d_counts + q0;
    if (rescore == 1) {
      VX_LAUNCH(1, launch_finish_keys(keys, kcnt, qc, K, k, kFinishFloatKey, ix->metric, dim, oi, os, oc, st));
    } else {
      RescoreArgs r{};
      r.nq = qc;
      r.dim = dim;
      r.k = k;
      r.Kc = K;
      r.flavor = kFlavorIvfRaw;
      r.metric = ix->metric;
      r.queries = dqc;
      r.rows = ix->rows32;
      r.row_stride = dim;
      r.cand = keys;
      r.cand_cnt = kcnt;
      r.check_margin = 0;
      r.n_rows = ix->n;
      r.out_ids = oi;
      r.out_scores = os;
      r.out_counts = oc;
      r.nflag = T.alloc<int32_t>(1);
      r.flag_list = T.alloc<int32_t>(qc);
      VX_LAUNCH(1, launch_rescore(r, false, st));
    }
    VX_LAUNCH(1, launch_min_score(os, qc, k, min_score, oc, st));
  }
  if (given_lists) {
    int32_t h_bad = 0;
    VX_CUDA(cudaMemcpyAsync(&h_bad, d_bad, 4, cudaMemcpyDeviceToHost, st));
    VX_CUDA(cudaStreamSynchronize(st));
    if (h_bad) return fail(VX_ERR_INVALID_ARGUMENT, "%d routed list ids are outside [-1, nlist)", h_bad);
  }
  return VX_OK;
}

// CentroidIndex routing alone: the min(nprobe, nlist) nearest lists of every query.
int route_ivf(vx_index* ix, const float* dq, int nq, int nprobe, int32_t* d_lists, cudaStream_t st) {
  const int dim = ix->dim;
  const int probes = std::min(nprobe, ix->nlist);
  const size_t per_q = (size_t)ix->nlist * 4 + (size_t)dim * 4 + 64;
  const int64_t qch = std::max<int64_t>(64, (int64_t)(scratch_budget() / per_q));
  for (int q0 = 0; q0 < nq; q0 += (int)qch) {
    const int qc = (int)std::min<int64_t>(qch, nq - q0);
    Scratch T(st);
    const float* dqc = dq + (size_t)q0 * dim;
    float* qn = T.alloc<float>((size_t)qc * dim);
    float* dist = T.alloc<float>((size_t)qc * ix->nlist);
    VX_TIMED(VX_PROF_ROUTE, st, route_launches(dqc, dim, ix->cent, ix->nlist, ix->metric),
             launch_route(dqc, qc, dim, ix->cent, ix->nlist, ix->metric, probes, qn, dist,
                          d_lists + (size_t)q0 * probes, st));
  }
  return VX_OK;
}

void fill_empty(int nq, int k, int32_t* d_ids, float* d_scores, int32_t* d_counts, cudaStream_t st) {
  if (nq <= 0) return;
  VX_CUDA(cudaMemsetAsync(d_counts, 0, (size_t)nq * 4, st));
  VX_CUDA(cudaMemsetAsync(d_ids, 0xFF, (size_t)nq * k * 4, st));
  VX_CUDA(cudaMemsetAsync(d_scores, 0, (size_t)nq * k * 4, st));
}

int validate_search(vx_index* ix, const void* q, int nq, int dim, int k, const void* a,
                    const void* b, const void* c) {
  if (!ix) return fail(VX_ERR_NULL_POINTER, "index must not be null");
  if (!q) return fail(VX_ERR_NULL_POINTER, "queries must not be null");
  if (!a || !b || !c) return fail(VX_ERR_NULL_POINTER, "output buffers must not be null");
  if (nq <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "queries must not be empty");
  if (k <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "k must be positive: %d", k);
  if (ix->n > 0 && dim != ix->dim)
    return fail(VX_ERR_INVALID_ARGUMENT, "Query dimension %d does not match index dimension %d", dim,
                ix->dim);
  return VX_OK;
}

// Exact-search view of a quantized index that was built with its fp32 rows: a FLAT index
// sharing those rows, created on first use (QuantizedFlatScanAdapter's `exact` delegate).
vx_index* flat_view(vx_index* ix) {
  std::lock_guard<std::mutex> g(ix->lazy_mu);
  if (!ix->flat) {
    vx_index* v = new vx_index();
    v->kind = VX_KIND_FLAT;
    v->device = ix->device;
    v->metric = ix->metric;
    v->n = ix->n;
    v->dim = ix->dim;
    v->num_sms = ix->num_sms;
    v->rows32 = ix->rows32;  // borrowed; owned by ix
    try {
      build_unit_f16(v);
    } catch (...) {
      free_index(v);
      throw;
    }
    ix->flat = v;
  }
  return ix->flat;
}

// PQ as a flat quantizer (QuantizedFlatScanAdapter over PQVectors): every query's one "list"
// holds all rows; the ADC kernels build (query - global centroid) tables and score rows with
// PQVectors' transforms; the K best keys per query, then either the reference scores
// (candidates) or the exact fp32 re-score of the two-pass search.
int search_pq_flat(vx_index* ix, const float* dq, int nq, int K, int k_out, bool rescore, int32_t* d_ids,
                   float* d_scores, int32_t* d_counts, cudaStream_t st) {
  const int dim = ix->dim;
  const StreamGeom g = stream_geom(K, 32);
  if (g.R < 0) return fail(VX_ERR_UNSUPPORTED, "k=%d is larger than this build supports", K);
  const StreamGeom gg = stream_geom(K, std::max(32, K));  // group buffers hold >= 2K keys
  const bool grouped = use_adc_group() && adc_group_supported(ix->M, ix->Ks, dim) && gg.R > 0 && gg.R <= 9;
  const size_t per_q = (size_t)K * 8 + 64;
  const int64_t qch = std::max<int64_t>(64, (int64_t)(scratch_budget() / per_q));
  for (int q0 = 0; q0 < nq; q0 += (int)qch) {
    const int qc = (int)std::min<int64_t>(qch, nq - q0);
    Scratch T(st);
    const float* dqc = dq + (size_t)q0 * dim;
    int32_t* lists = T.alloc<int32_t>(qc);
    int32_t* counts = T.alloc<int32_t>(1);
    int32_t* offsets = T.alloc<int32_t>(2);
    int32_t* cursor = T.alloc<int32_t>(1);
    int32_t* pairs = T.alloc<int32_t>(qc);
    float* qnorm = T.alloc<float>(qc);
    uint64_t* out = T.alloc<uint64_t>((size_t)qc * K);
    uint32_t* out_cnt = T.alloc<uint32_t>(qc);
    uint64_t* keys = T.alloc<uint64_t>((size_t)qc * K);
    uint32_t* kcnt = T.alloc<uint32_t>(qc);
    VX_CUDA(cudaMemsetAsync(lists, 0, (size_t)qc * 4, st));  // every query probes list 0
    VX_CUDA(cudaMemsetAsync(out_cnt, 0, (size_t)qc * 4, st));
    if (ix->metric == VX_COSINE) VX_LAUNCH(1, launch_pq_query_norms(dqc, qc, dim, ix->cent, qnorm, st));
    VX_LAUNCH(3, launch_group_pairs(lists, ix->list_off, qc, 1, counts, offsets, cursor, pairs, st));
    AdcArgs a;
    a.nq = qc;
    a.dim = dim;
    a.nprobe = 1;
    a.metric = ix->metric;
    a.M = ix->M;
    a.Ks = ix->Ks;
    a.Mp = ix->Mp;
    a.K = K;
    a.npairs = qc;
    a.pairs = pairs;
    a.pair_count = offsets + 1;
    a.lists = lists;
    a.queries = dqc;
    a.cent = ix->cent;
    a.list_off = ix->list_off;
    a.ordinals = ix->ordinals;
    a.codes = ix->pq_codes;
    a.codebooks = ix->codebooks;
    a.cb_off = ix->cb_off;
    a.sub = ix->sub;
    a.out = out;
    a.out_cnt = out_cnt;
    a.groups = nullptr;
    a.ngroups = nullptr;
    a.floor = nullptr;
    a.pq_flat = 1;
    a.qnorm = ix->metric == VX_COSINE ? qnorm : nullptr;
    a.rnorm = ix->pq_rnorm;
    const int grid = ix->num_sms * 2;
    if (grouped) {
      int2* groups = T.alloc<int2>((size_t)qc / kAdcGroupQ + 2);
      int32_t* ngroups = T.alloc<int32_t>(2);
      uint64_t* qfloor = T.alloc<uint64_t>(qc);
      VX_CUDA(cudaMemsetAsync(qfloor, 0, (size_t)qc * 8, st));
      VX_LAUNCH(1, launch_make_groups(counts, offsets, nullptr, 1, kAdcGroupQ, groups, ngroups, st));
      a.groups = groups;
      a.ngroups = ngroups;
      a.floor = qfloor;
      VX_TIMED(VX_PROF_ADC_SCAN, st, 1, launch_adc_group(a, gg.R, grid, st));
    } else {
      VX_TIMED(VX_PROF_ADC_SCAN, st, 1, launch_adc_scan(a, g.R, grid, st));
    }
    VX_TIMED(VX_PROF_MERGE, st, 1, launch_merge_streams(out, out_cnt, 1, qc, qc, K, K, keys, kcnt, st));
    int32_t* oi = d_ids + (size_t)q0 * k_out;
    float* os = d_scores + (size_t)q0 * k_out;
    int32_t* oc = d_counts + q0;
    if (!rescore) {
      VX_LAUNCH(1, launch_finish_keys(keys, kcnt, qc, K, k_out, kFinishFloatKey, ix->metric, dim, oi, os, oc, st));
    } else {
      RescoreArgs r{};
      r.nq = qc;
      r.dim = dim;
      r.k = k_out;
      r.Kc = K;
      r.flavor = kFlavorFlat;
      r.metric = ix->metric;
      r.queries = dqc;
      r.rows = ix->rows32;
      r.row_stride = dim;
      r.cand = keys;
      r.cand_cnt = kcnt;
      r.check_margin = 0;
      r.n_rows = ix->n;
      r.out_ids = oi;
      r.out_scores = os;
      r.out_counts = oc;
      r.nflag = T.alloc<int32_t>(1);
      r.flag_list = T.alloc<int32_t>(qc);
      VX_LAUNCH(1, launch_rescore(r, false, st));
    }
  }
  return VX_OK;
}

// FP16 two-pass: candidates by the fp16 score function, then exact fp32 re-score.
int search_fp16_two_pass(vx_index* ix, const float* dq, int nq, int ck, int k, int32_t* d_ids,
                         float* d_scores, int32_t* d_counts, cudaStream_t st) {
  Scratch S(st);
  int32_t* ci = S.alloc<int32_t>((size_t)nq * ck);
  float* cs = S.alloc<float>((size_t)nq * ck);
  int32_t* cc = S.alloc<int32_t>(nq);
  uint64_t* keys = S.alloc<uint64_t>((size_t)nq * ck);
  int rc = search_gemm_exact(ix, dq, nq, ck, ci, cs, cc, st);
  if (rc != VX_OK) return rc;
  VX_LAUNCH(1, launch_ids_to_keys(ci, cc, nq, ck, keys, st));
  RescoreArgs r{};
  r.nq = nq;
  r.dim = ix->dim;
  r.k = k;
  r.Kc = ck;
  r.flavor = kFlavorFlat;
  r.metric = ix->metric;
  r.queries = dq;
  r.rows = ix->rows32;
  r.row_stride = ix->dim;
  r.cand = keys;
  r.cand_cnt = (const uint32_t*)cc;
  r.check_margin = 0;
  r.n_rows = ix->n;
  r.out_ids = d_ids;
  r.out_scores = d_scores;
  r.out_counts = d_counts;
  r.nflag = S.alloc<int32_t>(1);
  r.flag_list = S.alloc<int32_t>(nq);
  VX_LAUNCH(1, launch_rescore(r, false, st));
  return VX_OK;
}

// Dispatch of IndexSpi.searchBatch semantics on device buffers.
int search_batch_dev(vx_index* ix, const float* dq, int nq, int dim, int k, int sls, float oqf,
                     int32_t* d_ids, float* d_scores, int32_t* d_counts, cudaStream_t st) {
  if (ix->n == 0) {  // empty index -> empty outcomes (FlatScanAdapter.java:117-122)
    fill_empty(nq, k, d_ids, d_scores, d_counts, st);
    return VX_OK;
  }
  const int kk = (int)std::min<int64_t>(k, ix->n);
  if (kk < k) fill_empty(nq, k, d_ids, d_scores, d_counts, st);
  // outputs are written with row stride k; run with kk and re-stride when needed
  auto run_k = [&](auto&& fn) -> int {
    if (kk == k) return fn(k, d_ids, d_scores, d_counts);
    Scratch S(st);
    int32_t* ti = S.alloc<int32_t>((size_t)nq * kk);
    float* ts = S.alloc<float>((size_t)nq * kk);
    int rc = fn(kk, ti, ts, d_counts);
    if (rc != VX_OK) return rc;
    VX_CUDA(cudaMemcpy2DAsync(d_ids, (size_t)k * 4, ti, (size_t)kk * 4, (size_t)kk * 4, nq,
                              cudaMemcpyDeviceToDevice, st));
    VX_CUDA(cudaMemcpy2DAsync(d_scores, (size_t)k * 4, ts, (size_t)kk * 4, (size_t)kk * 4, nq,
                              cudaMemcpyDeviceToDevice, st));
    return VX_OK;
  };
  switch (ix->kind) {
    case VX_KIND_FLAT:
      return run_k([&](int kq, int32_t* i, float* s, int32_t* c) {
        return search_gemm_exact(ix, dq, nq, kq, i, s, c, st);
      });
    case VX_KIND_FP16:
    case VX_KIND_SQ8:
    case VX_KIND_SQ4:
    case VX_KIND_BQ:
    case VX_KIND_BBQ:
    case VX_KIND_PQ: {
      if (!ix->rows32)
        return fail(VX_ERR_UNSUPPORTED,
                    "searchBatch on a quantized index needs the full-precision vectors at build; "
                    "use vx_scan_candidates for the compressed scores alone");
      if (oqf <= 1.0f) {
        // QuantizedFlatScanAdapter.java:67-69: delegate to the exact flat scan.
        vx_index* view = flat_view(ix);
        return run_k([&](int kq, int32_t* i, float* s, int32_t* c) {
          return search_gemm_exact(view, dq, nq, kq, i, s, c, st);
        });
      }
      // candidateK = min(n, max(k, ceil(k * overQueryFactor)))  (QuantizedFlatScanAdapter.java:71)
      const int64_t ck = std::min<int64_t>(
          ix->n, std::max<int64_t>(k, (int64_t)std::ceil((double)((float)k * oqf))));
      if (ix->kind == VX_KIND_FP16) {
        return run_k([&](int kq, int32_t* i, float* s, int32_t* c) {
          return search_fp16_two_pass(ix, dq, nq, (int)ck, kq, i, s, c, st);
        });
      }
      if (ix->kind == VX_KIND_PQ) {
        return run_k([&](int kq, int32_t* i, float* s, int32_t* c) {
          return search_pq_flat(ix, dq, nq, (int)ck, kq, true, i, s, c, st);
        });
      }
      return run_k([&](int kq, int32_t* i, float* s, int32_t* c) {
        return search_quantized_scan(ix, dq, nq, (int)ck, kq, true, i, s, c, st);
      });
    }
    case VX_KIND_IVFPQ: {
      // IvfPqAdapter.search (IvfPqAdapter.java:124-158)
      const int eff = sls > 0 ? sls : ix->nprobe;
      const bool two = oqf > 1.0f;
      const int probes = two ? (int)std::min<int64_t>((int64_t)std::ceil((double)((float)eff * oqf)), ix->nlist)
                             : std::min(eff, ix->nlist);
      const int rf = two ? std::max(ix->rescore, (int)std::ceil((double)((float)ix->rescore * oqf)))
                         : ix->rescore;
      return search_ivfpq(ix, dq, nq, k, probes, rf, -3.4028235e38f, d_ids, d_scores, d_counts, st);
    }
    case VX_KIND_IVFFLAT: {
      // IvfFlatAdapter.search (IvfFlatAdapter.java:102-140): the candidateK = ceil(k * oqf)
      // hits trimmed to k are the k best of the widened probe set
      const int eff = sls > 0 ? sls : ix->nprobe;
      const int probes = oqf > 1.0f ? (int)std::min<int64_t>((int64_t)std::ceil((double)((float)eff * oqf)), ix->nlist)
                                    : std::min(eff, ix->nlist);
      // the heap holds candidateK; only the EUCLIDEAN early exit depends on it
      const int cand_k = oqf > 1.0f ? (int)std::ceil((double)((float)k * oqf)) : k;
      const int heap_k = ix->metric == VX_EUCLIDEAN ? cand_k : k;
      return search_ivfflat(ix, dq, nq, k, heap_k, probes, -3.4028235e38f, d_ids, d_scores, d_counts, st, nullptr);
    }
    default:
      return fail(VX_ERR_INVALID_ARGUMENT, "unknown index kind");
  }
}

// Host-buffer wrapper: copies queries in, runs on the calling thread's stream, copies out.
template <class Fn>
int with_host_buffers(vx_index* ix, const float* queries, int nq, int dim, int k, int32_t* ids,
                      float* scores, int32_t* counts, Fn&& fn) {
  VX_CUDA(cudaSetDevice(ix->device));
  cudaStream_t st = cudaStreamPerThread;
  int rc;
  {
    Scratch S(st);
    const int qdim = ix->n > 0 ? ix->dim : dim;
    float* dq = S.alloc<float>((size_t)nq * qdim);
    int32_t* di = S.alloc<int32_t>((size_t)nq * k);
    float* ds = S.alloc<float>((size_t)nq * k);
    int32_t* dc = S.alloc<int32_t>(nq);
    VX_CUDA(cudaMemcpyAsync(dq, queries, (size_t)nq * qdim * 4, cudaMemcpyHostToDevice, st));
    rc = fn(dq, di, ds, dc, st);
    if (rc == VX_OK) {
      VX_CUDA(cudaMemcpyAsync(ids, di, (size_t)nq * k * 4, cudaMemcpyDeviceToHost, st));
      VX_CUDA(cudaMemcpyAsync(scores, ds, (size_t)nq * k * 4, cudaMemcpyDeviceToHost, st));
      VX_CUDA(cudaMemcpyAsync(counts, dc, (size_t)nq * 4, cudaMemcpyDeviceToHost, st));
    }
  }
  VX_CUDA(cudaStreamSynchronize(st));
  return rc;
}

}  // namespace
}  // namespace vx

// ======================================================================== C ABI
extern "C" {

int vx_abi_version(void) { return VX_ABI_VERSION; }

const char* vx_last_error(void) { return g_last_error.c_str(); }

int vx_debug_fail_next(int32_t status) {
  g_fail_next = status;
  return VX_OK;
}

int vx_debug_wait_timeout(int32_t device, int32_t timeout_ms) {
  return guarded([&]() -> int {
    if (timeout_ms < 1 || timeout_ms > 10000)
      return fail(VX_ERR_INVALID_ARGUMENT, "timeout_ms must be in [1, 10000]: %d", timeout_ms);
    int nsms = 0;
    if (int s = check_device(device, &nsms)) return s;
    cudaStream_t st = cudaStreamPerThread;
    Scratch S(st);
    int32_t* d_err = S.alloc<int32_t>(1);
    VX_CUDA(cudaMemsetAsync(d_err, 0, 4, st));
    VX_LAUNCH(1, launch_wait_probe((uint64_t)timeout_ms * 1000000ull, d_err, st));
    return check_device_error(d_err, st);
  });
}

int vx_kernel_launches(int64_t* count) {
  if (!count) return fail(VX_ERR_NULL_POINTER, "count must not be null");
  *count = g_launches.load();
  return VX_OK;
}

int vx_profile_enable(int32_t on) {
  g_prof_on.store(on != 0);
  return VX_OK;
}

int vx_profile_read(int32_t slot, double* total_ms, int64_t* launches) {
  if (slot < 0 || slot >= VX_PROF_SLOTS) return fail(VX_ERR_INVALID_ARGUMENT, "bad profile slot %d", slot);
  std::vector<ProfRec> recs;
  {
    std::lock_guard<std::mutex> g(g_prof_mu);
    recs.swap(g_prof);
  }
  for (auto& r : recs) {
    float ms = 0.0f;
    if (cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess) {
      g_prof_ms[r.slot] += ms;
      g_prof_n[r.slot] += 1;
    }
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  if (total_ms) *total_ms = g_prof_ms[slot];
  if (launches) *launches = g_prof_n[slot];
  return VX_OK;
}

int vx_profile_reset(void) {
  int64_t dummy;
  vx_profile_read(0, nullptr, &dummy);
  for (int i = 0; i < VX_PROF_SLOTS; i++) {
    g_prof_ms[i] = 0;
    g_prof_n[i] = 0;
  }
  return VX_OK;
}

int vx_device_count(int32_t* count) {
  return guarded([&]() -> int {
    if (!count) return fail(VX_ERR_NULL_POINTER, "count must not be null");
    int c = 0;
    cudaError_t e = cudaGetDeviceCount(&c);
    *count = (e == cudaSuccess) ? c : 0;
    return VX_OK;
  });
}

int vx_flat_build(int32_t device, const float* vectors, int64_t n, int32_t dim, int64_t row_stride,
                  int32_t metric, vx_index** out) {
  return guarded([&]() -> int {
    if (!out) return fail(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    if (n > 0 && !vectors) return fail(VX_ERR_NULL_POINTER, "vectors must not be null");
    if (n < 0 || n > INT32_MAX) return fail(VX_ERR_INVALID_ARGUMENT, "bad vector count %lld", (long long)n);
    if (n > 0 && (dim <= 0 || row_stride < dim))
      return fail(VX_ERR_INVALID_ARGUMENT, "bad dimension %d / stride %lld", dim, (long long)row_stride);
    if (int s = check_metric(metric)) return s;
    int nsms = 0;
    if (int s = check_device(device, &nsms)) return s;
    vx_index* ix = new vx_index();
    ix->kind = VX_KIND_FLAT;
    ix->device = device;
    ix->metric = metric;
    ix->n = n;
    ix->dim = n > 0 ? dim : 0;
    ix->num_sms = nsms;
    try {
      if (n > 0) {
        ix->rows32 = upload_rows32(ix, vectors, n, dim, row_stride);
        build_unit_f16(ix);
      }
    } catch (...) {
      free_index(ix);
      throw;
    }
    *out = ix;
    return VX_OK;
  });
}

int vx_fp16_build(int32_t device, const uint16_t* codes, int64_t n, int32_t dim, int32_t metric,
                  const float* vectors, int64_t row_stride, vx_index** out) {
  return guarded([&]() -> int {
    if (!out) return fail(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    if (n > 0 && !codes) return fail(VX_ERR_NULL_POINTER, "codes must not be null");
    if (n < 0 || n > INT32_MAX) return fail(VX_ERR_INVALID_ARGUMENT, "bad vector count");
    if (n > 0 && dim <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "bad dimension %d", dim);
    if (vectors && row_stride < dim) return fail(VX_ERR_INVALID_ARGUMENT, "bad row stride");
    if (int s = check_metric(metric)) return s;
    int nsms = 0;
    if (int s = check_device(device, &nsms)) return s;
    vx_index* ix = new vx_index();
    ix->kind = VX_KIND_FP16;
    ix->device = device;
    ix->metric = metric;
    ix->n = n;
    ix->dim = n > 0 ? dim : 0;
    ix->num_sms = nsms;
    try {
      if (n > 0) {
        ix->Dp = (int)round_up(dim, 64);
        DevTemp<__half> raw_buf((size_t)n * dim);
        __half* raw = raw_buf.p;
        VX_CUDA(cudaMemcpy(raw, codes, (size_t)n * dim * 2, cudaMemcpyDefault));
        ix->rows16 = dev_alloc<__half>(ix, (size_t)n * ix->Dp);
        ix->rowsq = dev_alloc<float>(ix, (size_t)n);
        ix->rowscale = dev_alloc<float>(ix, (size_t)n);
        ix->max_norm = dev_alloc<float>(ix, 1);
        VX_CUDA(cudaMemset(ix->max_norm, 0, 4));
        std::vector<float> ones((size_t)n, 1.0f);
        VX_CUDA(cudaMemcpy(ix->rowscale, ones.data(), (size_t)n * 4, cudaMemcpyDefault));
        VX_LAUNCH(1, launch_f16_rows_pad(raw, n, dim, ix->Dp, ix->rows16, ix->rowsq, ix->max_norm, 0));
        VX_CUDA(cudaDeviceSynchronize());
        make_tmap(&ix->tm_rows, ix->rows16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ix->Dp, n,
                 gemm_scan_db_box(gemm_two_sm()));
        ix->has_tm_rows = true;
        if (vectors) ix->rows32 = upload_rows32(ix, vectors, n, dim, row_stride);
      }
    } catch (...) {
      free_index(ix);
      throw;
    }
    *out = ix;
    return VX_OK;
  });
}

int vx_sq8_build(int32_t device, const int8_t* codes, const float* corrections, int64_t n,
                 int32_t dim, float min_quantile, float max_quantile, int32_t metric,
                 const float* vectors, int64_t row_stride, vx_index** out) {
  return vx::sq_build(device, codes, corrections, n, dim, min_quantile, max_quantile, 127, metric, vectors,
                      row_stride, out);
}

int vx_sq4_build(int32_t device, const uint8_t* packed, const float* corrections, int64_t n, int32_t dim,
                 float min_quantile, float max_quantile, int32_t metric, const float* vectors, int64_t row_stride,
                 vx_index** out) {
  return guarded([&]() -> int {
    if (!out) return fail(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    if (n > 0 && (!packed || !corrections)) return fail(VX_ERR_NULL_POINTER, "codes/corrections must not be null");
    if (n < 0 || n > INT32_MAX) return fail(VX_ERR_INVALID_ARGUMENT, "bad vector count");
    if (n > 0 && dim <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "bad dimension %d", dim);
    // unpackInt4 (ScalarQuantizer.java:330-336): low nibble = even dimension, high = odd
    const size_t nb = ((size_t)dim + 1) / 2;
    std::vector<uint8_t> host_packed;
    const uint8_t* src = packed;
    if (n > 0) {
      cudaPointerAttributes attr{};
      if (cudaPointerGetAttributes(&attr, packed) == cudaSuccess && attr.type == cudaMemoryTypeDevice) {
        host_packed.resize((size_t)n * nb);
        VX_CUDA(cudaMemcpy(host_packed.data(), packed, host_packed.size(), cudaMemcpyDeviceToHost));
        src = host_packed.data();
      }
      cudaGetLastError();
    }
    std::vector<int8_t> codes((size_t)std::max<int64_t>(n, 0) * (size_t)std::max(dim, 0));
    for (int64_t r = 0; r < n; r++)
      for (int i = 0; i < dim; i++) {
        const uint8_t b = src[(size_t)r * nb + (i >> 1)];
        codes[(size_t)r * dim + i] = (int8_t)((i & 1) ? (b >> 4) & 0x0F : b & 0x0F);
      }
    return vx::sq_build(device, codes.data(), corrections, n, dim, min_quantile, max_quantile, 15, metric,
                        vectors, row_stride, out);
  });
}

}  // extern "C"

namespace vx {
// ScalarQuantizedVectors with codes one per byte, maxValue 127 (SQ8) or 15 (SQ4 unpacked).
int sq_build(int32_t device, const int8_t* codes, const float* corrections, int64_t n, int32_t dim,
             float min_quantile, float max_quantile, int max_value, int32_t metric, const float* vectors,
             int64_t row_stride, vx_index** out) {
  return guarded([&]() -> int {
    if (!out) return fail(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    if (n > 0 && (!codes || !corrections)) return fail(VX_ERR_NULL_POINTER, "codes/corrections must not be null");
    if (n < 0 || n > INT32_MAX) return fail(VX_ERR_INVALID_ARGUMENT, "bad vector count");
    if (n > 0 && dim <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "bad dimension %d", dim);
    if (!(min_quantile < max_quantile))
      return fail(VX_ERR_INVALID_ARGUMENT, "minQuantile must be < maxQuantile: %g >= %g",
                  (double)min_quantile, (double)max_quantile);
    if (vectors && row_stride < dim) return fail(VX_ERR_INVALID_ARGUMENT, "bad row stride");
    if (int s = check_metric(metric)) return s;
    int nsms = 0;
    if (int s = check_device(device, &nsms)) return s;
    vx_index* ix = new vx_index();
    ix->kind = max_value == 15 ? VX_KIND_SQ4 : VX_KIND_SQ8;
    ix->sq_max = max_value;
    ix->device = device;
    ix->metric = metric;
    ix->n = n;
    ix->dim = n > 0 ? dim : 0;
    ix->num_sms = nsms;
    ix->min_q = min_quantile;
    ix->max_q = max_quantile;
    try {
      if (n > 0) {
        ix->Dp8 = (int)round_up(dim, 128);
        DevTemp<int8_t> raw_buf((size_t)n * dim);
        int8_t* raw = raw_buf.p;
        VX_CUDA(cudaMemcpy(raw, codes, (size_t)n * dim, cudaMemcpyDefault));
        ix->codes8 = dev_alloc<int8_t>(ix, (size_t)n * ix->Dp8);
        ix->vsq = dev_alloc<int32_t>(ix, (size_t)n);
        ix->vcorr = dev_alloc<float>(ix, (size_t)n);
        VX_CUDA(cudaMemcpy(ix->vcorr, corrections, (size_t)n * 4, cudaMemcpyDefault));
        VX_LAUNCH(1, launch_sq8_rows_pad(raw, n, dim, ix->Dp8, ix->codes8, ix->vsq, 0));
        VX_CUDA(cudaDeviceSynchronize());
        make_tmap(&ix->tm_codes8, ix->codes8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ix->Dp8, n,
                 gemm_scan_db_box(gemm_two_sm()));
        if (vectors) ix->rows32 = upload_rows32(ix, vectors, n, dim, row_stride);
      }
    } catch (...) {
      free_index(ix);
      throw;
    }
    *out = ix;
    return VX_OK;
  });
}
}  // namespace vx

extern "C" {

int vx_bbq_build(int32_t device, const uint64_t* words, const float* corrections, const float* centroid, int64_t n,
                 int32_t dim, int32_t metric, const float* vectors, int64_t row_stride, vx_index** out) {
  return guarded([&]() -> int {
    if (!out) return fail(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    if (!centroid) return fail(VX_ERR_NULL_POINTER, "centroid must not be null");
    if (n > 0 && (!words || !corrections)) return fail(VX_ERR_NULL_POINTER, "words/corrections must not be null");
    if (n < 0 || n > INT32_MAX) return fail(VX_ERR_INVALID_ARGUMENT, "bad vector count");
    if (dim <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "bad dimension %d", dim);
    const int nw = (dim + 63) / 64;
    const int nwp = bq_padded_words(nw);
    if (nwp < 0) return fail(VX_ERR_UNSUPPORTED, "BBQ dimension %d exceeds 2048", dim);
    // above 1024 dimensions only the int8 tensor operand serves BBQ (the popcount kernel keeps a
    // query's four bit planes in registers, up to 16 words each): whole, or in row windows
    if (!bbq_supported(nwp) && n > 0 && bq_tensor_budget() < (uint64_t)n * (uint64_t)round_up(dim, 128) &&
        bq_window_bytes() == 0)
      return fail(VX_ERR_UNSUPPORTED,
                  "BBQ above 1024 dimensions is scanned on the int8 tensor operand, which exceeds "
                  "VX_BQ_TENSOR_BYTES here (%lld rows x %d dims) with row windows off (VX_BQ_WINDOW_BYTES=0)",
                  (long long)n, dim);
    if (vectors && row_stride < dim) return fail(VX_ERR_INVALID_ARGUMENT, "bad row stride");
    if (int s = check_metric(metric)) return s;
    int nsms = 0;
    if (int s = check_device(device, &nsms)) return s;
    vx_index* ix = new vx_index();
    ix->kind = VX_KIND_BBQ;
    ix->device = device;
    ix->metric = metric;
    ix->n = n;
    ix->dim = dim;
    ix->num_sms = nsms;
    ix->nw_pad = nwp;
    try {
      ix->bbq_centroid = dev_alloc<float>(ix, (size_t)dim);
      VX_CUDA(cudaMemcpy(ix->bbq_centroid, centroid, (size_t)dim * 4, cudaMemcpyDefault));
      if (n > 0) {
        ix->words = dev_alloc<uint64_t>(ix, (size_t)n * nwp);
        VX_CUDA(cudaMemset(ix->words, 0, (size_t)n * nwp * 8));
        VX_CUDA(cudaMemcpy2D(ix->words, (size_t)nwp * 8, words, (size_t)nw * 8, (size_t)nw * 8, (size_t)n,
                             cudaMemcpyDefault));
        DevTemp<float> corr((size_t)n * 3);
        VX_CUDA(cudaMemcpy(corr.p, corrections, (size_t)n * 12, cudaMemcpyDefault));
        ix->bbq_rows = dev_alloc<float4>(ix, (size_t)n);
        VX_LAUNCH(1, launch_bbq_rowinfo(ix->words, nw, nwp, corr.p, n, ix->bbq_rows, 0));
        VX_CUDA(cudaDeviceSynchronize());
        // 0/1 int8 operand and epilogue records for the tensor-core scan (8 bytes per bit)
        const int Dp8 = (int)round_up(dim, 128);
        const bool whole = bq_tensor_budget() >= (uint64_t)n * Dp8;
        if (whole || bq_window_bytes() > 0) {
          // the epilogue records always; the operand itself whole, or per row window at search time
          ix->Dp8 = Dp8;
          ix->bbq_epi = dev_alloc<float4>(ix, (size_t)n);
          VX_LAUNCH(1, launch_bbq_epi_rows(ix->bbq_rows, n, dim, metric, ix->bbq_epi, 0));
          if (whole) {
            ix->codes8 = dev_alloc<int8_t>(ix, (size_t)n * Dp8);
            VX_LAUNCH(1, launch_bq_words_to_i8(ix->words, n, nwp, dim, Dp8, ix->codes8, 0, true));
            make_tmap(&ix->tm_codes8, ix->codes8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Dp8, n,
                      gemm_scan_db_box(gemm_two_sm()));
          } else {
            ix->bq_windows = true;
          }
          VX_CUDA(cudaDeviceSynchronize());
        }
        if (vectors) ix->rows32 = upload_rows32(ix, vectors, n, dim, row_stride);
      }
    } catch (...) {
      free_index(ix);
      throw;
    }
    *out = ix;
    return VX_OK;
  });
}

int vx_bq_build(int32_t device, const uint64_t* words, int64_t n, int32_t dim, int32_t metric,
                const float* vectors, int64_t row_stride, vx_index** out) {
  return guarded([&]() -> int {
    if (!out) return fail(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    if (n > 0 && !words) return fail(VX_ERR_NULL_POINTER, "words must not be null");
    if (n < 0 || n > INT32_MAX) return fail(VX_ERR_INVALID_ARGUMENT, "bad vector count");
    if (n > 0 && dim <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "bad dimension %d", dim);
    const int nw = (dim + 63) / 64;
    const int nwp = bq_padded_words(nw);
    if (n > 0 && nwp < 0) return fail(VX_ERR_UNSUPPORTED, "dimension %d exceeds 2048 bits", dim);
    if (vectors && row_stride < dim) return fail(VX_ERR_INVALID_ARGUMENT, "bad row stride");
    if (int s = check_metric(metric)) return s;
    int nsms = 0;
    if (int s = check_device(device, &nsms)) return s;
    vx_index* ix = new vx_index();
    ix->kind = VX_KIND_BQ;
    ix->device = device;
    ix->metric = metric;
    ix->n = n;
    ix->dim = n > 0 ? dim : 0;
    ix->num_sms = nsms;
    ix->nw_pad = nwp;
    try {
      if (n > 0) {
        ix->words = dev_alloc<uint64_t>(ix, (size_t)n * nwp);
        VX_CUDA(cudaMemset(ix->words, 0, (size_t)n * nwp * 8));
        VX_CUDA(cudaMemcpy2D(ix->words, (size_t)nwp * 8, words, (size_t)nw * 8, (size_t)nw * 8, (size_t)n,
                             cudaMemcpyDefault));
        // +-1 int8 operand for the tensor-core Hamming scan (8 bytes per bit of storage): whole
        // within VX_BQ_TENSOR_BYTES, else expanded per row window at search time
        const int Dp8 = (int)round_up(dim, 128);
        if (bq_tensor_budget() >= (uint64_t)n * Dp8) {
          ix->Dp8 = Dp8;
          ix->codes8 = dev_alloc<int8_t>(ix, (size_t)n * Dp8);
          VX_LAUNCH(1, launch_bq_words_to_i8(ix->words, n, nwp, dim, Dp8, ix->codes8, 0));
          VX_CUDA(cudaDeviceSynchronize());
          make_tmap(&ix->tm_codes8, ix->codes8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, Dp8, n,
                    gemm_scan_db_box(gemm_two_sm()));
        } else if (bq_window_bytes() > 0) {
          ix->Dp8 = Dp8;
          ix->bq_windows = true;
        }
        if (vectors) ix->rows32 = upload_rows32(ix, vectors, n, dim, row_stride);
      }
    } catch (...) {
      free_index(ix);
      throw;
    }
    // The no-allocation BQ scan's static scratch is placed on this device here, at build time,
    // so that vx_bq_scan_candidates_noalloc never loads a module (and with it 64 MiB) itself.
    noalloc_prepare(device);
    *out = ix;
    return VX_OK;
  });
}

int vx_ivfpq_build(int32_t device, const float* centroids, int32_t nlist, int32_t dim,
                   const int64_t* list_offsets, const int32_t* list_ordinals, int32_t m, int32_t ks,
                   const float* codebooks, const uint8_t* codes, int64_t n, int32_t metric,
                   const float* vectors, int32_t nprobe, int32_t rescore_factor, vx_index** out) {
  return vx::ivfpq_build_strided(device, centroids, nlist, dim, list_offsets, list_ordinals, m, ks, codebooks,
                                 codes, n, metric, vectors, dim, nprobe, rescore_factor, out);
}

int vx_pq_build(int32_t device, const float* codebooks, const float* global_centroid, const uint8_t* codes, int64_t n,
                int32_t dim, int32_t m, int32_t ks, int32_t metric, const float* vectors, int64_t row_stride,
                vx_index** out) {
  return guarded([&]() -> int {
    if (!out) return fail(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    if (!codebooks) return fail(VX_ERR_NULL_POINTER, "codebooks must not be null");
    if (n > 0 && !codes) return fail(VX_ERR_NULL_POINTER, "codes must not be null");
    if (n < 0 || n > INT32_MAX || dim <= 0)
      return fail(VX_ERR_INVALID_ARGUMENT, "bad PQ shape n=%lld dim=%d", (long long)n, dim);
    if (vectors && row_stride < dim)
      return fail(VX_ERR_INVALID_ARGUMENT, "row_stride %lld < dimension %d", (long long)row_stride, dim);
    // one list holding every row in ordinal order; the list's "centroid" is the global
    // centroid (or zeros), which the flat-PQ tables subtract from every query
    std::vector<float> cent((size_t)dim, 0.0f);
    if (global_centroid) VX_CUDA(cudaMemcpy(cent.data(), global_centroid, (size_t)dim * 4, cudaMemcpyDefault));
    const int64_t offs[2] = {0, n};
    std::vector<int32_t> ords((size_t)std::max<int64_t>(n, 1));
    for (int64_t i = 0; i < n; i++) ords[(size_t)i] = (int32_t)i;
    vx_index* ix = nullptr;
    int st = vx::ivfpq_build_strided(device, cent.data(), 1, dim, offs, ords.data(), m, ks, codebooks, codes, n,
                                     metric, vectors, vectors ? row_stride : dim, 1, 1, &ix);
    if (st != VX_OK) return st;
    ix->kind = VX_KIND_PQ;
    try {
      if (metric == VX_COSINE && n > 0) {
        ix->pq_rnorm = dev_alloc<float>(ix, (size_t)n);
        DevTemp<float> cnorm((size_t)m * ks);
        VX_LAUNCH(2, launch_pq_row_norms(ix->pq_codes, n, ix->M, ix->Mp, ix->Ks, ix->sub, ix->codebooks, ix->cb_off,
                                         cnorm.p, ix->pq_rnorm, 0));
        VX_CUDA(cudaDeviceSynchronize());
      }
    } catch (...) {
      free_index(ix);
      throw;
    }
    *out = ix;
    return VX_OK;
  });
}

}  // extern "C"

namespace vx {
// vx_ivfpq_build with full-precision rows `row_stride` floats apart (a vectors.bin mapping).
int ivfpq_build_strided(int32_t device, const float* centroids, int32_t nlist, int32_t dim,
                        const int64_t* list_offsets, const int32_t* list_ordinals, int32_t m, int32_t ks,
                        const float* codebooks, const uint8_t* codes, int64_t n, int32_t metric,
                        const float* vectors, int64_t row_stride, int32_t nprobe, int32_t rescore_factor,
                        vx_index** out) {
  return guarded([&]() -> int {
    if (!out) return fail(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    if (!centroids || !list_offsets || !codebooks) return fail(VX_ERR_NULL_POINTER, "null IVF-PQ component");
    if (n > 0 && (!list_ordinals || !codes)) return fail(VX_ERR_NULL_POINTER, "null IVF-PQ component");
    if (nlist <= 0 || dim <= 0 || n < 0 || n > INT32_MAX)
      return fail(VX_ERR_INVALID_ARGUMENT, "bad IVF shape nlist=%d dim=%d n=%lld", nlist, dim, (long long)n);
    if (m <= 0 || m > dim) return fail(VX_ERR_INVALID_ARGUMENT, "numSubspaces must be in [1, dim]: %d", m);
    if (ks <= 0 || ks > 256) return fail(VX_ERR_INVALID_ARGUMENT, "numClusters must be in [1, 256]: %d", ks);
    if (nprobe <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "nprobe must be positive: %d", nprobe);
    if (rescore_factor < 1) return fail(VX_ERR_INVALID_ARGUMENT, "rescoreFactor must be >= 1: %d", rescore_factor);
    if (vectors && row_stride < dim)
      return fail(VX_ERR_INVALID_ARGUMENT, "row_stride %lld < dimension %d", (long long)row_stride, dim);
    if (int s = check_metric(metric)) return s;
    // The lists may hold a subset of the n coded rows (a list-sharded index keeps only its
    // own lists): offsets run from 0 to nl <= n, ordinals index the codes.
    const int64_t nl = list_offsets[nlist];
    if (list_offsets[0] != 0 || nl < 0 || nl > n)
      return fail(VX_ERR_INVALID_ARGUMENT, "list offsets must run from 0 to at most n");
    for (int l = 0; l < nlist; l++)
      if (list_offsets[l + 1] < list_offsets[l]) return fail(VX_ERR_INVALID_ARGUMENT, "list offsets must be non-decreasing");
    if (nl > 0 && !list_ordinals) return fail(VX_ERR_NULL_POINTER, "null IVF-PQ component");
    for (int64_t i = 0; i < nl; i++)
      if (list_ordinals[i] < 0 || list_ordinals[i] >= n)
        return fail(VX_ERR_INVALID_ARGUMENT, "list ordinal %d out of range", list_ordinals[i]);
    int nsms = 0;
    if (int s = check_device(device, &nsms)) return s;
    vx_index* ix = new vx_index();
    ix->kind = VX_KIND_IVFPQ;
    ix->device = device;
    ix->metric = metric;
    ix->n = n;
    ix->dim = dim;
    ix->num_sms = nsms;
    ix->nlist = nlist;
    ix->M = m;
    ix->Ks = ks;
    ix->Mp = (int)round_up(m, 16);
    ix->nprobe = nprobe;
    ix->rescore = rescore_factor;
    try {
      ix->cent = dev_alloc<float>(ix, (size_t)nlist * dim);
      VX_CUDA(cudaMemcpy(ix->cent, centroids, (size_t)nlist * dim * 4, cudaMemcpyDefault));
      ix->list_off = dev_alloc<int64_t>(ix, (size_t)nlist + 1);
      VX_CUDA(cudaMemcpy(ix->list_off, list_offsets, (size_t)(nlist + 1) * 8, cudaMemcpyDefault));
      ix->list_order = upload_list_order(ix, list_offsets, nlist);
      // subspaces (ProductQuantizer.computeSubspaceSizesAndOffsets, ProductQuantizer.java:686-700)
      std::vector<int32_t> sub(2 * (size_t)m);
      std::vector<int64_t> cboff(m);
      int base = dim / m, rem = dim % m, off = 0;
      int64_t co = 0;
      for (int i = 0; i < m; i++) {
        int size = base + (i < rem ? 1 : 0);
        sub[2 * i] = size;
        sub[2 * i + 1] = off;
        cboff[i] = co;
        off += size;
        co += (int64_t)ks * size;
      }
      ix->sub = dev_alloc<int32_t>(ix, sub.size());
      VX_CUDA(cudaMemcpy(ix->sub, sub.data(), sub.size() * 4, cudaMemcpyDefault));
      ix->cb_off = dev_alloc<int64_t>(ix, cboff.size());
      VX_CUDA(cudaMemcpy(ix->cb_off, cboff.data(), cboff.size() * 8, cudaMemcpyDefault));
      ix->codebooks = dev_alloc<float>(ix, (size_t)co);
      VX_CUDA(cudaMemcpy(ix->codebooks, codebooks, (size_t)co * 4, cudaMemcpyDefault));
      // codes regrouped list-contiguous, rows padded to Mp bytes
      ix->ordinals = dev_alloc<int32_t>(ix, (size_t)std::max<int64_t>(nl, 1));
      ix->pq_codes = dev_alloc<uint8_t>(ix, (size_t)std::max<int64_t>(nl, 1) * ix->Mp);
      if (nl > 0) {
        VX_CUDA(cudaMemcpy(ix->ordinals, list_ordinals, (size_t)nl * 4, cudaMemcpyDefault));
        std::vector<uint8_t> grouped((size_t)nl * ix->Mp, 0);
        for (int64_t i = 0; i < nl; i++)
          std::memcpy(&grouped[(size_t)i * ix->Mp], codes + (size_t)list_ordinals[i] * m, (size_t)m);
        VX_CUDA(cudaMemcpy(ix->pq_codes, grouped.data(), grouped.size(), cudaMemcpyDefault));
      }
      if (vectors && n > 0) ix->rows32 = upload_rows32(ix, vectors, n, dim, row_stride);
    } catch (...) {
      free_index(ix);
      throw;
    }
    *out = ix;
    return VX_OK;
  });
}
}  // namespace vx

extern "C" {

int vx_ivfflat_build(int32_t device, const float* centroids, int32_t nlist, int32_t dim, const int64_t* list_offsets,
                     const int32_t* list_ordinals, const float* vectors, int64_t n, int64_t row_stride, int32_t metric,
                     int32_t nprobe, vx_index** out) {
  return guarded([&]() -> int {
    if (!out) return fail(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    if (!centroids || !list_offsets) return fail(VX_ERR_NULL_POINTER, "null IVF component");
    if (n > 0 && (!list_ordinals || !vectors)) return fail(VX_ERR_NULL_POINTER, "null IVF component");
    if (nlist <= 0 || dim <= 0 || n < 0 || n > INT32_MAX)
      return fail(VX_ERR_INVALID_ARGUMENT, "bad IVF shape nlist=%d dim=%d n=%lld", nlist, dim, (long long)n);
    if (vectors && row_stride < dim)
      return fail(VX_ERR_INVALID_ARGUMENT, "row_stride %lld < dimension %d", (long long)row_stride, dim);
    if (nprobe <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "nprobe must be positive: %d", nprobe);
    if (int s = check_metric(metric)) return s;
    const int64_t nl = list_offsets[nlist];
    if (list_offsets[0] != 0 || nl < 0 || nl > n)
      return fail(VX_ERR_INVALID_ARGUMENT, "list offsets must run from 0 to at most n");
    for (int l = 0; l < nlist; l++)
      if (list_offsets[l + 1] < list_offsets[l]) return fail(VX_ERR_INVALID_ARGUMENT, "list offsets must be non-decreasing");
    for (int64_t i = 0; i < nl; i++)
      if (list_ordinals[i] < 0 || list_ordinals[i] >= n)
        return fail(VX_ERR_INVALID_ARGUMENT, "list ordinal %d out of range", list_ordinals[i]);
    int nsms = 0;
    if (int s = check_device(device, &nsms)) return s;
    vx_index* ix = new vx_index();
    ix->kind = VX_KIND_IVFFLAT;
    ix->device = device;
    ix->metric = metric;
    ix->n = n;
    ix->dim = dim;
    ix->num_sms = nsms;
    ix->nlist = nlist;
    ix->nprobe = nprobe;
    ix->Dp_flat = (int)round_up(dim, 4);
    try {
      ix->cent = dev_alloc<float>(ix, (size_t)nlist * dim);
      VX_CUDA(cudaMemcpy(ix->cent, centroids, (size_t)nlist * dim * 4, cudaMemcpyDefault));
      ix->list_off = dev_alloc<int64_t>(ix, (size_t)nlist + 1);
      VX_CUDA(cudaMemcpy(ix->list_off, list_offsets, (size_t)(nlist + 1) * 8, cudaMemcpyDefault));
      ix->list_order = upload_list_order(ix, list_offsets, nlist);
      ix->ordinals = dev_alloc<int32_t>(ix, (size_t)std::max<int64_t>(nl, 1));
      ix->flat_rows = dev_alloc<float>(ix, (size_t)std::max<int64_t>(nl, 1) * ix->Dp_flat);
      if (metric == VX_COSINE) ix->flat_norms = dev_alloc<float>(ix, (size_t)std::max<int64_t>(nl, 1));
      if (nl > 0) {
        VX_CUDA(cudaMemcpy(ix->ordinals, list_ordinals, (size_t)nl * 4, cudaMemcpyDefault));
        // the rows as dense [n][dim] on the device, then gathered into list order, padded
        DevTemp<float> dense((size_t)n * dim);
        VX_CUDA(cudaMemcpy2D(dense.p, (size_t)dim * 4, vectors, (size_t)row_stride * 4, (size_t)dim * 4, (size_t)n,
                             cudaMemcpyDefault));
        VX_LAUNCH(1, launch_pad_rows(dense.p, nl, dim, dim, ix->ordinals, ix->Dp_flat, ix->flat_rows, 0));
        VX_CUDA(cudaDeviceSynchronize());
        if (ix->flat_norms) VX_LAUNCH(1, launch_row_norms(ix->flat_rows, nl, dim, ix->Dp_flat, ix->flat_norms, 0));
        VX_CUDA(cudaDeviceSynchronize());
      }
      // BuoyIndex.computeRadii over the partitions (vx_ivf_set_buoy replaces them with a
      // prebuilt BuoyIndex's own)
      ix->radii = dev_alloc<float>(ix, (size_t)nlist);
      VX_LAUNCH(1, launch_list_radii(ix->flat_rows, nl, dim, ix->Dp_flat, ix->list_off, nlist, ix->cent, ix->radii, 0));
      VX_CUDA(cudaDeviceSynchronize());
    } catch (...) {
      free_index(ix);
      throw;
    }
    *out = ix;
    return VX_OK;
  });
}

int vx_ivf_set_buoy(vx_index* ix, const float* radii, const int32_t* spill_targets) {
  return guarded([&]() -> int {
    if (!ix) return fail(VX_ERR_NULL_POINTER, "index must not be null");
    if (ix->kind != VX_KIND_IVFPQ && ix->kind != VX_KIND_IVFFLAT)
      return fail(VX_ERR_UNSUPPORTED, "not an IVF index");
    VX_CUDA(cudaSetDevice(ix->device));
    if (radii) {
      if (!ix->radii) ix->radii = dev_alloc<float>(ix, (size_t)ix->nlist);
      VX_CUDA(cudaMemcpy(ix->radii, radii, (size_t)ix->nlist * 4, cudaMemcpyDefault));
    }
    if (spill_targets) {
      if (!ix->spill) ix->spill = dev_alloc<int32_t>(ix, (size_t)ix->nlist);
      VX_CUDA(cudaMemcpy(ix->spill, spill_targets, (size_t)ix->nlist * 4, cudaMemcpyDefault));
    }
    return VX_OK;
  });
}

int vx_ivf_set_key_dims(vx_index* ix, const int32_t* key_dim_counts) {
  return guarded([&]() -> int {
    if (!ix) return fail(VX_ERR_NULL_POINTER, "index must not be null");
    if (ix->kind != VX_KIND_IVFFLAT) return fail(VX_ERR_UNSUPPORTED, "not an IVF-flat index");
    VX_CUDA(cudaSetDevice(ix->device));
    bool any = false;
    std::vector<uint8_t> flags((size_t)ix->nlist, 0);
    if (key_dim_counts)
      for (int l = 0; l < ix->nlist; l++) {
        if (key_dim_counts[l] < 0) return fail(VX_ERR_INVALID_ARGUMENT, "negative key dimension count for list %d", l);
        flags[(size_t)l] = key_dim_counts[l] > 0;
        any |= key_dim_counts[l] > 0;
      }
    if (!any) {
      ix->keyed = nullptr;  // the array (if any) stays owned by the index until it is freed
      return VX_OK;
    }
    uint8_t* d = dev_alloc<uint8_t>(ix, (size_t)ix->nlist);
    VX_CUDA(cudaMemcpy(d, flags.data(), (size_t)ix->nlist, cudaMemcpyHostToDevice));
    ix->keyed = d;
    return VX_OK;
  });
}

int vx_ivf_set_gamma(vx_index* ix, float gamma) {
  return guarded([&]() -> int {
    if (!ix) return fail(VX_ERR_NULL_POINTER, "index must not be null");
    if (ix->kind != VX_KIND_IVFPQ && ix->kind != VX_KIND_IVFFLAT)
      return fail(VX_ERR_UNSUPPORTED, "not an IVF index");
    if (!(gamma >= 0.0f)) return fail(VX_ERR_INVALID_ARGUMENT, "gamma must be >= 0, got %g", (double)gamma);
    ix->gamma = gamma;
    return VX_OK;
  });
}

int vx_index_info(const vx_index* ix, int32_t* kind, int64_t* size, int32_t* dim, int32_t* metric) {
  if (!ix) return fail(VX_ERR_NULL_POINTER, "index must not be null");
  if (kind) *kind = ix->kind;
  if (size) *size = ix->n;
  if (dim) *dim = ix->dim;
  if (metric) *metric = ix->metric;
  return VX_OK;
}

int vx_index_free(vx_index* ix) {
  return guarded([&]() -> int {
    free_index(ix);
    return VX_OK;
  });
}

int vx_search_batch_device(vx_index* ix, const float* d_queries, int32_t nq, int32_t dim, int32_t k,
                           int32_t sls, float oqf, int32_t* d_ids, float* d_scores,
                           int32_t* d_counts, void* stream) {
  return guarded([&]() -> int {
    if (int s = validate_search(ix, d_queries, nq, dim, k, d_ids, d_scores, d_counts)) return s;
    VX_CUDA(cudaSetDevice(ix->device));
    return search_batch_dev(ix, d_queries, nq, dim, k, sls, oqf, d_ids, d_scores, d_counts,
                            (cudaStream_t)stream);
  });
}

int vx_search_batch(vx_index* ix, const float* queries, int32_t nq, int32_t dim, int32_t k,
                    int32_t sls, float oqf, int32_t* ids, float* scores, int32_t* counts) {
  return guarded([&]() -> int {
    if (int s = validate_search(ix, queries, nq, dim, k, ids, scores, counts)) return s;
    return with_host_buffers(ix, queries, nq, dim, k, ids, scores, counts,
                             [&](float* dq, int32_t* di, float* ds, int32_t* dc, cudaStream_t st) {
                               return search_batch_dev(ix, dq, nq, dim, k, sls, oqf, di, ds, dc, st);
                             });
  });
}

static int scan_candidates_dev(vx_index* ix, const float* dq, int nq, int dim, int k, int32_t* di,
                               float* ds, int32_t* dc, cudaStream_t st) {
  if (ix->kind != VX_KIND_SQ8 && ix->kind != VX_KIND_SQ4 && ix->kind != VX_KIND_BQ && ix->kind != VX_KIND_BBQ &&
      ix->kind != VX_KIND_FP16 && ix->kind != VX_KIND_PQ)
    return fail(VX_ERR_UNSUPPORTED, "candidate scans apply to SQ8, SQ4, BQ, BBQ, FP16 and PQ indexes");
  if (ix->n == 0) {
    fill_empty(nq, k, di, ds, dc, st);
    return VX_OK;
  }
  const int kk = (int)std::min<int64_t>(k, ix->n);
  if (kk < k) fill_empty(nq, k, di, ds, dc, st);
  Scratch S(st);
  int32_t* ti = di;
  float* ts = ds;
  if (kk < k) {
    ti = S.alloc<int32_t>((size_t)nq * kk);
    ts = S.alloc<float>((size_t)nq * kk);
  }
  int rc = (ix->kind == VX_KIND_FP16) ? search_gemm_exact(ix, dq, nq, kk, ti, ts, dc, st)
           : (ix->kind == VX_KIND_PQ) ? search_pq_flat(ix, dq, nq, kk, kk, false, ti, ts, dc, st)
                                      : search_quantized_scan(ix, dq, nq, kk, kk, false, ti, ts, dc, st);
  if (rc != VX_OK) return rc;
  if (kk < k) {
    VX_CUDA(cudaMemcpy2DAsync(di, (size_t)k * 4, ti, (size_t)kk * 4, (size_t)kk * 4, nq,
                              cudaMemcpyDeviceToDevice, st));
    VX_CUDA(cudaMemcpy2DAsync(ds, (size_t)k * 4, ts, (size_t)kk * 4, (size_t)kk * 4, nq,
                              cudaMemcpyDeviceToDevice, st));
  }
  return VX_OK;
}

int vx_scan_candidates_device(vx_index* ix, const float* d_queries, int32_t nq, int32_t dim,
                              int32_t k, int32_t* d_ids, float* d_scores, int32_t* d_counts,
                              void* stream) {
  return guarded([&]() -> int {
    if (int s = validate_search(ix, d_queries, nq, dim, k, d_ids, d_scores, d_counts)) return s;
    VX_CUDA(cudaSetDevice(ix->device));
    return scan_candidates_dev(ix, d_queries, nq, dim, k, d_ids, d_scores, d_counts,
                               (cudaStream_t)stream);
  });
}

int vx_scan_candidates(vx_index* ix, const float* queries, int32_t nq, int32_t dim, int32_t k,
                       int32_t* ids, float* scores, int32_t* counts) {
  return guarded([&]() -> int {
    if (int s = validate_search(ix, queries, nq, dim, k, ids, scores, counts)) return s;
    return with_host_buffers(ix, queries, nq, dim, k, ids, scores, counts,
                             [&](float* dq, int32_t* di, float* ds, int32_t* dc, cudaStream_t st) {
                               return scan_candidates_dev(ix, dq, nq, dim, k, di, ds, dc, st);
                             });
  });
}

static int ivfpq_dev(vx_index* ix, const float* dq, int nq, int k, int nprobe, int rf, float min_score,
                     int32_t* di, float* ds, int32_t* dc, cudaStream_t st) {
  if (ix->kind != VX_KIND_IVFPQ && ix->kind != VX_KIND_IVFFLAT) return fail(VX_ERR_UNSUPPORTED, "not an IVF index");
  if (nprobe < 1) return fail(VX_ERR_INVALID_ARGUMENT, "nprobe must be >= 1, got %d", nprobe);
  if (rf < 1) return fail(VX_ERR_INVALID_ARGUMENT, "rescoreFactor must be >= 1, got %d", rf);
  if (ix->n == 0) {
    fill_empty(nq, k, di, ds, dc, st);
    return VX_OK;
  }
  return search_ivfpq(ix, dq, nq, k, nprobe, rf, min_score, di, ds, dc, st);
}

int vx_ivfpq_search_device(vx_index* ix, const float* d_queries, int32_t nq, int32_t dim, int32_t k,
                           int32_t nprobe, int32_t rf, float min_score, int32_t* d_ids,
                           float* d_scores, int32_t* d_counts, void* stream) {
  return guarded([&]() -> int {
    if (int s = validate_search(ix, d_queries, nq, dim, k, d_ids, d_scores, d_counts)) return s;
    VX_CUDA(cudaSetDevice(ix->device));
    return ivfpq_dev(ix, d_queries, nq, k, nprobe, rf, min_score, d_ids, d_scores, d_counts,
                     (cudaStream_t)stream);
  });
}

int vx_ivf_route_device(vx_index* ix, const float* d_queries, int32_t nq, int32_t dim, int32_t nprobe,
                        int32_t* d_lists, void* stream) {
  return guarded([&]() -> int {
    if (!ix) return fail(VX_ERR_NULL_POINTER, "index must not be null");
    if (!d_queries || !d_lists) return fail(VX_ERR_NULL_POINTER, "null buffer");
    if (ix->kind != VX_KIND_IVFPQ && ix->kind != VX_KIND_IVFFLAT) return fail(VX_ERR_UNSUPPORTED, "not an IVF index");
    if (nq <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "queries must not be empty");
    if (dim != ix->dim)
      return fail(VX_ERR_INVALID_ARGUMENT, "Query dimension %d does not match index dimension %d", dim, ix->dim);
    if (nprobe < 1) return fail(VX_ERR_INVALID_ARGUMENT, "nprobe must be >= 1, got %d", nprobe);
    VX_CUDA(cudaSetDevice(ix->device));
    return route_ivf(ix, d_queries, nq, nprobe, d_lists, (cudaStream_t)stream);
  });
}

int vx_ivfpq_search_routed_device(vx_index* ix, const float* d_queries, int32_t nq, int32_t dim, int32_t k,
                                  int32_t nprobe, int32_t rf, float min_score, const int32_t* d_lists,
                                  int32_t* d_ids, float* d_scores, int32_t* d_counts, void* stream) {
  return guarded([&]() -> int {
    if (int s = validate_search(ix, d_queries, nq, dim, k, d_ids, d_scores, d_counts)) return s;
    if (!d_lists) return fail(VX_ERR_NULL_POINTER, "lists must not be null");
    if (ix->kind != VX_KIND_IVFPQ && ix->kind != VX_KIND_IVFFLAT) return fail(VX_ERR_UNSUPPORTED, "not an IVF index");
    if (nprobe < 1) return fail(VX_ERR_INVALID_ARGUMENT, "nprobe must be >= 1, got %d", nprobe);
    if (rf < 1) return fail(VX_ERR_INVALID_ARGUMENT, "rescoreFactor must be >= 1, got %d", rf);
    VX_CUDA(cudaSetDevice(ix->device));
    const cudaStream_t st = (cudaStream_t)stream;
    if (ix->n == 0) {
      fill_empty(nq, k, d_ids, d_scores, d_counts, st);
      return VX_OK;
    }
    return search_ivfpq(ix, d_queries, nq, k, nprobe, rf, min_score, d_ids, d_scores, d_counts, st, d_lists);
  });
}

int vx_ivf_route_dist_device(vx_index* ix, const float* d_queries, int32_t nq, int32_t dim, int32_t nprobe,
                             int32_t* d_lists, float* d_list_dist, void* stream) {
  return guarded([&]() -> int {
    if (!ix) return fail(VX_ERR_NULL_POINTER, "index must not be null");
    if (!d_queries || !d_lists || !d_list_dist) return fail(VX_ERR_NULL_POINTER, "null buffer");
    if (ix->kind != VX_KIND_IVFPQ && ix->kind != VX_KIND_IVFFLAT) return fail(VX_ERR_UNSUPPORTED, "not an IVF index");
    if (nq <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "queries must not be empty");
    if (dim != ix->dim)
      return fail(VX_ERR_INVALID_ARGUMENT, "Query dimension %d does not match index dimension %d", dim, ix->dim);
    if (nprobe < 1) return fail(VX_ERR_INVALID_ARGUMENT, "nprobe must be >= 1, got %d", nprobe);
    VX_CUDA(cudaSetDevice(ix->device));
    return route_ivf_dist(ix, d_queries, nq, nprobe, d_lists, d_list_dist, (cudaStream_t)stream);
  });
}

// Shared checks of the two pair entry points: an IVF-flat index the split serves, k in range.
static int check_pair_split(vx_index* ix, int32_t nq, int32_t k, int32_t nprobe) {
  if (!ix) return fail(VX_ERR_NULL_POINTER, "index must not be null");
  if (ix->kind != VX_KIND_IVFFLAT) return fail(VX_ERR_UNSUPPORTED, "not an IVF-flat index");
  if (nq <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "queries must not be empty");
  if (k <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "k must be positive: %d", k);
  if (nprobe < 1) return fail(VX_ERR_INVALID_ARGUMENT, "nprobe must be >= 1, got %d", nprobe);
  if (ix->n == 0) return fail(VX_ERR_UNSUPPORTED, "the pair split needs a non-empty index");
  if (ix->keyed) return fail(VX_ERR_UNSUPPORTED, "partitions with HARMONY key dimensions are searched whole (vx_search_batch)");
  if ((int64_t)nq * std::min(nprobe, ix->nlist) > INT32_MAX)
    return fail(VX_ERR_INVALID_ARGUMENT, "nq * nprobe slots exceed one call (%d queries): split the batch", nq);
  const int K = (int)std::min<int64_t>(k, ix->n);
  if (!flat_list_supported(K) || !early_exit_supported(K))
    return fail(VX_ERR_UNSUPPORTED, "k = %d is larger than the IVF-flat scan keeps (256)", K);
  return VX_OK;
}

int vx_ivfflat_scan_pairs_device(vx_index* ix, const float* d_queries, int32_t nq, int32_t dim, int32_t k,
                                 int32_t nprobe, const int32_t* d_lists, uint64_t* d_pair_keys,
                                 uint32_t* d_pair_counts, void* stream) {
  return guarded([&]() -> int {
    if (int s = check_pair_split(ix, nq, k, nprobe)) return s;
    if (!d_queries || !d_lists || !d_pair_keys || !d_pair_counts) return fail(VX_ERR_NULL_POINTER, "null buffer");
    if (dim != ix->dim)
      return fail(VX_ERR_INVALID_ARGUMENT, "Query dimension %d does not match index dimension %d", dim, ix->dim);
    VX_CUDA(cudaSetDevice(ix->device));
    const int K = (int)std::min<int64_t>(k, ix->n);
    return ivfflat_scan_pairs(ix, d_queries, nq, K, std::min(nprobe, ix->nlist), d_lists, d_pair_keys, d_pair_counts,
                              (cudaStream_t)stream);
  });
}

int vx_ivfflat_merge_pairs_device(vx_index* ix, int32_t nq, int32_t k, int32_t nprobe, const int32_t* d_lists,
                                  const float* d_list_dist, const uint64_t* d_pair_keys,
                                  const uint32_t* d_pair_counts, float min_score, int32_t* d_ids, float* d_scores,
                                  int32_t* d_counts, void* stream) {
  return guarded([&]() -> int {
    if (int s = check_pair_split(ix, nq, k, nprobe)) return s;
    if (!d_lists || !d_list_dist || !d_pair_keys || !d_pair_counts || !d_ids || !d_scores || !d_counts)
      return fail(VX_ERR_NULL_POINTER, "null buffer");
    VX_CUDA(cudaSetDevice(ix->device));
    const int K = (int)std::min<int64_t>(k, ix->n);
    return ivfflat_merge_pairs(ix, nq, k, K, std::min(nprobe, ix->nlist), d_lists, d_list_dist, d_pair_keys,
                               d_pair_counts, min_score, d_ids, d_scores, d_counts, (cudaStream_t)stream);
  });
}

int vx_ivfpq_search(vx_index* ix, const float* queries, int32_t nq, int32_t dim, int32_t k,
                    int32_t nprobe, int32_t rf, float min_score, int32_t* ids, float* scores,
                    int32_t* counts) {
  return guarded([&]() -> int {
    if (int s = validate_search(ix, queries, nq, dim, k, ids, scores, counts)) return s;
    return with_host_buffers(ix, queries, nq, dim, k, ids, scores, counts,
                             [&](float* dq, int32_t* di, float* ds, int32_t* dc, cudaStream_t st) {
                               return ivfpq_dev(ix, dq, nq, k, nprobe, rf, min_score, di, ds, dc, st);
                             });
  });
}

int vx_merge_shards_device(int32_t device, int32_t nshards, const int64_t* d_offsets,
                           const int32_t* d_shard_ids, const float* d_shard_scores,
                           const int32_t* d_shard_counts, int32_t kin, int32_t nq, int32_t k,
                           int32_t* d_ids, float* d_scores, int32_t* d_counts, void* stream) {
  return guarded([&]() -> int {
    if (!d_offsets || !d_shard_ids || !d_shard_scores || !d_shard_counts || !d_ids || !d_scores || !d_counts)
      return fail(VX_ERR_NULL_POINTER, "null buffer");
    if (nshards <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "shards must not be empty");
    if (kin <= 0 || k <= 0 || nq <= 0) return fail(VX_ERR_INVALID_ARGUMENT, "bad merge shape");
    VX_CUDA(cudaSetDevice(device));
    VX_LAUNCH(1, launch_merge_shards(nshards, d_offsets, d_shard_ids, d_shard_scores, d_shard_counts,
                                     kin, nq, k, d_ids, d_scores, d_counts, (cudaStream_t)stream));
    return VX_OK;
  });
}

}  // extern "C"
