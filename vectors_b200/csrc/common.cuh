// common.cuh -- shared device helpers for the scan kernels.
//
// Ranking keys.  Every scan ranks by (score desc, id asc), the canonical order of
// TopK.select (vectors-core/.../TopK.java:96-116).  A candidate is packed into one
// 64-bit key so that "larger key" == "better candidate":
//     key = (order_preserving_bits(score) << 32) | (0xFFFFFFFF - id)
// ids are int32 ordinals (< 2^31), so the low word is >= 2^31 and a real key is never 0;
// 0 means "empty".  Integer-distance scans (Hamming) put (0xFFFFFFFF - distance) in the
// high word instead of float bits.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace vx {

constexpr uint64_t kEmptyKey = 0ull;

__host__ __device__ __forceinline__ uint32_t float_order_bits(float f) {
#ifdef __CUDA_ARCH__
  uint32_t b = __float_as_uint(f);
#else
  uint32_t b;
  __builtin_memcpy(&b, &f, 4);
#endif
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__host__ __device__ __forceinline__ float order_bits_float(uint32_t o) {
  uint32_t b = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
#ifdef __CUDA_ARCH__
  return __uint_as_float(b);
#else
  float f;
  __builtin_memcpy(&f, &b, 4);
  return f;
#endif
}
__host__ __device__ __forceinline__ uint64_t make_key(uint32_t hi, uint32_t id) {
  return ((uint64_t)hi << 32) | (uint64_t)(0xFFFFFFFFu - id);
}
__host__ __device__ __forceinline__ uint64_t float_key(float s, uint32_t id) {
  return make_key(float_order_bits(s), id);
}
__host__ __device__ __forceinline__ uint32_t key_id(uint64_t k) {
  return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
}
__host__ __device__ __forceinline__ uint32_t key_hi(uint64_t k) { return (uint32_t)(k >> 32); }
__host__ __device__ __forceinline__ float key_score(uint64_t k) { return order_bits_float(key_hi(k)); }

// Error word shared by all kernels of one call: the first failing site records its code.
enum DeviceError : int32_t {
  kDevOk = 0,
  kDevWaitTimeout = 1,   // an mbarrier / flag wait exceeded its time budget
  kDevBadShape = 2,      // a launch was given sizes the kernel cannot handle
};

__device__ __forceinline__ void record_error(int32_t* err, int32_t code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Warp-wide 64-bit min.
__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    uint64_t w = __shfl_xor_sync(0xFFFFFFFFu, v, o);
    v = w < v ? w : v;
  }
  return v;
}

// --------------------------------------------------------------------------------------
// Lane-owned streaming top-K.
//
// Each lane of a warp owns one query's candidate stream (the GEMM epilogue gives one
// TMEM lane = one query per thread).  The lane keeps a threshold `thr` (keys <= thr can
// no longer reach its top-K) and appends admitted keys to its own buffer of C = 32*R
// slots in global memory.  When some lane's buffer may overflow, the whole warp helps
// that lane shrink its buffer to exactly its K best keys (bitwise search for the K-th
// largest key over the lane's buffer, spread 32 ways), and raises its threshold to the
// smallest kept key.  Appends between two checks must be <= C - K - 1 (the caller's
// "slack").
// --------------------------------------------------------------------------------------
template <int R>
__device__ __forceinline__ void warp_compact_one(uint64_t* base, uint32_t n, uint32_t K,
                                                 uint64_t& thr_out, uint32_t& cnt_out) {
  const int lane = threadIdx.x & 31;
  uint64_t e[R];
#pragma unroll
  for (int r = 0; r < R; r++) {
    uint32_t i = lane + 32 * r;
    e[r] = (i < n) ? base[i] : kEmptyKey;
  }
  // Largest t with #(keys >= t) >= K, i.e. the K-th largest key; stop early once the
  // prefix already isolates exactly K keys.
  uint64_t t = 0;
  for (int b = 63; b >= 0; b--) {
    uint64_t cand = t | (1ull << b);
    uint32_t c = 0;
#pragma unroll
    for (int r = 0; r < R; r++) c += (e[r] >= cand) ? 1u : 0u;
    c = __reduce_add_sync(0xFFFFFFFFu, c);
    if (c >= K) {
      t = cand;
      if (c == K) break;
    }
  }
  // Keep keys >= t (exactly K of them), compact to the front.
  uint32_t mine = 0;
#pragma unroll
  for (int r = 0; r < R; r++) mine += (e[r] >= t && e[r] != kEmptyKey) ? 1u : 0u;
  uint32_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    uint32_t v = __shfl_up_sync(0xFFFFFFFFu, incl, o);
    if (lane >= o) incl += v;
  }
  uint32_t pos = incl - mine;
  uint64_t mn = ~0ull;
  __syncwarp();
#pragma unroll
  for (int r = 0; r < R; r++) {
    if (e[r] >= t && e[r] != kEmptyKey) {
      base[pos++] = e[r];
      mn = e[r] < mn ? e[r] : mn;
    }
  }
  __syncwarp();
  mn = warp_min_u64(mn);
  thr_out = mn;
  cnt_out = __shfl_sync(0xFFFFFFFFu, incl, 31);
}

// Shrinks, for every lane whose predicate holds, that lane's buffer to its K best keys.
template <int R>
__device__ __forceinline__ void warp_compact_lanes(bool need, uint64_t* my_base, uint32_t& my_cnt,
                                                   uint64_t& my_thr, uint32_t K) {
  const int lane = threadIdx.x & 31;
  uint32_t mask = __ballot_sync(0xFFFFFFFFu, need);
  while (mask) {
    int src = __ffs(mask) - 1;
    mask &= mask - 1;
    uint64_t* base = (uint64_t*)__shfl_sync(0xFFFFFFFFu, (unsigned long long)my_base, src);
    uint32_t n = __shfl_sync(0xFFFFFFFFu, my_cnt, src);
    uint64_t thr;
    uint32_t cnt;
    warp_compact_one<R>(base, n, K, thr, cnt);
    if (lane == src) {
      my_thr = thr;
      my_cnt = cnt;
    }
  }
}

// Lane-owned stream state.
struct LaneStream {
  uint64_t* base;  // this lane's buffer (C slots)
  uint64_t thr;
  uint32_t cnt;
  __device__ __forceinline__ void offer(uint64_t key) {
    if (key > thr) base[cnt++] = key;
  }
};

}  // namespace vx
