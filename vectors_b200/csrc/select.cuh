// select.cuh -- block-level K-best selection and sorting over 64-bit ranking keys.
#pragma once
#include "common.cuh"

namespace vx {

// Block-wide sum of a per-thread count (blockDim.x a multiple of 32, <= 1024).
__device__ __forceinline__ uint32_t block_sum_u32(uint32_t v, uint32_t* s_red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = __reduce_add_sync(0xFFFFFFFFu, v);
  __syncthreads();
  if (lane == 0) s_red[warp] = v;
  __syncthreads();
  uint32_t t = 0;
  for (int i = 0; i < nw; i++) t += s_red[i];
  return t;
}

// Largest key t with #(keys >= t) >= K among s_keys[0, n) (keys unique, n > K > 0).
// Every thread returns the same t; #(keys >= t) == K afterwards.
__device__ __forceinline__ uint64_t block_kth_largest(const uint64_t* s_keys, uint32_t n, uint32_t K,
                                                      uint32_t* s_red) {
  uint64_t t = 0;
  for (int b = 63; b >= 0; b--) {
    uint64_t cand = t | (1ull << b);
    uint32_t c = 0;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) c += (s_keys[i] >= cand) ? 1u : 0u;
    c = block_sum_u32(c, s_red);
    if (c >= K) {
      t = cand;
      if (c == K) break;
    }
  }
  return t;
}

// Keeps the K largest of s_keys[0, n) in s_keys[0, min(n,K)); returns the new count.
// Uses s_tmp (>= n slots) as scratch.  Order of the survivors is unspecified.
__device__ __forceinline__ uint32_t block_keep_top(uint64_t* s_keys, uint32_t n, uint32_t K,
                                                   uint64_t* s_tmp, uint32_t* s_red,
                                                   uint32_t* s_counter) {
  if (n <= K) return n;
  uint64_t t = block_kth_largest(s_keys, n, K, s_red);
  if (threadIdx.x == 0) *s_counter = 0;
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    uint64_t k = s_keys[i];
    if (k >= t) s_tmp[atomicAdd(s_counter, 1u)] = k;
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < K; i += blockDim.x) s_keys[i] = s_tmp[i];
  __syncthreads();
  return K;
}

// Sorts s_keys[0, n) descending (bitonic over the next power of two; pads with empty keys).
__device__ __forceinline__ void block_sort_desc(uint64_t* s_keys, uint32_t n, uint32_t cap) {
  uint32_t p = 1;
  while (p < n) p <<= 1;
  for (uint32_t i = n + threadIdx.x; i < p && i < cap; i += blockDim.x) s_keys[i] = kEmptyKey;
  __syncthreads();
  for (uint32_t size = 2; size <= p; size <<= 1) {
    for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
      for (uint32_t i = threadIdx.x; i < p / 2; i += blockDim.x) {
        uint32_t lo = 2 * i - (i & (stride - 1));
        uint32_t hi = lo + stride;
        bool desc = ((lo & size) == 0);
        uint64_t a = s_keys[lo], b = s_keys[hi];
        if ((a < b) == desc) {
          s_keys[lo] = b;
          s_keys[hi] = a;
        }
      }
      __syncthreads();
    }
  }
}

}  // namespace vx
