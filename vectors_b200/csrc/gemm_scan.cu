// gemm_scan.cu -- tcgen05 / TMA query x database scoring with a fused top-K epilogue.
//
// One kernel skeleton serves two hot paths:
//   * kind::f16  -- the FLAT approximate pass: fp16 copies of the (row-normalised) database
//                   and queries, fp32 accumulation in TMEM.  Its candidates are re-scored
//                   exactly in fp32 afterwards (rescore.cu), restating FlatScanAdapter
//                   (vectors-db/.../index/FlatScanAdapter.java:51-175).
//   * kind::i8   -- the SQ8 scan: 7-bit codes (ScalarQuantizer.java:243-272) multiplied
//                   exactly into int32, followed by the reference score epilogue
//                   (ScalarQuantizedVectors.java:82-107), bit-exact.
//
// Tiling.  A tile is 128 queries (TMEM lanes) x 256 database rows (TMEM columns), reduced
// over the padded dimension in 128-byte K chunks (64 fp16 or 128 int8 elements) staged by
// TMA with 128-byte swizzle through a 4-deep shared-memory ring (48 KB per stage).  Two
// 256-column fp32/s32 accumulators (all 512 TMEM columns) let the epilogue of tile t overlap
// the MMAs of tile t+1.  The (row-tile, query-block) pairs are dealt to CTAs in row-major
// order so that consecutive tiles of one CTA reuse the same database tile from L2 and the
// database streams from HBM about once per batch.
//
// Warp roles (192 threads): warp 0 issues TMA, warp 1 owns TMEM and issues tcgen05.mma,
// warps 2-5 drain TMEM (warp w reads TMEM lanes 32*(w%4)..+31, i.e. one query per thread)
// and feed each query's candidate stream (common.cuh).  Every wait is bounded in time; on
// expiry the kernel records kDevWaitTimeout, the roles unwind and TMEM is released.
#include <cuda.h>
#include "gemm_scan.h"
#include "sm100.cuh"

namespace vx {
namespace {

using namespace sm100;

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK_BYTES = 128;
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK_BYTES;
constexpr int B_BYTES = BN * BK_BYTES;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int NUM_THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr size_t SMEM_BYTES = 1024 + (size_t)STAGES * STAGE_BYTES + 4 * 2 * 256 * sizeof(float) + 256;

__device__ __forceinline__ float thr_to_float(uint64_t thr) {
  return thr == 0 ? -INFINITY : key_score(thr);
}

// Pair p -> (row tile, query block): row-tile-major (consecutive pairs share the database
// tile) or query-block-major (one CTA sweeps its query block over every row tile).
__device__ __forceinline__ void tile_of(int64_t p, const ScanArgs& a, int64_t& nt, int& mb) {
  if (a.m_major) {
    mb = (int)(p / a.ntiles);
    nt = p % a.ntiles;
  } else {
    nt = p / a.num_mblocks;
    mb = (int)(p % a.num_mblocks);
  }
}

// Raises the stream's threshold to the shared floor (admit keys >= floor).
__device__ __forceinline__ void apply_floor(const ScanArgs& a, int q, bool active, uint64_t& thr) {
  if (a.floor && active) {
    const uint64_t f = __ldcg((const unsigned long long*)a.floor + q);  // other CTAs raise it
    if (f > 1 && f - 1 > thr) thr = f - 1;
  }
}

template <bool kI8, int kMode, int R>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_scan_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const ScanArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t* stages = smem;
  float* s_cols = (float*)(smem + (size_t)STAGES * STAGE_BYTES);  // [4 warps][2][256]
  uint64_t* full = (uint64_t*)(s_cols + 4 * 2 * 256);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = (uint32_t*)(tempty + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t total = a.ntiles * (int64_t)a.num_mblocks;
  const int64_t p0 = total * blockIdx.x / gridDim.x;
  const int64_t p1 = total * (blockIdx.x + 1) / gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  auto give_up = [&]() {
    *abort_flag = 1;
    record_error(a.err, kDevWaitTimeout);
  };

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      const uint64_t pol_a = policy_evict_last();  // query tiles are re-read by every row tile
      int stage = 0;
      uint32_t phase = 0;
      uint32_t used = 0;      // bit s: stage s has had a load issued
      uint32_t last_par = 0;  // bit s: parity of the last phase issued on stage s
      for (int64_t p = p0; p < p1 && !*abort_flag; p++) {
        int64_t nt;
        int mb;
        tile_of(p, a, nt, mb);
        for (int kc = 0; kc < a.kchunks; kc++) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, globaltimer_ns() + a.timeout_ns, abort_flag)) {
            give_up();
            break;
          }
          mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
          uint8_t* sa = stages + (size_t)stage * STAGE_BYTES;
          const int x = kc * (kI8 ? 128 : 64);
          tma_load_2d_hint(sa, &tmA, &full[stage], x, mb * BM, pol_a);
          tma_load_2d(sa + A_BYTES, &tmB, &full[stage], x, (int32_t)(nt * BN));
          used |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort_flag) {
        // Let every load already issued land before the CTA's shared memory is released.
        const uint64_t until = globaltimer_ns() + a.timeout_ns;
        for (;;) {
          bool all = true;
          for (int s = 0; s < STAGES; s++)
            if ((used >> s) & 1u)
              if (!mbar_try_wait(&full[s], (last_par >> s) & 1u)) all = false;
          if (all || globaltimer_ns() > until) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = kI8 ? idesc_s8_s32(BM, BN) : idesc_f16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int64_t t = 0;
      for (int64_t p = p0; p < p1 && !*abort_flag; p++, t++) {
        const int acc = (int)(t & 1);
        const uint32_t acc_phase = (uint32_t)((t >> 1) & 1);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, globaltimer_ns() + a.timeout_ns, abort_flag)) {
          give_up();
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kc = 0; kc < a.kchunks; kc++) {
          if (!mbar_wait(&full[stage], phase, globaltimer_ns() + a.timeout_ns, abort_flag)) {
            give_up();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_addr(stages + (size_t)stage * STAGE_BYTES);
          const uint64_t da = sw128_kmajor_desc(sa);
          const uint64_t db = sw128_kmajor_desc(sa + A_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const uint32_t accum = (kc | kk) != 0 ? 1u : 0u;
            if (kI8)
              mma_i8(d, da + 2ull * kk, db + 2ull * kk, idesc, accum);
            else
              mma_f16(d, da + 2ull * kk, db + 2ull * kk, idesc, accum);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&tfull[acc]);
      }
    }
  } else {
    // ---------------- epilogue: warps 2..5, one query (TMEM lane) per thread
    const int quarter = warp & 3;
    const int row_in_block = quarter * 32 + lane;
    const int etid = threadIdx.x - 64;
    const int Qp = a.num_mblocks * BM;
    int64_t t = 0;
    for (int64_t p = p0; p < p1; p++, t++) {
      int64_t nt;
      int mb;
      tile_of(p, a, nt, mb);
      const int acc = (int)(t & 1);
      const uint32_t acc_phase = (uint32_t)((t >> 1) & 1);
      const int64_t col0 = nt * BN;
      float* s_col = s_cols + (warp - 2) * 512;  // this warp's private column data
      float* s_col2 = s_col + 256;
      if (kMode != kEpiF16Plain) {
        __syncwarp();
        for (int i = lane; i < BN; i += 32) {
          const int64_t row = col0 + i;
          const bool in = row < a.n;
          if (kMode == kEpiF16Scaled || kMode == kEpiF16L2) {
            s_col[i] = in ? a.epi.xnorm[row] : 0.0f;
            if (kMode == kEpiF16L2) s_col2[i] = in ? a.epi.rowsq[row] : 0.0f;
          } else if (kMode == kEpiSq8Dot || kMode == kEpiSq8Mip) {
            s_col[i] = in ? a.epi.vcorr[row] : 0.0f;
          } else {  // kEpiSq8L2
            s_col[i] = __int_as_float(in ? a.epi.vsq[row] : 0);
          }
        }
        __syncwarp();
      }
      if (__shfl_sync(0xFFFFFFFFu, *abort_flag, 0)) break;
      {
        bool ok = mbar_wait(&tfull[acc], acc_phase, globaltimer_ns() + a.timeout_ns, abort_flag);
        ok = __all_sync(0xFFFFFFFFu, ok);
        if (!ok) {
          if (lane == 0) give_up();
          break;
        }
      }
      tc_fence_after();
      const int q = mb * BM + row_in_block;
      const bool active = q < a.nq;
      const size_t sidx = (size_t)blockIdx.x * Qp + (size_t)q;
      LaneStream st;
      st.base = a.bufs + sidx * (size_t)a.C;
      st.cnt = active ? a.cnts[sidx] : 0u;
      st.thr = active ? a.thrs[sidx] : ~0ull;
      apply_floor(a, q, active, st.thr);
      float tf = active ? thr_to_float(st.thr) : INFINITY;
      float qa = 0.0f;
      int32_t qi = 0;
      if (active) {
        if (kMode == kEpiF16L2) qa = 2.0f * a.epi.qscale[q];  // key = 2|q||x| acc - |x|^2
        if (kMode == kEpiSq8Dot || kMode == kEpiSq8Mip) qa = a.epi.qscale[q];
        if (kMode == kEpiSq8L2) qi = a.epi.qsq[q];
      }
      const int64_t left = a.n - col0;
      const int valid = left < BN ? (int)left : BN;
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ch++) {
        uint32_t v[32];
        __syncwarp();
        tmem_ld_32x32b_x32(taddr + (uint32_t)(ch * 32), v);
        tmem_ld_wait();
        if (ch * 32 < valid) {
#pragma unroll
          for (int j = 0; j < 32; j++) {
            const int col = ch * 32 + j;
            float s;
            if (kMode == kEpiF16Plain) {
              s = __uint_as_float(v[j]);
            } else if (kMode == kEpiF16Scaled) {
              s = __uint_as_float(v[j]) * s_col[col];
            } else if (kMode == kEpiF16L2) {
              s = fmaf(qa * s_col[col], __uint_as_float(v[j]), -s_col2[col]);
            } else if (kMode == kEpiSq8Dot || kMode == kEpiSq8Mip) {
              // rawDot * constMultiplier + queryCorrection + corrections[ordinal]
              const float adj = __fadd_rn(
                  __fadd_rn(__fmul_rn(__int2float_rn((int32_t)v[j]), a.epi.cm), qa),
                  s_col[col]);
              if (kMode == kEpiSq8Dot) {
                const float h = __fmul_rn(__fadd_rn(1.0f, adj), 0.5f);  // (1f + adj) / 2f
                s = h >= 0.0f ? h : (h != h ? h : 0.0f);               // Math.max(h, 0f)
              } else {
                s = scale_mip(adj);
              }
            } else {  // kEpiSq8L2: sum (q-v)^2 = sum q^2 + sum v^2 - 2 q.v, exact in int32
              const int32_t sq = qi + __float_as_int(s_col[col]) - 2 * (int32_t)v[j];
              s = __fdiv_rn(1.0f, __fadd_rn(1.0f, __fmul_rn(__int2float_rn(sq), a.epi.cm)));
            }
            if (col < valid && s >= tf) {
              const uint64_t key = float_key(s, (uint32_t)(col0 + col));
              if (key > st.thr) st.base[st.cnt++] = key;
            }
          }
        }
        const bool need = st.cnt > (uint32_t)(a.C - 32);
        if (__any_sync(0xFFFFFFFFu, need)) {
          warp_compact_lanes<R>(need, st.base, st.cnt, st.thr, (uint32_t)a.K);
          if (need && a.floor && st.cnt == (uint32_t)a.K)
            atomicMax((unsigned long long*)&a.floor[q], (unsigned long long)st.thr);
          apply_floor(a, q, active, st.thr);
          tf = active ? thr_to_float(st.thr) : INFINITY;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      if (active) {
        a.cnts[sidx] = st.cnt;
        a.thrs[sidx] = st.thr;
      }
    }
    // Leave every stream this CTA wrote with at most K keys.
    if (!__shfl_sync(0xFFFFFFFFu, *abort_flag, 0)) {
      for (int mb = 0; mb < a.num_mblocks; mb++) {
        const int q = mb * BM + row_in_block;
        const bool active = q < a.nq;
        const size_t sidx = (size_t)blockIdx.x * Qp + (size_t)q;
        uint64_t* base = a.bufs + sidx * (size_t)a.C;
        uint32_t cnt = active ? a.cnts[sidx] : 0u;
        uint64_t thr = active ? a.thrs[sidx] : ~0ull;
        const bool need = cnt > (uint32_t)a.K;
        warp_compact_lanes<R>(need, base, cnt, thr, (uint32_t)a.K);
        if (active) {
          a.cnts[sidx] = cnt;
          a.thrs[sidx] = thr;
          if (need && a.floor) atomicMax((unsigned long long*)&a.floor[q], (unsigned long long)thr);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <bool kI8, int kMode>
cudaError_t launch_mode(const CUtensorMap& tmA, const CUtensorMap& tmB, const ScanArgs& a, int grid,
                        int R, cudaStream_t st) {
#define VX_GS_CASE(RR)                                                                         \
  case RR: {                                                                                   \
    auto kern = gemm_scan_kernel<kI8, kMode, RR>;                                              \
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,    \
                                         (int)SMEM_BYTES);                                     \
    if (e != cudaSuccess) return e;                                                            \
    kern<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(tmA, tmB, a);                                  \
    return cudaGetLastError();                                                                 \
  }
  switch (R) {
    VX_GS_CASE(3)
    VX_GS_CASE(5)
    VX_GS_CASE(9)
    VX_GS_CASE(17)
    VX_GS_CASE(33)
    default: return cudaErrorInvalidValue;
  }
#undef VX_GS_CASE
}

}  // namespace

int gemm_scan_grid(int64_t ntiles, int num_mblocks, int num_sms) {
  int64_t total = ntiles * (int64_t)num_mblocks;
  int64_t g = num_sms;
  if (g > total) g = total;
  return (int)(g < 1 ? 1 : g);
}

int gemm_scan_stream_R(int K) {
  StreamGeom g = stream_geom(K, 32);
  return g.R == 2 ? 3 : g.R;  // the GEMM scan instantiates R in {3,5,9,17,33}
}

cudaError_t launch_gemm_scan(int mode, const CUtensorMap& tmA, const CUtensorMap& tmB,
                             const ScanArgs& a, int grid, int R, cudaStream_t st) {
  switch (mode) {
    case kEpiF16Plain: return launch_mode<false, kEpiF16Plain>(tmA, tmB, a, grid, R, st);
    case kEpiF16Scaled: return launch_mode<false, kEpiF16Scaled>(tmA, tmB, a, grid, R, st);
    case kEpiF16L2: return launch_mode<false, kEpiF16L2>(tmA, tmB, a, grid, R, st);
    case kEpiSq8Dot: return launch_mode<true, kEpiSq8Dot>(tmA, tmB, a, grid, R, st);
    case kEpiSq8Mip: return launch_mode<true, kEpiSq8Mip>(tmA, tmB, a, grid, R, st);
    case kEpiSq8L2: return launch_mode<true, kEpiSq8L2>(tmA, tmB, a, grid, R, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace vx
