// gemm_scan.cu -- tcgen05 / TMA query x database scoring with a fused top-K epilogue.
//
// One kernel skeleton serves two hot paths:
//   * kind::f16  -- the FLAT approximate pass: fp16 copies of the (row-normalised) database
//                   and queries, fp32 accumulation in TMEM.  Its candidates are re-scored
//                   exactly in fp32 afterwards (rescore.cu), restating FlatScanAdapter
//                   (vectors-db/.../index/FlatScanAdapter.java:51-175).
//   * kind::i8   -- the SQ8 scan: 7-bit codes (ScalarQuantizer.java:243-272) multiplied
//                   exactly into int32, followed by the reference score epilogue
//                   (ScalarQuantizedVectors.java:82-107), bit-exact.  The same pipeline serves
//                   sign-bit BQ (+-1 operands, Hamming epilogue) and BBQ (0/1 row bits x 4-bit
//                   query codes = rawAsymDot, BinaryQuantizedVectors.java:110-275, epilogue in
//                   bbq.cuh).
//
// Tiling.  The default variant runs on 2-CTA clusters (tcgen05 cta_group::2): a cluster owns
// a 256-query x 256-row tile; each CTA stages only its own 128 query rows and 128 database
// rows of every 128-byte K chunk (64 fp16 / 128 int8 elements) through a 6-deep TMA ring (5-deep
// for BBQ, whose per-row epilogue records take four words instead of two) with 128-byte swizzle, i.e. 32 KB of shared memory traffic per SM for 128 x 256 x 64 MACs.  The
// leader CTA issues the pair MMA; each CTA's TMEM holds its 128 queries x 256 rows in
// fp32/s32, double buffered (512 columns) so that the epilogue of tile t overlaps the MMAs of
// tile t+1.  A 1-CTA variant (128 x 256 tiles, 48 KB per stage) is kept for comparison.
// (row-tile, query-block) pairs are dealt to clusters in row-major order so that consecutive
// tiles reuse one database tile from L2 and the database streams from HBM about once per batch.
//
// Warp roles (192 threads per CTA): warp 0 issues TMA, warp 1 owns TMEM and (leader only)
// issues tcgen05.mma, warps 2-5 drain TMEM (warp w reads TMEM lanes 32*(w%4)..+31, i.e. one
// query per thread) and feed each query's candidate stream (common.cuh).  The two CTAs of a
// cluster own disjoint queries, so they share one set of streams.  Every wait is bounded in
// time; on expiry the kernel records kDevWaitTimeout, the roles unwind and TMEM is released.
// No TMA load uses cluster multicast.
#include <cuda.h>
#include "bbq.cuh"
#include "gemm_scan.h"
#include "sm100.cuh"

namespace vx {
namespace {

using namespace sm100;

constexpr int BN = 256;        // database rows per tile (TMEM columns per accumulator)
constexpr int BK_BYTES = 128;  // bytes of K per stage row
constexpr int TMEM_COLS = 512;
constexpr int kStageRowWords = 36;  // per-lane staging row: 32 values + 4 words of padding
                                    // (16-byte stores of 8 lanes hit 8 distinct bank quads)

// Per-row float arrays the epilogue stages for each tile: two (row scale, |x|^2 or the SQ8
// terms), four for BBQ.
__host__ __device__ constexpr int cols_of(int mode) { return epi_is_bbq(mode) ? 4 : 2; }

template <bool k2Sm, int kCols>
struct Geo {
  static constexpr int kStages = k2Sm ? (kCols > 2 ? 5 : 6) : (kCols > 2 ? 3 : 4);
  static constexpr int kRowsB = k2Sm ? 128 : 256;  // database rows staged per CTA
  static constexpr int kABytes = 128 * BK_BYTES;    // 128 query rows per CTA
  static constexpr int kBBytes = kRowsB * BK_BYTES;
  static constexpr int kStageBytes = kABytes + kBBytes;               // per CTA
  static constexpr int kTxBytes = k2Sm ? 2 * kStageBytes : kStageBytes;  // on the leader's barrier
  static constexpr int kQueriesPerTile = k2Sm ? 256 : 128;
  static constexpr size_t kSmem = 1024 + (size_t)kStages * kStageBytes + 4 * kCols * 256 * sizeof(float) +
                                  4 * 32 * kStageRowWords * sizeof(uint32_t) + 256;
  static_assert(kSmem <= 232448, "shared memory above the per-block limit");
};

__device__ __forceinline__ float thr_to_float(uint64_t thr) {
  return thr == 0 ? -INFINITY : key_score(thr);
}

// Pair p -> (row tile, query block): row-tile-major (consecutive pairs share the database
// tile) or query-block-major (one CTA / cluster sweeps its query block over every row tile).
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

// BBQ: computeBbqDot of one accumulator value (rawAsymDot) against the staged row record
// s_col[col] = vl, s_col[256 + col] = width, s_col[512 + col] = vl * D + width * pop
// (s_col[768 + col] = |v - c| or |v - c|^2); qb holds the lane's query (queryMin,
// queryWidth / 15, querySum, queryNormSq or queryNorm).  Neither a 16-byte record load per
// column nor an integer-to-float by the 2^23 bias (LOP3 + FADD) made the scan faster.
__device__ __forceinline__ float bbq_approx_at(uint32_t v, int col, const float* s_col, const float4& qb) {
  return bbq_approx(qb.x, qb.y, qb.z, s_col[col], s_col[256 + col], s_col[512 + col], __int2float_rn((int32_t)v));
}

// Ranking score of one accumulator value in epilogue mode kMode (gemm_scan.h), split into a
// per-column inner quantity and a monotone tail applied to it: group_max computes every
// column's inner quantity once and leaves it in the accumulator registers in place of the raw
// value, so the admission slow path applies only the tail.  Inner quantities: F16Plain /
// F16Scaled / F16L2 / BbqCos the score (no tail); Sq8Dot / Sq8Mip adj = rawDot *
// constMultiplier + queryCorrection + correction[ordinal]; Sq8L2 the integer squared distance;
// BqHamming the raw +-1 dot; BbqDot / BbqMip computeBbqDot; BbqL2 the clamped distance term.
template <int kMode>
__device__ __forceinline__ uint32_t inner_of(uint32_t v, int col, const float* s_col, const float* s_col2,
                                             float qa, int32_t qi, float cm, const float4& qb) {
  if constexpr (kMode == kEpiBbqDot || kMode == kEpiBbqMip) {
    return __float_as_uint(bbq_approx_at(v, col, s_col, qb));
  } else if constexpr (kMode == kEpiBbqL2) {
    return __float_as_uint(bbq_l2_adj(bbq_approx_at(v, col, s_col, qb), qb.w, s_col[768 + col]));
  } else if constexpr (kMode == kEpiBbqCos) {
    return __float_as_uint(bbq_cos_score(bbq_approx_at(v, col, s_col, qb), qb.w, s_col[768 + col]));
  } else if constexpr (kMode == kEpiF16Scaled) {
    return __float_as_uint(__uint_as_float(v) * s_col[col]);
  } else if constexpr (kMode == kEpiF16L2) {
    return __float_as_uint(fmaf(qa * s_col[col], __uint_as_float(v), -s_col2[col]));
  } else if constexpr (kMode == kEpiSq8Dot || kMode == kEpiSq8Mip) {
    return __float_as_uint(__fadd_rn(__fadd_rn(__fmul_rn(__int2float_rn((int32_t)v), cm), qa), s_col[col]));
  } else if constexpr (kMode == kEpiSq8L2) {
    return (uint32_t)(qi + __float_as_int(s_col[col]) - 2 * (int32_t)v);
  } else {  // F16Plain, BqHamming
    return v;
  }
}

template <int kMode>
__device__ __forceinline__ float tail_of(uint32_t x, int32_t qi, float cm) {
  if constexpr (kMode == kEpiSq8Dot) {
    const float h = __fmul_rn(__fadd_rn(1.0f, __uint_as_float(x)), 0.5f);  // (1f + adj) / 2f
    return h >= 0.0f ? h : (h != h ? h : 0.0f);                            // Math.max(h, 0f)
  } else if constexpr (kMode == kEpiSq8Mip || kMode == kEpiBbqMip) {
    return scale_mip(__uint_as_float(x));
  } else if constexpr (kMode == kEpiSq8L2) {
    return __fdiv_rn(1.0f, __fadd_rn(1.0f, __fmul_rn(__int2float_rn((int32_t)x), cm)));
  } else if constexpr (kMode == kEpiBqHamming) {
    return -(float)((qi - (int32_t)x) >> 1);
  } else if constexpr (kMode == kEpiBbqDot) {
    return bbq_dot_score(__uint_as_float(x));
  } else if constexpr (kMode == kEpiBbqL2) {
    return bbq_l2_score(__uint_as_float(x));
  } else {
    return __uint_as_float(x);
  }
}

// Per-lane state of one query's stream during a tile.
struct TileStream {
  LaneStream st;
  float tf;     // score of the admission threshold
  uint64_t t1;  // best admitted key
  uint64_t t2;  // second best admitted key
  bool dirty;   // keys were appended or the buffer compacted: the state goes back to memory
  uint64_t ceil;  // keys >= ceil are not admitted (~0: no bound)
};

// SQ8 DOT_PRODUCT / COSINE: a bound below the smallest adj whose score max((1 + adj) / 2, 0)
// reaches tf.  For tf > 0 such an adj has fl(1 + adj) >= 2 tf, so adj >= 2 tf - 1 less half an
// ulp of 2 tf; the margin (|2 tf| + 1) 2^-20 covers that and the rounding of 2 tf - 1 many
// times over.  tf <= 0 (or NaN): every score reaches it (NaN scores never: NaN >= x is false
// either way).  tf >= 1e38, where 2 tf overflows: tf itself (2 tf - 1 > tf).
__device__ __forceinline__ float sq8dot_adj_bound(float tf) {
  if (!(tf > 0.0f)) return -INFINITY;
  if (!(tf < 1.0e38f)) return tf;
  const float two = 2.0f * tf;
  return __fsub_rn(__fsub_rn(two, 1.0f), __fmul_rn(fabsf(two) + 1.0f, 9.5367431640625e-7f));
}

// BQ: the smallest raw +-1 dot whose Hamming score -((D - raw) >> 1) can reach tf.  raw = D - 2h
// for a distance h in [0, D], so -h >= tf iff h <= floor(-tf) iff raw >= D - 2 floor(-tf) (one
// less keeps every raw of D's parity).  tf > 0, NaN or +inf (inactive lane): none; -tf at or
// above 2^24 (tf = -inf before any key): all.
__device__ __forceinline__ int32_t bq_min_raw(float tf, int32_t d) {
  const float u = -tf;
  if (!(u >= 0.0f)) return d + 1;
  if (u >= 16777216.0f) return -d;
  return d - 2 * (int32_t)floorf(u) - 1;
}

// Slow path of one 32-column group, taken when some lane of the warp may admit a column:
// builds the lane's pass mask from the inner quantities group_max left in v[] (SQ8 DOT, BBQ DOT
// and BQ: against a bound in the inner quantity itself, a superset of the columns that reach
// the threshold),
// stages them in the lane's private shared-memory row (so that the append loop can index
// them), compacts first when the stream could overflow, then appends, in ascending column
// order, the passing columns whose exact keys clear the threshold.
template <int kMode, int R>
__device__ __forceinline__ void offer_group(const ScanArgs& a, TileStream& ts, int q, bool active,
                                            const uint32_t (&v)[32], int c0, int limit, int64_t col0,
                                            int32_t qi, uint32_t* stage_row) {
  uint32_t pm = 0;
  if constexpr (kMode == kEpiSq8Dot) {
    const float lo = sq8dot_adj_bound(ts.tf);
#pragma unroll
    for (int j = 0; j < 32; j++) pm |= (__uint_as_float(v[j]) >= lo ? 1u : 0u) << j;
  } else if constexpr (kMode == kEpiBqHamming) {
    const int32_t lo = bq_min_raw(ts.tf, qi);
#pragma unroll
    for (int j = 0; j < 32; j++) pm |= ((int32_t)v[j] >= lo ? 1u : 0u) << j;
  } else if constexpr (kMode == kEpiBbqDot) {
    // max((1 + approx) / 2, 0) with NaN -> 0: above 0 the same bound as SQ8 DOT; at or below 0
    // every column (a NaN approx included) reaches the threshold
    const float lo = sq8dot_adj_bound(ts.tf);
    if (ts.tf > 0.0f) {
#pragma unroll
      for (int j = 0; j < 32; j++) pm |= (__uint_as_float(v[j]) >= lo ? 1u : 0u) << j;
    } else {
      pm = 0xFFFFFFFFu;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; j++) pm |= (tail_of<kMode>(v[j], qi, a.epi.cm) >= ts.tf ? 1u : 0u) << j;
  }
  if (limit < 32) pm &= limit <= 0 ? 0u : (0xFFFFFFFFu >> (32 - limit));  // rows beyond n
  if (pm) {
    uint4* d = reinterpret_cast<uint4*>(stage_row);
#pragma unroll
    for (int i = 0; i < 8; i++) d[i] = make_uint4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
  }
  ts.dirty |= pm != 0;
  const bool need = ts.st.cnt + (uint32_t)__popc(pm) > (uint32_t)a.C;
  ts.dirty |= need;
  if (__any_sync(0xFFFFFFFFu, need)) {
    warp_compact_lanes<R>(need, ts.st.base, ts.st.cnt, ts.st.thr, (uint32_t)a.K);
    if (need && a.floor && ts.st.cnt == (uint32_t)a.K)
      atomicMax((unsigned long long*)&a.floor[q], (unsigned long long)ts.st.thr);
    apply_floor(a, q, active, ts.st.thr);
    ts.tf = active ? thr_to_float(ts.st.thr) : INFINITY;
  }
  while (pm) {
    const int j = __ffs(pm) - 1;
    pm &= pm - 1;
    const int col = c0 + j;
    const float sc = tail_of<kMode>(stage_row[j], qi, a.epi.cm);
    const uint64_t key = float_key(sc, (uint32_t)(col0 + col));
    if (key > ts.st.thr && key < ts.ceil) {
      ts.st.base[ts.st.cnt++] = key;
      if (key > ts.t1) {
        ts.t2 = ts.t1;
        ts.t1 = key;
      } else if (key > ts.t2) {
        ts.t2 = key;
      }
    }
  }
}

// Largest score of a 32-column group, exact: every column's inner quantity (left in v[] for the
// admission slow path), their extreme (largest; smallest for the integer squared distance and
// the clamped BBQ distance term, never NaN, whose scores fall as they grow) by a pairwise tree
// (one epilogue warp per scheduler, so the dependency depth matters more than the operation
// count), and the monotone tail of that extreme.
template <int kMode>
__device__ __forceinline__ float group_max(uint32_t (&v)[32], int c0, const float* s_col, const float* s_col2,
                                           float qa, int32_t qi, const EpiParams& e, const float4& qb) {
#pragma unroll
  for (int j = 0; j < 32; j++) v[j] = inner_of<kMode>(v[j], c0 + j, s_col, s_col2, qa, qi, e.cm, qb);
  if constexpr (kMode == kEpiBqHamming || kMode == kEpiSq8L2) {
    constexpr bool kMin = kMode == kEpiSq8L2;
    int32_t m[16];
#pragma unroll
    for (int i = 0; i < 16; i++)
      m[i] = kMin ? min((int32_t)v[2 * i], (int32_t)v[2 * i + 1]) : max((int32_t)v[2 * i], (int32_t)v[2 * i + 1]);
#pragma unroll
    for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
      for (int i = 0; i < w; i++) m[i] = kMin ? min(m[i], m[i + w]) : max(m[i], m[i + w]);
    return tail_of<kMode>((uint32_t)m[0], qi, e.cm);
  } else {
    constexpr bool kMin = kMode == kEpiBbqL2;
    float m[16];
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float x0 = __uint_as_float(v[2 * i]), x1 = __uint_as_float(v[2 * i + 1]);
      m[i] = kMin ? fminf(x0, x1) : fmaxf(x0, x1);
    }
#pragma unroll
    for (int w = 8; w >= 1; w >>= 1)
#pragma unroll
      for (int i = 0; i < w; i++) m[i] = kMin ? fminf(m[i], m[i + w]) : fmaxf(m[i], m[i + w]);
    return tail_of<kMode>(__float_as_uint(m[0]), qi, e.cm);
  }
}

// Pooled-floor check after row tile li (0-based) of a unit's range: right after its first
// tiles, then every 32nd (every 4th, 8th and 16th measured slower: the checks' loads cost more
// than the earlier floors save).
__device__ __forceinline__ bool pool_check_due(int64_t li) {
  return li < 32 ? (li == 0 || li == 1 || li == 3 || li == 7 || li == 15 || li == 31) : ((li & 31) == 31);
}

template <bool kI8, int kMode, int R, bool k2Sm, int kEpi>
__global__ void __launch_bounds__(64 + 32 * kEpi, 1)
    gemm_scan_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const ScanArgs a) {
  using G = Geo<k2Sm, cols_of(kMode)>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  constexpr int n_epi = kEpi;  // epilogue warps: 4, or 8 (two per TMEM lane quarter)
  const int n_stages = a.stages;
  uint8_t* stages = smem;
  float* s_cols = (float*)(smem + (size_t)n_stages * G::kStageBytes);  // [epilogue warps][kCols][256]
  uint32_t* stage_rows = (uint32_t*)(s_cols + n_epi * cols_of(kMode) * 256);  // [epilogue warps][32][36]
  uint64_t* full = (uint64_t*)(stage_rows + n_epi * 32 * kStageRowWords);
  uint64_t* empty = full + n_stages;
  uint64_t* tfull = empty + n_stages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = (uint32_t*)(tempty + 2);
  volatile int* abort_flag = (volatile int*)(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = k2Sm ? cluster_ctarank() : 0u;
  const bool leader = rank == 0;
  const int unit = k2Sm ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;  // work unit: cluster or CTA
  const int units = k2Sm ? (int)(gridDim.x >> 1) : (int)gridDim.x;
  const int64_t total = a.ntiles * (int64_t)a.num_mblocks;
  const int64_t p0 = total * unit / units;
  const int64_t p1 = total * (unit + 1) / units;

  if (threadIdx.x == 0) {
    for (int s = 0; s < n_stages; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], k2Sm ? 2 * n_epi : n_epi);  // the epilogue warps of every CTA of the MMA
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if (k2Sm) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if (k2Sm)
    cluster_sync();  // both CTAs' barriers are initialised before any remote arrive
  else
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
      const uint64_t pol_b = policy_evict_normal();
      const uint32_t full0 = k2Sm ? mapa_shared(smem_addr(&full[0]), 0) : smem_addr(&full[0]);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t used = 0;      // bit s: stage s has had a load issued
      uint32_t last_par = 0;  // bit s: parity of the last phase issued on stage s
      for (int64_t p = p0; p < p1 && !*abort_flag; p++) {
        int64_t nt;
        int mb;
        tile_of(p, a, nt, mb);
        const int32_t ya = mb * G::kQueriesPerTile + (int)rank * 128;
        const int32_t yb = (int32_t)(nt * BN) + (int)rank * G::kRowsB;
        for (int kc = 0; kc < a.kchunks; kc++) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, a.timeout_ns, abort_flag)) {
            give_up();
            break;
          }
          uint8_t* sa = stages + (size_t)stage * G::kStageBytes;
          const int x = kc * (kI8 ? 128 : 64);
          if (k2Sm) {
            // both CTAs' bytes complete on the leader's full barrier
            if (leader) mbar_arrive_expect_tx(&full[stage], G::kTxBytes);
            const uint32_t bar = full0 + (uint32_t)(stage * 8);
            tma_load_2d_pair(sa, &tmA, bar, x, ya, pol_a);
            tma_load_2d_pair(sa + G::kABytes, &tmB, bar, x, yb, pol_b);
          } else {
            mbar_arrive_expect_tx(&full[stage], G::kTxBytes);
            tma_load_2d_hint(sa, &tmA, &full[stage], x, ya, pol_a);
            tma_load_2d_hint(sa + G::kABytes, &tmB, &full[stage], x, yb, pol_b);
          }
          used |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (++stage == n_stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (*abort_flag && leader) {
        // Let every load already issued land before the cluster's shared memory is released.
        const uint64_t until = globaltimer_ns() + a.timeout_ns;
        for (;;) {
          bool all = true;
          for (int s = 0; s < n_stages; s++)
            if ((used >> s) & 1u)
              if (!mbar_try_wait(&full[s], (last_par >> s) & 1u)) all = false;
          if (all || globaltimer_ns() > until) break;
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      const uint32_t idesc = kI8 ? idesc_s8_s32(k2Sm ? 256 : 128, BN) : idesc_f16_f32(k2Sm ? 256 : 128, BN);
      int stage = 0;
      uint32_t phase = 0;
      int64_t t = 0;
      for (int64_t p = p0; p < p1 && !*abort_flag; p++, t++) {
        const int acc = (int)(t & 1);
        const uint32_t acc_phase = (uint32_t)((t >> 1) & 1);
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, a.timeout_ns, abort_flag)) {
          give_up();
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        bool ok = true;
        for (int kc = 0; kc < a.kchunks; kc++) {
          if (!mbar_wait(&full[stage], phase, a.timeout_ns, abort_flag)) {
            give_up();
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_addr(stages + (size_t)stage * G::kStageBytes);
          const uint64_t da = sw128_kmajor_desc(sa);
          const uint64_t db = sw128_kmajor_desc(sa + G::kABytes);
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const uint32_t accum = (kc | kk) != 0 ? 1u : 0u;
            if (k2Sm) {
              if (kI8)
                mma_i8_pair(d, da + 2ull * kk, db + 2ull * kk, idesc, accum);
              else
                mma_f16_pair(d, da + 2ull * kk, db + 2ull * kk, idesc, accum);
            } else {
              if (kI8)
                mma_i8(d, da + 2ull * kk, db + 2ull * kk, idesc, accum);
              else
                mma_f16(d, da + 2ull * kk, db + 2ull * kk, idesc, accum);
            }
          }
          if (k2Sm)
            mma_commit_pair_mc(&empty[stage], (uint16_t)0x3);
          else
            mma_commit(&empty[stage]);
          if (++stage == n_stages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (k2Sm)
          mma_commit_pair_mc(&tfull[acc], (uint16_t)0x3);
        else
          mma_commit(&tfull[acc]);
      }
    }
  } else {
    // ---------------- epilogue: warps 2.., one query (TMEM lane) per thread; with 8 epilogue
    // warps two share each TMEM lane quarter, warp 2 + i taking the first half of every tile's
    // columns and warp 6 + i the second, each with its own candidate stream per query
    const int quarter = warp & 3;
    const int halves = n_epi >> 2;
    const int half = (warp - 2) >> 2;
    const int gpw = (BN / 32) / halves;  // 32-column groups per warp
    const int g_lo = half * gpw;
    const int nstreams = units * halves;
    const int my_stream = unit * halves + half;
    const int row_in_block = (int)rank * 128 + quarter * 32 + lane;
    const int Qp = a.num_mblocks * G::kQueriesPerTile;
    const uint32_t tempty0 = k2Sm ? mapa_shared(smem_addr(&tempty[0]), 0) : smem_addr(&tempty[0]);
    float* s_col = s_cols + (warp - 2) * (cols_of(kMode) * 256);  // this warp's private column data
    float* s_col2 = s_col + 256;
    uint32_t* stage_row = stage_rows + (warp - 2) * (32 * kStageRowWords) + lane * kStageRowWords;
    const int64_t nt_first = p0 / a.num_mblocks;  // first row tile of this unit (row-major dealing)
    int64_t cols_nt = -1;                         // row tile whose column data s_col holds
    int64_t t = 0;
    for (int64_t p = p0; p < p1; p++, t++) {
      int64_t nt;
      int mb;
      tile_of(p, a, nt, mb);
      const int acc = (int)(t & 1);
      const uint32_t acc_phase = (uint32_t)((t >> 1) & 1);
      const int64_t col0 = nt * BN;
      // per-row column data: loaded when the row tile changes (a unit takes every query block
      // of a row tile in turn)
      if (kMode != kEpiF16Plain && kMode != kEpiBqHamming && nt != cols_nt) {
        cols_nt = nt;
        __syncwarp();
        for (int i = g_lo * 32 + lane; i < (g_lo + gpw) * 32; i += 32) {
          const int64_t row = col0 + i;
          const bool in = row < a.n;
          if (kMode == kEpiF16Scaled || kMode == kEpiF16L2) {
            s_col[i] = in ? a.epi.xnorm[row] : 0.0f;
            if (kMode == kEpiF16L2) s_col2[i] = in ? a.epi.rowsq[row] : 0.0f;
          } else if (kMode == kEpiSq8Dot || kMode == kEpiSq8Mip) {
            s_col[i] = in ? a.epi.vcorr[row] : 0.0f;
          } else if (epi_is_bbq(kMode)) {
            const float4 r = in ? a.epi.bbq_rows[row] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            s_col[i] = r.x;
            s_col[256 + i] = r.y;
            s_col[512 + i] = r.z;
            s_col[768 + i] = r.w;
          } else {  // kEpiSq8L2
            s_col[i] = __int_as_float(in ? a.epi.vsq[row] : 0);
          }
        }
        __syncwarp();
      }
      const int q = mb * G::kQueriesPerTile + row_in_block;
      const bool active = q < a.nq;
      const size_t sidx = (size_t)my_stream * Qp + (size_t)q;
      // Stream state does not depend on the accumulator: load it before waiting.
      const bool probe = a.probe != nullptr;
      const bool live = active && !probe;
      TileStream ts;
      ts.st.base = a.bufs + sidx * (size_t)a.C;
      ts.st.cnt = live ? a.cnts[sidx] : 0u;
      ts.st.thr = live ? a.thrs[sidx] : ~0ull;
      ts.t1 = (a.top1 && live) ? a.top1[sidx] : 0ull;
      ts.t2 = (a.top1 && live) ? a.top2[sidx] : 0ull;
      ts.dirty = false;
      ts.ceil = (a.ceil && live) ? a.ceil[q] : ~0ull;
      apply_floor(a, q, live, ts.st.thr);
      float qa = 0.0f;
      int32_t qi = 0;
      if (active) {
        if (kMode == kEpiF16L2) qa = 2.0f * a.epi.qscale[q];  // key = 2|q||x| acc - |x|^2
        if (kMode == kEpiSq8Dot || kMode == kEpiSq8Mip) qa = a.epi.qscale[q];
        if (kMode == kEpiSq8L2) qi = a.epi.qsq[q];
      }
      if (kMode == kEpiBqHamming) qi = a.epi.bits;
      float4 qb = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (epi_is_bbq(kMode) && active) {
        const BbqQuery b = a.epi.bbq_q[q];
        qb = make_float4(b.qmin, b.w15, (float)b.qsum, kMode == kEpiBbqL2 ? b.nsq : b.norm);
      }
      if (__shfl_sync(0xFFFFFFFFu, *abort_flag, 0)) break;
      {
        bool ok = mbar_wait(&tfull[acc], acc_phase, a.timeout_ns, abort_flag);
        ok = __all_sync(0xFFFFFFFFu, ok);
        if (!ok) {
          if (lane == 0) give_up();
          break;
        }
      }
      tc_fence_after();
      ts.tf = active ? thr_to_float(ts.st.thr) : INFINITY;
      const int64_t left = a.n - col0;
      const int valid = left < BN ? (int)left : BN;
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      // 32-column groups up to the last row (tile-uniform); the TMEM load of the next group is
      // in flight while the current one is processed
      const int g_end = (valid + 31) / 32 < g_lo + gpw ? (valid + 31) / 32 : g_lo + gpw;
      auto process = [&](uint32_t(&v)[32], int g) {
        const int c0 = g * 32;
        const float m = group_max<kMode>(v, c0, s_col, s_col2, qa, qi, a.epi, qb);
        if (probe) {  // exact group maxima: the floor needs scores that rows reach
          if (active) a.probe[(size_t)q * a.probe_groups + (size_t)((col0 + c0) >> 5)] = m;
          return;
        }
        if (__any_sync(0xFFFFFFFFu, m >= ts.tf))
          offer_group<kMode, R>(a, ts, q, active, v, c0, valid - c0, col0, qi, stage_row);
      };
      uint32_t va[32], vb[32];
      __syncwarp();
      if (g_lo < g_end) tmem_ld_32x32b_x32(taddr + (uint32_t)(g_lo * 32), va);
#pragma unroll 1
      for (int g = g_lo; g < g_end; g += 2) {
        __syncwarp();
        tmem_ld_wait_v(va);
        if (g + 1 < g_end) tmem_ld_32x32b_x32(taddr + (uint32_t)((g + 1) * 32), vb);
        process(va, g);
        if (g + 1 >= g_end) break;
        __syncwarp();
        tmem_ld_wait_v(vb);
        if (g + 2 < g_end) tmem_ld_32x32b_x32(taddr + (uint32_t)((g + 2) * 32), va);
        process(vb, g + 1);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (k2Sm)
          mbar_arrive_cluster(tempty0 + (uint32_t)(acc * 8));  // the leader issues the next MMA
        else
          mbar_arrive(&tempty[acc]);
      }
      if (live && ts.dirty) {  // a threshold raised only by the shared floor is not stored: the
        a.cnts[sidx] = ts.st.cnt;  // floor is applied again on the next load
        a.thrs[sidx] = ts.st.thr;
        if (a.top1) {
          a.top1[sidx] = ts.t1;
          a.top2[sidx] = ts.t2;
        }
      }
      // Pooled floor: propose this stream's j-th best key when enough streams of the query
      // match it (staggered: each unit checks every 32nd row tile).
      if (a.top1 && pool_check_due(nt - nt_first)) {
        const uint64_t mine = a.pool_j == 1 ? ts.t1 : ts.t2;
        const uint64_t* arr = a.pool_j == 1 ? a.top1 : a.top2;
        __syncwarp();
        int c = 0;
        for (int u = 0; u < nstreams; u++) c += __ldcg((const unsigned long long*)arr + (size_t)u * Qp + q) >= mine;
        if (active && mine != 0 && c >= a.pool_g)
          atomicMax((unsigned long long*)&a.floor[q], (unsigned long long)mine);
      }
    }
    // Leave every stream this CTA wrote with at most K keys.
    if (!a.probe && !__shfl_sync(0xFFFFFFFFu, *abort_flag, 0)) {
      for (int mb = 0; mb < a.num_mblocks; mb++) {
        const int q = mb * G::kQueriesPerTile + row_in_block;
        const bool active = q < a.nq;
        const size_t sidx = (size_t)my_stream * Qp + (size_t)q;
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
  if (k2Sm)
    cluster_sync();  // the pair's MMAs, loads and both epilogues are done with TMEM and smem
  else
    __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (k2Sm)
      tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else
      tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// Shared memory of one CTA with `stages` ring stages and `epi` epilogue warps.
template <bool k2Sm, int kCols>
constexpr size_t scan_smem(int stages, int epi) {
  return 1024 + (size_t)stages * Geo<k2Sm, kCols>::kStageBytes + (size_t)epi * kCols * 256 * sizeof(float) +
         (size_t)epi * 32 * kStageRowWords * sizeof(uint32_t) + 256;
}

template <bool kI8, int kMode, int R, bool k2Sm, int kEpi>
cudaError_t launch_one(const CUtensorMap& tmA, const CUtensorMap& tmB, const ScanArgs& args, int grid,
                       cudaStream_t st) {
  auto kern = gemm_scan_kernel<kI8, kMode, R, k2Sm, kEpi>;
  using G = Geo<k2Sm, cols_of(kMode)>;
  ScanArgs a = args;
  // the deepest ring that fits next to the epilogue warps' staging (at most the 4-warp depth)
  a.stages = G::kStages;
  while (a.stages > 2 && scan_smem<k2Sm, cols_of(kMode)>(a.stages, kEpi) > 232448) a.stages--;
  const size_t smem = scan_smem<k2Sm, cols_of(kMode)>(a.stages, kEpi);
  const int threads = 64 + 32 * kEpi;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  if (!k2Sm) {
    kern<<<grid, threads, smem, st>>>(tmA, tmB, a);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tmA, tmB, a);
}

template <bool kI8, int kMode, bool k2Sm>
cudaError_t launch_mode(const CUtensorMap& tmA, const CUtensorMap& tmB, const ScanArgs& a, int grid,
                        int R, cudaStream_t st) {
  if (a.epi_warps == 8) {
    // built only where gemm_scan_epi8 says so: fp16 scans with 17-row streams (the 320-thread
    // block leaves 168 registers a thread, enough for R = 17 with 16-36 spilled bytes)
    if constexpr (!kI8) {
      if (R == 17) return launch_one<kI8, kMode, 17, k2Sm, 8>(tmA, tmB, a, grid, st);
    }
    return cudaErrorInvalidValue;
  }
  if (a.epi_warps != 4) return cudaErrorInvalidValue;
  switch (R) {
    case 3: return launch_one<kI8, kMode, 3, k2Sm, 4>(tmA, tmB, a, grid, st);
    case 5: return launch_one<kI8, kMode, 5, k2Sm, 4>(tmA, tmB, a, grid, st);
    case 9: return launch_one<kI8, kMode, 9, k2Sm, 4>(tmA, tmB, a, grid, st);
    case 17: return launch_one<kI8, kMode, 17, k2Sm, 4>(tmA, tmB, a, grid, st);
    case 33: return launch_one<kI8, kMode, 33, k2Sm, 4>(tmA, tmB, a, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

template <bool k2Sm>
cudaError_t launch_variant(int mode, const CUtensorMap& tmA, const CUtensorMap& tmB, const ScanArgs& a,
                           int grid, int R, cudaStream_t st) {
  switch (mode) {
    case kEpiF16Plain: return launch_mode<false, kEpiF16Plain, k2Sm>(tmA, tmB, a, grid, R, st);
    case kEpiF16Scaled: return launch_mode<false, kEpiF16Scaled, k2Sm>(tmA, tmB, a, grid, R, st);
    case kEpiF16L2: return launch_mode<false, kEpiF16L2, k2Sm>(tmA, tmB, a, grid, R, st);
    case kEpiSq8Dot: return launch_mode<true, kEpiSq8Dot, k2Sm>(tmA, tmB, a, grid, R, st);
    case kEpiSq8Mip: return launch_mode<true, kEpiSq8Mip, k2Sm>(tmA, tmB, a, grid, R, st);
    case kEpiSq8L2: return launch_mode<true, kEpiSq8L2, k2Sm>(tmA, tmB, a, grid, R, st);
    case kEpiBqHamming: return launch_mode<true, kEpiBqHamming, k2Sm>(tmA, tmB, a, grid, R, st);
    case kEpiBbqDot: return launch_mode<true, kEpiBbqDot, k2Sm>(tmA, tmB, a, grid, R, st);
    case kEpiBbqMip: return launch_mode<true, kEpiBbqMip, k2Sm>(tmA, tmB, a, grid, R, st);
    case kEpiBbqL2: return launch_mode<true, kEpiBbqL2, k2Sm>(tmA, tmB, a, grid, R, st);
    case kEpiBbqCos: return launch_mode<true, kEpiBbqCos, k2Sm>(tmA, tmB, a, grid, R, st);
    default: return cudaErrorInvalidValue;
  }
}

// The pipeline's bounded wait with nothing to wait for: one thread waits on an mbarrier that no
// thread arrives on, gives up after timeout_ns (mbar_wait), records kDevWaitTimeout and the
// kernel returns -- the give-up path of the scan's waits without the scan around it.
__global__ void wait_probe_kernel(uint64_t timeout_ns, int32_t* err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait(&bar, 0, timeout_ns, &abort_flag)) {
    abort_flag = 1;
    record_error(err, kDevWaitTimeout);
  }
  __syncthreads();
}

}  // namespace

cudaError_t launch_wait_probe(uint64_t timeout_ns, int32_t* err, cudaStream_t st) {
  wait_probe_kernel<<<1, 32, 0, st>>>(timeout_ns, err);
  return cudaGetLastError();
}

int gemm_scan_units(int64_t ntiles, int num_mblocks, int num_sms, bool two_sm) {
  const int64_t total = ntiles * (int64_t)num_mblocks;
  int64_t u = two_sm ? num_sms / 2 : num_sms;
  if (u > total) u = total;
  return (int)(u < 1 ? 1 : u);
}

bool gemm_scan_epi8(int mode, int R) {
  return (mode == kEpiF16Plain || mode == kEpiF16Scaled || mode == kEpiF16L2) && R == 17;
}

int gemm_scan_stream_R(int K) {
  StreamGeom g = stream_geom(K, 32);  // at most 32 appends between overflow checks
  return g.R == 2 ? 3 : g.R;          // the GEMM scan instantiates R in {3,5,9,17,33}
}

cudaError_t launch_gemm_scan(int mode, const CUtensorMap& tmA, const CUtensorMap& tmB,
                             const ScanArgs& a, int units, int R, bool two_sm, cudaStream_t st) {
  return two_sm ? launch_variant<true>(mode, tmA, tmB, a, 2 * units, R, st)
                : launch_variant<false>(mode, tmA, tmB, a, units, R, st);
}

}  // namespace vx
