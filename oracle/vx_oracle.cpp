// vx_oracle.cpp -- CPU restatement of the integrallis/vectors hot path.
//
// TEST INFRASTRUCTURE ONLY (see vx_oracle.h).  Built with -ffp-contract=off so that
// every a*b+c the Java source writes as two operations stays two roundings; std::fma
// appears exactly where the Java code calls Math.fma or FloatVector.fma.
#include "vx_oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <functional>
#include <limits>
#include <numeric>
#include <thread>
#include <vector>

namespace {

constexpr int kLanes = 8;  // FLOAT_SPECIES at the 256-bit cap (PanamaConstants.java:47)

// Runs fn(lo, hi) over [0, n) split into nthreads contiguous chunks.
void parallel_for(int64_t n, int nthreads, const std::function<void(int64_t, int64_t)>& fn) {
  if (nthreads <= 1 || n < 2) {
    fn(0, n);
    return;
  }
  int t = (int)std::min<int64_t>(nthreads, n);
  std::vector<std::thread> pool;
  pool.reserve(t);
  for (int i = 0; i < t; i++) {
    int64_t lo = n * i / t, hi = n * (i + 1) / t;
    pool.emplace_back([=, &fn] { fn(lo, hi); });
  }
  for (auto& th : pool) th.join();
}

// FloatVector lane sum in the explicit order of PanamaVectorUtilSupport.reduceAdd
// (PanamaVectorUtilSupport.java:1377-1386, 8-lane case).  Also used for reduceLanes(ADD),
// whose JVM order is unspecified.
inline float reduce_add8(const float* l) {
  float even = (l[4] + l[0]) + (l[6] + l[2]);
  float odd = (l[5] + l[1]) + (l[7] + l[3]);
  return even + odd;
}

// dotProductBody (PanamaVectorUtilSupport.java:227-271).
float dot_body(const float* a, const float* b, int limit) {
  float acc1[kLanes] = {0}, acc2[kLanes] = {0}, acc3[kLanes] = {0}, acc4[kLanes] = {0};
  int unrolled = limit - 3 * kLanes;
  int i = 0;
  for (; i < unrolled; i += 4 * kLanes) {
    for (int j = 0; j < kLanes; j++) acc1[j] = std::fma(a[i + j], b[i + j], acc1[j]);
    for (int j = 0; j < kLanes; j++) acc2[j] = std::fma(a[i + 8 + j], b[i + 8 + j], acc2[j]);
    for (int j = 0; j < kLanes; j++) acc3[j] = std::fma(a[i + 16 + j], b[i + 16 + j], acc3[j]);
    for (int j = 0; j < kLanes; j++) acc4[j] = std::fma(a[i + 24 + j], b[i + 24 + j], acc4[j]);
  }
  for (; i < limit; i += kLanes)
    for (int j = 0; j < kLanes; j++) acc1[j] = std::fma(a[i + j], b[i + j], acc1[j]);
  float s[kLanes];
  for (int j = 0; j < kLanes; j++) s[j] = (acc1[j] + acc2[j]) + (acc3[j] + acc4[j]);
  return reduce_add8(s);
}

// squareDistanceBody (PanamaVectorUtilSupport.java:299-343).
float sqdist_body(const float* a, const float* b, int limit) {
  float acc1[kLanes] = {0}, acc2[kLanes] = {0}, acc3[kLanes] = {0}, acc4[kLanes] = {0};
  int unrolled = limit - 3 * kLanes;
  int i = 0;
  for (; i < unrolled; i += 4 * kLanes) {
    for (int j = 0; j < kLanes; j++) {
      float d = a[i + j] - b[i + j];
      acc1[j] = std::fma(d, d, acc1[j]);
    }
    for (int j = 0; j < kLanes; j++) {
      float d = a[i + 8 + j] - b[i + 8 + j];
      acc2[j] = std::fma(d, d, acc2[j]);
    }
    for (int j = 0; j < kLanes; j++) {
      float d = a[i + 16 + j] - b[i + 16 + j];
      acc3[j] = std::fma(d, d, acc3[j]);
    }
    for (int j = 0; j < kLanes; j++) {
      float d = a[i + 24 + j] - b[i + 24 + j];
      acc4[j] = std::fma(d, d, acc4[j]);
    }
  }
  for (; i < limit; i += kLanes)
    for (int j = 0; j < kLanes; j++) {
      float d = a[i + j] - b[i + j];
      acc1[j] = std::fma(d, d, acc1[j]);
    }
  float s[kLanes];
  for (int j = 0; j < kLanes; j++) s[j] = (acc1[j] + acc2[j]) + (acc3[j] + acc4[j]);
  return reduce_add8(s);
}

inline float transform(int metric, float raw) {
  switch (metric) {
    case VO_EUCLIDEAN: return 1.0f / (1.0f + raw);      // SimilarityFunction.java:39
    case VO_DOT_PRODUCT: return (1.0f + raw) / 2.0f;    // SimilarityFunction.java:60
    case VO_COSINE: return (1.0f + raw) / 2.0f;         // SimilarityFunction.java:83
    default: return vo_scale_mip(raw);                  // SimilarityFunction.java:105-106
  }
}

// Java Math.round(float): nearest int, ties toward +infinity, NaN -> 0.
inline int32_t java_round(float x) {
  if (std::isnan(x)) return 0;
  float f = std::floor(x);
  float diff = x - f;  // exact for |x| < 2^23
  double r = (diff >= 0.5f) ? (double)f + 1.0 : (double)f;
  if (r >= 2147483647.0) return INT32_MAX;
  if (r <= -2147483648.0) return INT32_MIN;
  return (int32_t)r;
}

inline float java_max(float a, float b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<float>::quiet_NaN();
  if (a == 0.0f && b == 0.0f) return std::signbit(a) ? b : a;
  return a >= b ? a : b;
}
inline float java_min(float a, float b) {
  if (std::isnan(a) || std::isnan(b)) return std::numeric_limits<float>::quiet_NaN();
  if (a == 0.0f && b == 0.0f) return std::signbit(a) ? a : b;
  return a <= b ? a : b;
}

// ---------------------------------------------------------------- top-k policies
// Reference bounded min-heap: FlatScanAdapter.java:72-95,193-232 (identical in
// QuantizedFlatScanAdapter.java:139-176 and, with <= rejection, TopKHeap.java:60-95).
struct RefHeap {
  std::vector<int32_t> ids;
  std::vector<float> sc;
  int size = 0, cap = 0;
  explicit RefHeap(int c) : ids(c), sc(c), cap(c) {}
  void sift_up(int idx) {
    while (idx > 0) {
      int p = (idx - 1) >> 1;
      if (sc[p] <= sc[idx]) break;
      std::swap(sc[p], sc[idx]);
      std::swap(ids[p], ids[idx]);
      idx = p;
    }
  }
  void sift_down(int idx, int n) {
    for (;;) {
      int l = 2 * idx + 1, r = l + 1, s = idx;
      if (l < n && sc[l] < sc[s]) s = l;
      if (r < n && sc[r] < sc[s]) s = r;
      if (s == idx) break;
      std::swap(sc[s], sc[idx]);
      std::swap(ids[s], ids[idx]);
      idx = s;
    }
  }
  void offer(int32_t id, float s) {
    if (size < cap) {
      ids[size] = id;
      sc[size] = s;
      size++;
      sift_up(size - 1);
    } else if (s > sc[0]) {
      ids[0] = id;
      sc[0] = s;
      sift_down(0, size);
    }
  }
  // drain into descending order (FlatScanAdapter.java:86-95)
  int drain(int32_t* out_ids, float* out_sc) {
    int n = size;
    for (int i = n - 1; i >= 0; i--) {
      out_ids[i] = ids[0];
      out_sc[i] = sc[0];
      ids[0] = ids[i];
      sc[0] = sc[i];
      sift_down(0, i);
    }
    return n;
  }
};

// Canonical order (score desc, id asc), TopK.java:96-116; NaN never admitted.
struct CanonTopK {
  std::vector<std::pair<float, int32_t>> v;  // kept as a heap, worst at front
  int cap;
  explicit CanonTopK(int c) : cap(c) { v.reserve(c); }
  static bool better(const std::pair<float, int32_t>& a, const std::pair<float, int32_t>& b) {
    if (a.first != b.first) return a.first > b.first;
    return a.second < b.second;
  }
  void offer(int32_t id, float s) {
    if (std::isnan(s)) return;
    std::pair<float, int32_t> e{s, id};
    auto cmp = [](const std::pair<float, int32_t>& a, const std::pair<float, int32_t>& b) {
      return better(a, b);
    };
    if ((int)v.size() < cap) {
      v.push_back(e);
      std::push_heap(v.begin(), v.end(), cmp);
    } else if (better(e, v.front())) {
      std::pop_heap(v.begin(), v.end(), cmp);
      v.back() = e;
      std::push_heap(v.begin(), v.end(), cmp);
    }
  }
  int drain(int32_t* out_ids, float* out_sc) {
    std::sort(v.begin(), v.end(), better);
    for (size_t i = 0; i < v.size(); i++) {
      out_ids[i] = v[i].second;
      out_sc[i] = v[i].first;
    }
    return (int)v.size();
  }
};

// Runs a per-query scan with the chosen policy; score(q, row) supplies the value.
template <class ScoreFn>
void scan_topk(int64_t n, int32_t nq, int32_t k, int32_t policy, int32_t nthreads, ScoreFn score,
               int32_t* ids, float* scores, int32_t* counts) {
  int kk = (int)std::min<int64_t>(k, n);
  parallel_for(nq, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t q = lo; q < hi; q++) {
      int32_t* oi = ids + q * k;
      float* os = scores + q * k;
      if (kk <= 0) {
        counts[q] = 0;
        continue;
      }
      if (policy == VO_POLICY_REFERENCE_HEAP) {
        RefHeap h(kk);
        for (int64_t r = 0; r < n; r++) h.offer((int32_t)r, score(q, r));
        counts[q] = h.drain(oi, os);
      } else {
        CanonTopK h(kk);
        for (int64_t r = 0; r < n; r++) h.offer((int32_t)r, score(q, r));
        counts[q] = h.drain(oi, os);
      }
    }
  });
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------- java.util.Random
static const uint64_t kMult = 0x5DEECE66DULL, kMask = (1ULL << 48) - 1;
void vo_jrandom_init(vo_jrandom* r, int64_t seed) {
  r->seed = ((uint64_t)seed ^ kMult) & kMask;
  r->have_next_next_gaussian = 0;
  r->next_next_gaussian = 0;
}
static int32_t jr_next(vo_jrandom* r, int bits) {
  r->seed = (r->seed * kMult + 0xBULL) & kMask;
  return (int32_t)(int64_t)(r->seed >> (48 - bits));
}
int32_t vo_jrandom_next_int(vo_jrandom* r) { return jr_next(r, 32); }
int32_t vo_jrandom_next_int_bound(vo_jrandom* r, int32_t bound) {
  if ((bound & -bound) == bound) return (int32_t)(((int64_t)bound * (int64_t)jr_next(r, 31)) >> 31);
  int32_t bits, val;
  do {
    bits = jr_next(r, 31);
    val = bits % bound;
  } while ((int32_t)((uint32_t)bits - (uint32_t)val + (uint32_t)(bound - 1)) < 0);
  return val;
}
int64_t vo_jrandom_next_long(vo_jrandom* r) {
  int64_t hi = (int64_t)jr_next(r, 32);
  int64_t lo = (int64_t)jr_next(r, 32);
  return (int64_t)((uint64_t)hi << 32) + lo;
}
float vo_jrandom_next_float(vo_jrandom* r) { return jr_next(r, 24) / (float)(1 << 24); }
double vo_jrandom_next_double(vo_jrandom* r) {
  int64_t a = jr_next(r, 26), b = jr_next(r, 27);
  return (double)((a << 27) + b) * 0x1.0p-53;
}
void vo_jrandom_next_bytes(vo_jrandom* r, int8_t* out, int32_t n) {
  for (int32_t i = 0; i < n;) {
    int32_t rnd = vo_jrandom_next_int(r);
    for (int m = std::min(n - i, 4); m-- > 0; rnd >>= 8) out[i++] = (int8_t)rnd;
  }
}

// ---------------------------------------------------------------- synthetic data
uint64_t vo_splitmix64_at(uint64_t seed, uint64_t index) {
  uint64_t z = seed + (index + 1) * 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}
double vo_uniform_at(uint64_t seed, uint64_t index) {
  return (double)(vo_splitmix64_at(seed, index) >> 11) * 0x1.0p-53;
}
double vo_normal_at(uint64_t seed, uint64_t index) {
  double u1 = 1.0 - vo_uniform_at(seed, 2 * index);  // (0, 1]
  double u2 = vo_uniform_at(seed, 2 * index + 1);
  return std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2);
}
void vo_gen_mixture(float* out, int64_t first_row, int64_t n, int32_t dim, int32_t n_centres,
                    float sigma, uint64_t seed_centres, uint64_t seed_points, int32_t normalize,
                    int32_t nthreads) {
  std::vector<float> centres((size_t)n_centres * dim);
  for (int64_t i = 0; i < (int64_t)centres.size(); i++)
    centres[i] = (float)vo_normal_at(seed_centres, (uint64_t)i);
  const uint64_t comp_seed = seed_points ^ 0xA5A5A5A5A5A5A5A5ULL;
  parallel_for(n, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t r = lo; r < hi; r++) {
      int64_t row = first_row + r;
      int32_t c = (int32_t)(vo_uniform_at(comp_seed, (uint64_t)row) * n_centres);
      if (c >= n_centres) c = n_centres - 1;
      float* o = out + r * dim;
      const float* ce = centres.data() + (size_t)c * dim;
      for (int d = 0; d < dim; d++)
        o[d] = (float)((double)ce[d] +
                       (double)sigma * vo_normal_at(seed_points, (uint64_t)row * dim + d));
      if (normalize) vo_l2normalize(o, dim);
    }
  });
}

// ---------------------------------------------------------------- L0 kernels
// dotProduct(float[],int,float[],int,int): PanamaVectorUtilSupport.java:208-225.
float vo_dot(const float* a, const float* b, int32_t len) {
  int i = 0;
  float res = 0.0f;
  if (len > 2 * kLanes) {
    int limit = len & ~(kLanes - 1);
    res += dot_body(a, b, limit);
    i = limit;
  }
  for (; i < len; i++) res = std::fma(a[i], b[i], res);
  return res;
}
// squareDistance: PanamaVectorUtilSupport.java:280-297 (scalar tail: two roundings, no FMA).
float vo_square_distance(const float* a, const float* b, int32_t len) {
  int i = 0;
  float res = 0.0f;
  if (len > 2 * kLanes) {
    int limit = len & ~(kLanes - 1);
    res += sqdist_body(a, b, limit);
    i = limit;
  }
  for (; i < len; i++) {
    float diff = a[i] - b[i];
    res += diff * diff;
  }
  return res;
}
// cosine: PanamaVectorUtilSupport.java:347-456.
float vo_cosine(const float* a, const float* b, int32_t len) {
  int i = 0;
  float sum = 0.0f, n1 = 0.0f, n2 = 0.0f;
  if (len >= 4 * kLanes) {
    int limit = len & ~(kLanes - 1);
    float s[4][kLanes] = {{0}}, x[4][kLanes] = {{0}}, y[4][kLanes] = {{0}};
    int unrolled = limit - 3 * kLanes;
    int p = 0;
    for (; p < unrolled; p += 4 * kLanes)
      for (int u = 0; u < 4; u++)
        for (int j = 0; j < kLanes; j++) {
          float va = a[p + u * kLanes + j], vb = b[p + u * kLanes + j];
          s[u][j] = std::fma(va, vb, s[u][j]);
          x[u][j] = std::fma(va, va, x[u][j]);
          y[u][j] = std::fma(vb, vb, y[u][j]);
        }
    for (; p < limit; p += kLanes)
      for (int j = 0; j < kLanes; j++) {
        float va = a[p + j], vb = b[p + j];
        s[0][j] = std::fma(va, vb, s[0][j]);
        x[0][j] = std::fma(va, va, x[0][j]);
        y[0][j] = std::fma(vb, vb, y[0][j]);
      }
    float rs[kLanes], rx[kLanes], ry[kLanes];
    for (int j = 0; j < kLanes; j++) {
      rs[j] = (s[0][j] + s[1][j]) + (s[2][j] + s[3][j]);
      rx[j] = (x[0][j] + x[1][j]) + (x[2][j] + x[3][j]);
      ry[j] = (y[0][j] + y[1][j]) + (y[2][j] + y[3][j]);
    }
    sum = reduce_add8(rs);
    n1 = reduce_add8(rx);
    n2 = reduce_add8(ry);
    i = limit;
  } else if (len >= kLanes) {
    int limit = len & ~(kLanes - 1);
    float s[kLanes] = {0}, x[kLanes] = {0}, y[kLanes] = {0};
    for (int p = 0; p < limit; p += kLanes)
      for (int j = 0; j < kLanes; j++) {
        s[j] = std::fma(a[p + j], b[p + j], s[j]);
        x[j] = std::fma(a[p + j], a[p + j], x[j]);
        y[j] = std::fma(b[p + j], b[p + j], y[j]);
      }
    sum = reduce_add8(s);
    n1 = reduce_add8(x);
    n2 = reduce_add8(y);
    i = limit;
  }
  for (; i < len; i++) {
    sum = std::fma(a[i], b[i], sum);
    n1 = std::fma(a[i], a[i], n1);
    n2 = std::fma(b[i], b[i], n2);
  }
  return (float)((double)sum / std::sqrt((double)n1 * (double)n2));
}
float vo_scale_mip(float dot) {  // SimilarityFunction.java:155-161
  if (dot >= 0) return dot + 1.0f;
  return 1.0f / (1.0f - dot);
}
float vo_compare(int32_t metric, const float* a, const float* b, int32_t len) {
  switch (metric) {
    case VO_EUCLIDEAN: return transform(metric, vo_square_distance(a, b, len));
    case VO_COSINE: return transform(metric, vo_cosine(a, b, len));
    default: return transform(metric, vo_dot(a, b, len));
  }
}
// l2normalize: PanamaVectorUtilSupport.java:5178-5230, MathUtil.java:33-35.
void vo_l2normalize(float* v, int32_t len) {
  double sq = (double)vo_dot(v, v, len);
  if (sq == 0.0) return;
  if (std::fabs((float)sq - 1.0f) < 1e-5f) return;
  float inv = 1.0f / (float)std::sqrt(sq);
  for (int i = 0; i < len; i++) v[i] *= inv;
}
int32_t vo_byte_dot(const int8_t* a, const int8_t* b, int32_t len) {
  int32_t s = 0;
  for (int i = 0; i < len; i++) s += (int32_t)a[i] * (int32_t)b[i];
  return s;
}
int32_t vo_byte_square_distance(const int8_t* a, const int8_t* b, int32_t len) {
  int32_t s = 0;
  for (int i = 0; i < len; i++) {
    int32_t d = (int32_t)a[i] - (int32_t)b[i];
    s += d * d;
  }
  return s;
}
int32_t vo_hamming(const uint64_t* a, const uint64_t* b, int32_t nwords) {
  int32_t h = 0;
  for (int i = 0; i < nwords; i++) h += __builtin_popcountll(a[i] ^ b[i]);
  return h;
}
// matVecSquaredL2: PanamaVectorUtilSupport.java:5547-5598 (rows in groups of 4 use one
// 8-lane accumulator each; the last nrows % 4 rows use squareDistance).
void vo_mat_vec_square_l2(const float* q, const float* rows, int32_t nrows, int32_t dim,
                          float* out) {
  int group = nrows & ~3;
  int limit = dim & ~(kLanes - 1);
  for (int r = 0; r < group; r++) {
    const float* row = rows + (size_t)r * dim;
    float acc[kLanes] = {0};
    for (int i = 0; i < limit; i += kLanes)
      for (int j = 0; j < kLanes; j++) {
        float d = q[i + j] - row[i + j];
        acc[j] = std::fma(d, d, acc[j]);
      }
    float s = reduce_add8(acc);
    for (int i = limit; i < dim; i++) {
      float e = q[i] - row[i];
      s = std::fma(e, e, s);
    }
    out[r] = s;
  }
  for (int r = group; r < nrows; r++) out[r] = vo_square_distance(q, rows + (size_t)r * dim, dim);
}
// matVecDot: PanamaVectorUtilSupport.java:5353-5397.
void vo_mat_vec_dot(const float* q, const float* rows, int32_t nrows, int32_t dim, float* out) {
  int group = nrows & ~3;
  int limit = dim & ~(kLanes - 1);
  for (int r = 0; r < group; r++) {
    const float* row = rows + (size_t)r * dim;
    float acc[kLanes] = {0};
    for (int i = 0; i < limit; i += kLanes)
      for (int j = 0; j < kLanes; j++) acc[j] = std::fma(q[i + j], row[i + j], acc[j]);
    float s = reduce_add8(acc);
    for (int i = limit; i < dim; i++) s = std::fma(q[i], row[i], s);
    out[r] = s;
  }
  for (int r = group; r < nrows; r++) out[r] = vo_dot(q, rows + (size_t)r * dim, dim);
}

// ---------------------------------------------------------------- SQ8
// ReservoirSampler.sampleIndices (ReservoirSampler.java:43-61).
static std::vector<int32_t> reservoir(int64_t n, int32_t max_samples, int64_t seed) {
  int32_t s = (int32_t)std::min<int64_t>(n, max_samples);
  std::vector<int32_t> idx(s);
  for (int32_t i = 0; i < s; i++) idx[i] = i;
  vo_jrandom r;
  vo_jrandom_init(&r, seed);
  for (int64_t i = s; i < n; i++) {
    int32_t j = vo_jrandom_next_int_bound(&r, (int32_t)(i + 1));
    if (j < s) idx[j] = (int32_t)i;
  }
  return idx;
}
// ScalarQuantizer.computeQuantiles (ScalarQuantizer.java:362-409, 451-456).
void vo_sq8_train(const float* data, int64_t n, int32_t dim, float ci, float* min_q,
                  float* max_q) {
  std::vector<int32_t> idx = reservoir(n, 25000, 42);
  auto degenerate = [&](float v) {
    float a = std::fabs(v);
    float eps = a > 0 ? a * 1e-6f : 1e-6f;
    *min_q = v - eps;
    *max_q = v + eps;
  };
  if (ci >= 1.0f) {
    float mn = INFINITY, mx = -INFINITY;
    for (int32_t r : idx)
      for (int d = 0; d < dim; d++) {
        float v = data[(int64_t)r * dim + d];
        if (v < mn) mn = v;
        if (v > mx) mx = v;
      }
    if (mn == mx) return degenerate(mn);
    *min_q = mn;
    *max_q = mx;
    return;
  }
  std::vector<float> all((size_t)idx.size() * dim);
  for (size_t i = 0; i < idx.size(); i++)
    std::memcpy(&all[i * dim], data + (int64_t)idx[i] * dim, sizeof(float) * dim);
  int64_t len = (int64_t)all.size();
  int32_t sel = (int32_t)((float)len * (1.0f - ci) / 2.0f + 0.5f);
  sel = (int32_t)std::max<int64_t>(0, std::min<int64_t>(sel, len - 1));
  int64_t maxi = len - 1 - sel;
  // quickSelect returns the order statistic, independent of the array's prior order.
  std::nth_element(all.begin(), all.begin() + sel, all.end());
  float lo = all[sel];
  std::nth_element(all.begin(), all.begin() + maxi, all.end());
  float hi = all[maxi];
  if (lo == hi) return degenerate(lo);
  *min_q = lo;
  *max_q = hi;
}
struct Sq8Params {
  float min_q, max_q, scale, alpha, cm;
  int max_value;
};
// ScalarQuantizer constructor (ScalarQuantizer.java:59-69): maxValue 127 for INT8, 15 for INT4
// (ScalarBits.java:30-33).
static Sq8Params sq8_params(float min_q, float max_q, int max_value = 127) {
  Sq8Params p;
  p.min_q = min_q;
  p.max_q = max_q;
  p.max_value = max_value;
  float range = max_q - min_q;
  p.scale = (range == 0.0f) ? 0.0f : (float)max_value / range;
  p.alpha = (range == 0.0f) ? 0.0f : range / (float)max_value;
  p.cm = p.alpha * p.alpha;
  return p;
}
// encodeInt8 / encodeInt4Unpacked / quantizeValue / correctionTerm (ScalarQuantizer.java:243-272,
// 343-351): one code per byte (0..maxValue).
float vo_sq_encode(float min_q, float max_q, int32_t max_value, const float* v, int32_t dim, int8_t* dst) {
  Sq8Params p = sq8_params(min_q, max_q, max_value);
  float corr = 0.0f;
  for (int i = 0; i < dim; i++) {
    float dxc = java_max(p.min_q, java_min(p.max_q, v[i])) - p.min_q;
    int32_t q = java_round(p.scale * dxc);
    q = std::max(0, std::min(p.max_value, q));
    dst[i] = (int8_t)q;
    float dx = v[i] - p.min_q;
    float dxq = (float)q * p.alpha;
    float half = p.min_q / 2.0f;
    float t1 = p.min_q * (v[i] - half);
    float t2 = (dx - dxq) * dxq;
    corr += t1 + t2;
  }
  return corr;
}
float vo_sq8_encode(float min_q, float max_q, const float* v, int32_t dim, int8_t* dst) {
  return vo_sq_encode(min_q, max_q, 127, v, dim, dst);
}
// scoreFunctionInt8 / scoreFunctionInt4 (ScalarQuantizedVectors.java:82-140): the INT4 codes
// unpacked one per byte, the same formulas with the INT4 constants.
float vo_sq_score(int32_t metric, float min_q, float max_q, int32_t max_value, const int8_t* qc, float qcorr,
                  const int8_t* vc, float vcorr, int32_t dim) {
  Sq8Params p = sq8_params(min_q, max_q, max_value);
  if (metric == VO_EUCLIDEAN) {
    int32_t sq = vo_byte_square_distance(qc, vc, dim);
    float adj = (float)sq * p.cm;
    return 1.0f / (1.0f + adj);
  }
  int32_t raw = vo_byte_dot(qc, vc, dim);
  float adj = (float)raw * p.cm + qcorr + vcorr;
  if (metric == VO_MAXIMUM_INNER_PRODUCT) return vo_scale_mip(adj);
  return java_max((1.0f + adj) / 2.0f, 0.0f);
}
float vo_sq8_score(int32_t metric, float min_q, float max_q, const int8_t* qc, float qcorr,
                   const int8_t* vc, float vcorr, int32_t dim) {
  return vo_sq_score(metric, min_q, max_q, 127, qc, qcorr, vc, vcorr, dim);
}

// ---------------------------------------------------------------- BQ (sign bit)
// packBits + bytesToLongs (BinaryQuantizer.java:207-232): bit d of the vector is
// bit (d & 63) of word (d >> 6), set when v >= 0.
void vo_bq_encode(const float* v, int32_t dim, uint64_t* words) {
  int nw = (dim + 63) >> 6;
  for (int w = 0; w < nw; w++) words[w] = 0;
  for (int d = 0; d < dim; d++)
    if (v[d] >= 0) words[d >> 6] |= 1ULL << (d & 63);
}
// signBitScoreFunction (BinaryQuantizedVectors.java:81-107).
float vo_bq_score(int32_t metric, int32_t h, int32_t dim) {
  switch (metric) {
    case VO_EUCLIDEAN: return 1.0f / (1.0f + 4.0f * (float)h);
    case VO_MAXIMUM_INNER_PRODUCT: return vo_scale_mip((float)(dim - 2 * h) / (float)dim);
    default: return 1.0f - (float)h / (float)dim;
  }
}

// ---------------------------------------------------------------- FP16
// Float.floatToFloat16: round to nearest even (Fp16Quantizer.java:72-85).
uint16_t vo_f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7FFFFFFFu;
  if (ax >= 0x7F800000u) {  // Inf / NaN
    if (ax == 0x7F800000u) return (uint16_t)(sign | 0x7C00u);
    return (uint16_t)(sign | 0x7C00u | 0x200u | ((ax >> 13) & 0x3FFu));
  }
  if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to >= 65520 -> Inf
  if (ax < 0x38800000u) {                                      // result subnormal or zero
    if (ax < 0x33000000u) return (uint16_t)sign;               // < 2^-25 -> 0
    uint32_t mant = (ax & 0x7FFFFFu) | 0x800000u;
    int e = (int)(ax >> 23);  // 102..112
    int shift = 126 - e;      // 14..24
    uint32_t half = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1);
    uint32_t mid = 1u << (shift - 1);
    if (rem > mid || (rem == mid && (half & 1u))) half++;
    return (uint16_t)(sign | half);
  }
  uint32_t e = (ax >> 23) - 112;
  uint32_t mant = ax & 0x7FFFFFu;
  uint32_t h = (e << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}
float vo_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else {
      float v = (float)m * 0x1.0p-24f;
      std::memcpy(&x, &v, 4);
      x |= sign;
    }
  } else if (e == 31) {
    x = sign | 0x7F800000u | (m << 13);
  } else {
    x = sign | ((e + 112) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &x, 4);
  return f;
}

// ---------------------------------------------------------------- PQ
// computeSubspaceSizesAndOffsets (ProductQuantizer.java:686-700).
void vo_pq_subspaces(int32_t dim, int32_t m, int32_t* so) {
  int base = dim / m, rem = dim % m, off = 0;
  for (int i = 0; i < m; i++) {
    int size = base + (i < rem ? 1 : 0);
    so[2 * i] = size;
    so[2 * i + 1] = off;
    off += size;
  }
}
static std::vector<int64_t> codebook_offsets(int32_t dim, int32_t m, int32_t ks,
                                             std::vector<int32_t>& so) {
  so.assign(2 * m, 0);
  vo_pq_subspaces(dim, m, so.data());
  std::vector<int64_t> off(m + 1, 0);
  for (int i = 0; i < m; i++) off[i + 1] = off[i] + (int64_t)ks * so[2 * i];
  return off;
}
// KMeansPlusPlusClusterer.cluster with UNWEIGHTED threshold (KMeansPlusPlusClusterer.java:41-200).
static void kmeanspp_cluster(const float* data, int np, int dim, int k, int max_iter,
                             vo_jrandom* rng, float* cent) {
  if (np <= k) {
    std::memset(cent, 0, sizeof(float) * (size_t)k * dim);
    std::memcpy(cent, data, sizeof(float) * (size_t)np * dim);
    return;
  }
  int first = vo_jrandom_next_int_bound(rng, np);
  std::memcpy(cent, data + (size_t)first * dim, sizeof(float) * dim);
  std::vector<float> mind(np), scratch(np);
  vo_mat_vec_square_l2(data + (size_t)first * dim, data, np, dim, mind.data());
  for (int c = 1; c < k; c++) {
    double total = 0;
    for (int i = 0; i < np; i++) total += mind[i];
    int chosen;
    if (total == 0) {
      chosen = vo_jrandom_next_int_bound(rng, np);
    } else {
      double thr = vo_jrandom_next_double(rng) * total;
      double cum = 0;
      int sel = np - 1;
      for (int i = 0; i < np; i++) {
        cum += mind[i];
        if (cum >= thr) {
          sel = i;
          break;
        }
      }
      chosen = sel;
    }
    std::memcpy(cent + (size_t)c * dim, data + (size_t)chosen * dim, sizeof(float) * dim);
    vo_mat_vec_square_l2(data + (size_t)chosen * dim, data, np, dim, scratch.data());
    for (int i = 0; i < np; i++)
      if (scratch[i] < mind[i]) mind[i] = scratch[i];
  }
  std::vector<int> assign(np, 0);
  std::vector<float> d(k), sums((size_t)k * dim);
  std::vector<int> counts(k);
  for (int it = 0; it < max_iter; it++) {
    int changed = 0;
    for (int i = 0; i < np; i++) {
      vo_mat_vec_square_l2(data + (size_t)i * dim, cent, k, dim, d.data());
      int best = 0;
      float bd = d[0];
      for (int c = 1; c < k; c++)
        if (d[c] < bd) {
          bd = d[c];
          best = c;
        }
      if (assign[i] != best) {
        assign[i] = best;
        changed++;
      }
    }
    std::fill(sums.begin(), sums.end(), 0.0f);
    std::fill(counts.begin(), counts.end(), 0);
    for (int i = 0; i < np; i++) {
      int c = assign[i];
      counts[c]++;
      for (int j = 0; j < dim; j++) sums[(size_t)c * dim + j] += data[(size_t)i * dim + j];
    }
    for (int c = 0; c < k; c++)
      if (counts[c] > 0)
        for (int j = 0; j < dim; j++) cent[(size_t)c * dim + j] = sums[(size_t)c * dim + j] / (float)counts[c];
    if ((float)changed / (float)np < 0.01f) break;
  }
}
// ProductQuantizer.train(dataset, m, ks, center=false, trainThreads=1) (ProductQuantizer.java:246-289,706-714).
void vo_pq_train(const float* data, int64_t n, int32_t dim, int32_t m, int32_t ks,
                 float* codebooks) {
  std::vector<int32_t> so;
  std::vector<int64_t> off = codebook_offsets(dim, m, ks, so);
  std::vector<int32_t> idx = reservoir(n, 25000, 42);
  int np = (int)idx.size();
  vo_jrandom rng;
  vo_jrandom_init(&rng, 42);
  for (int s = 0; s < m; s++) {
    int sub = so[2 * s], o = so[2 * s + 1];
    std::vector<float> subv((size_t)np * sub);
    for (int i = 0; i < np; i++)
      std::memcpy(&subv[(size_t)i * sub], data + (int64_t)idx[i] * dim + o, sizeof(float) * sub);
    kmeanspp_cluster(subv.data(), np, sub, ks, 10, &rng, codebooks + off[s]);
  }
}
// ProductQuantizer.encodeInto, nearest-L2 path (ProductQuantizer.java:548-579).
void vo_pq_encode(const float* v, int32_t dim, int32_t m, int32_t ks, const float* cb,
                  uint8_t* code) {
  std::vector<int32_t> so;
  std::vector<int64_t> off = codebook_offsets(dim, m, ks, so);
  for (int s = 0; s < m; s++) {
    int sub = so[2 * s], o = so[2 * s + 1];
    const float* book = cb + off[s];
    int nearest = 0;
    float nd = vo_square_distance(v + o, book, sub);
    for (int c = 1; c < ks; c++) {
      float d = vo_square_distance(v + o, book + (size_t)c * sub, sub);
      if (d < nd) {
        nd = d;
        nearest = c;
      }
    }
    code[s] = (uint8_t)nearest;
  }
}
// buildADCTable (ProductQuantizer.java:521-544) without a global centroid.
void vo_pq_adc_table(const float* q, int32_t dim, int32_t m, int32_t ks, const float* cb,
                     int32_t use_dot, float* table) {
  std::vector<int32_t> so;
  std::vector<int64_t> off = codebook_offsets(dim, m, ks, so);
  for (int s = 0; s < m; s++) {
    int sub = so[2 * s], o = so[2 * s + 1];
    for (int c = 0; c < ks; c++) {
      const float* cc = cb + off[s] + (size_t)c * sub;
      table[(size_t)s * ks + c] = use_dot ? vo_dot(q + o, cc, sub) : vo_square_distance(q + o, cc, sub);
    }
  }
}
// KMeans.train serial path (KMeans.java:54-135,172-183,239-277).
void vo_kmeans_train(const float* data, int64_t n, int32_t dim, int32_t k, int32_t max_iter,
                     int64_t seed, float* cent, int32_t nthreads) {
  vo_jrandom rng;
  vo_jrandom_init(&rng, seed);
  int32_t first = vo_jrandom_next_int_bound(&rng, (int32_t)n);
  std::memcpy(cent, data + (int64_t)first * dim, sizeof(float) * dim);
  std::vector<float> mind(n, std::numeric_limits<float>::max()), sd(n);
  for (int c = 1; c < k; c++) {
    const float* prev = cent + (size_t)(c - 1) * dim;
    // batchSquaredL2(newest centroid, all points): the grouped kernel for rows < (n & ~3),
    // squareDistance for the rest (PanamaVectorUtilSupport.java:5547-5598).
    {
      int64_t grp = n & ~3LL;
      int limit = dim & ~(kLanes - 1);
      parallel_for(n, nthreads, [&](int64_t lo, int64_t hi) {
        for (int64_t i = lo; i < hi; i++) {
          const float* row = data + i * dim;
          if (i < grp) {
            float acc[kLanes] = {0};
            for (int p = 0; p < limit; p += kLanes)
              for (int j = 0; j < kLanes; j++) {
                float d = prev[p + j] - row[p + j];
                acc[j] = std::fma(d, d, acc[j]);
              }
            float s = reduce_add8(acc);
            for (int p = limit; p < dim; p++) {
              float e = prev[p] - row[p];
              s = std::fma(e, e, s);
            }
            sd[i] = s;
          } else {
            sd[i] = vo_square_distance(prev, row, dim);
          }
        }
      });
    }
    for (int64_t i = 0; i < n; i++)
      if (sd[i] < mind[i]) mind[i] = sd[i];
    double total = 0.0;
    for (int64_t i = 0; i < n; i++) total += mind[i];
    double thr = vo_jrandom_next_double(&rng) * total;
    double cum = 0.0;
    int64_t chosen = n - 1;
    for (int64_t i = 0; i < n; i++) {
      cum += mind[i];
      if (cum >= thr) {
        chosen = i;
        break;
      }
    }
    std::memcpy(cent + (size_t)c * dim, data + chosen * dim, sizeof(float) * dim);
  }
  std::vector<int32_t> assign(n, -1), next(n);
  std::vector<double> sums((size_t)k * dim);
  std::vector<int64_t> counts(k);
  for (int it = 0; it < max_iter; it++) {
    vo_kmeans_assign(data, n, dim, cent, k, next.data(), nthreads);
    bool changed = false;
    for (int64_t i = 0; i < n; i++)
      if (next[i] != assign[i]) {
        assign[i] = next[i];
        changed = true;
      }
    if (!changed) break;
    std::fill(sums.begin(), sums.end(), 0.0);
    std::fill(counts.begin(), counts.end(), 0);
    for (int64_t i = 0; i < n; i++) {
      int c = assign[i];
      counts[c]++;
      for (int d = 0; d < dim; d++) sums[(size_t)c * dim + d] += data[i * dim + d];
    }
    for (int c = 0; c < k; c++)
      if (counts[c] > 0)
        for (int d = 0; d < dim; d++)
          cent[(size_t)c * dim + d] = (float)(sums[(size_t)c * dim + d] / (double)counts[c]);
  }
}
// KMeans.nearestCentroid / BuoyIndex.route(v, 1, 0) (KMeans.java:239-251).
void vo_kmeans_assign(const float* data, int64_t n, int32_t dim, const float* cent, int32_t k,
                      int32_t* out, int32_t nthreads) {
  parallel_for(n, nthreads, [&](int64_t lo, int64_t hi) {
    std::vector<float> d(k);
    for (int64_t i = lo; i < hi; i++) {
      vo_mat_vec_square_l2(data + i * dim, cent, k, dim, d.data());
      int best = 0;
      float bd = d[0];
      for (int c = 1; c < k; c++)
        if (d[c] < bd) {
          bd = d[c];
          best = c;
        }
      out[i] = best;
    }
  });
}

// ---------------------------------------------------------------- batch encoders
void vo_sq8_encode_all(float min_q, float max_q, const float* data, int64_t n, int32_t dim,
                       int8_t* codes, float* corrections, int32_t nthreads) {
  parallel_for(n, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; i++)
      corrections[i] = vo_sq8_encode(min_q, max_q, data + i * dim, dim, codes + i * dim);
  });
}
void vo_bq_encode_all(const float* data, int64_t n, int32_t dim, uint64_t* words, int32_t nthreads) {
  int nw = (dim + 63) >> 6;
  parallel_for(n, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; i++) vo_bq_encode(data + i * dim, dim, words + i * nw);
  });
}
// BBQ encode: packBits with the centroid (distToC = sum (v - c)^2 in order) and
// computeCorrections (BinaryQuantizer.java:207-270): corr = (distToC, vl = min, width = max - min).
void vo_bbq_encode_all(const float* data, const float* cent, int64_t n, int32_t dim, uint64_t* words, float* corr,
                       int32_t nthreads) {
  int nw = (dim + 63) >> 6;
  parallel_for(n, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; i++) {
      const float* v = data + i * dim;
      uint64_t* w = words + i * nw;
      for (int j = 0; j < nw; j++) w[j] = 0;
      float dist = 0.0f, mn = INFINITY, mx = -INFINITY;
      for (int d = 0; d < dim; d++) {
        float c = v[d] - cent[d];
        dist += c * c;
        if (c >= 0) w[d >> 6] |= 1ULL << (d & 63);
      }
      for (int d = 0; d < dim; d++) {
        float c = v[d] - cent[d];
        if (c < mn) mn = c;
        if (c > mx) mx = c;
      }
      corr[i * 3] = dist;
      corr[i * 3 + 1] = mn;
      corr[i * 3 + 2] = mx - mn;
    }
  });
}
// bbqScoreFunction / computeBbqDot / asymmetricDot / extractBitPlanes
// (BinaryQuantizedVectors.java:110-275).
void vo_bbq_search(const uint64_t* words, const float* corr, const float* cent, int64_t n, int32_t dim,
                   int32_t metric, const float* queries, int32_t nq, int32_t k, int32_t policy, int32_t nthreads,
                   int32_t* ids, float* scores, int32_t* counts) {
  const int nw = (dim + 63) >> 6;
  struct Q {
    float qmin, w15, nsq, norm;
    int32_t qsum;
  };
  std::vector<Q> qs(nq);
  std::vector<uint64_t> planes((size_t)nq * 4 * nw, 0);
  for (int q = 0; q < nq; q++) {
    const float* v = queries + (int64_t)q * dim;
    std::vector<float> c(dim);
    for (int d = 0; d < dim; d++) c[d] = v[d] - cent[d];  // VectorUtil.subInPlace
    float nsq = 0.0f, mn = INFINITY, mx = -INFINITY;
    for (int d = 0; d < dim; d++) {
      nsq += c[d] * c[d];
      if (c[d] < mn) mn = c[d];
      if (c[d] > mx) mx = c[d];
    }
    const float width = mx - mn;
    const float norm = (float)std::sqrt((double)nsq);
    const float scale = width > 0 ? 15.0f / width : 0.0f;
    int32_t qsum = 0;
    uint64_t* pl = &planes[(size_t)q * 4 * nw];
    for (int d = 0; d < dim; d++) {
      int32_t qv = java_round((c[d] - mn) * scale);
      qv = std::max(0, std::min(15, qv));
      qsum += qv;
      for (int b = 0; b < 4; b++)
        if ((qv >> b) & 1) pl[(size_t)b * nw + (d >> 6)] |= 1ULL << (d & 63);
    }
    qs[q] = Q{mn, width / 15.0f, nsq, norm, qsum};
  }
  scan_topk(n, nq, k, policy, nthreads,
            [&](int64_t q, int64_t r) {
              const Q& qi = qs[q];
              const uint64_t* w = words + r * nw;
              const uint64_t* pl = &planes[(size_t)q * 4 * nw];
              int32_t raw = 0, pop = 0;
              for (int b = 0; b < 4; b++) {
                int32_t ps = 0;
                for (int j = 0; j < nw; j++) ps += __builtin_popcountll(w[j] & pl[(size_t)b * nw + j]);
                raw += ps << b;
              }
              for (int j = 0; j < nw; j++) pop += __builtin_popcountll(w[j]);
              const float dist = corr[r * 3], vl = corr[r * 3 + 1], width = corr[r * 3 + 2];
              const float approx = qi.qmin * (vl * (float)dim + width * (float)pop) +
                                   qi.w15 * (vl * (float)qi.qsum + width * (float)raw);
              switch (metric) {
                case VO_EUCLIDEAN: {
                  float adj = qi.nsq + dist - 2.0f * approx;
                  return 1.0f / (1.0f + java_max(adj, 0.0f));
                }
                case VO_COSINE: {
                  float vn = (float)std::sqrt((double)dist);
                  if (qi.norm == 0.0f || vn == 0.0f) return 0.0f;
                  float cosv = approx / (qi.norm * vn);
                  return java_max((1.0f + cosv) / 2.0f, 0.0f);
                }
                case VO_MAXIMUM_INNER_PRODUCT:
                  return vo_scale_mip(approx);
                default:
                  return java_max((1.0f + approx) / 2.0f, 0.0f);
              }
            },
            ids, scores, counts);
}
void vo_fp16_encode_all(const float* data, int64_t n, int32_t dim, uint16_t* codes, int32_t nthreads) {
  parallel_for(n * dim, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; i++) codes[i] = vo_f32_to_f16(data[i]);
  });
}
void vo_pq_encode_all(const float* data, int64_t n, int32_t dim, int32_t m, int32_t ks,
                      const float* codebooks, uint8_t* codes, int32_t nthreads) {
  parallel_for(n, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; i++) vo_pq_encode(data + i * dim, dim, m, ks, codebooks, codes + i * m);
  });
}

// ---------------------------------------------------------------- searches
// FlatScanAdapter.search / searchBatch (FlatScanAdapter.java:51-175).
void vo_flat_search(const float* db, int64_t n, int32_t dim, int32_t metric, const float* queries,
                    int32_t nq, int32_t k, int32_t policy, int32_t nthreads, int32_t* ids,
                    float* scores, int32_t* counts) {
  scan_topk(n, nq, k, policy, nthreads,
            [&](int64_t q, int64_t r) {
              return vo_compare(metric, queries + q * dim, db + r * dim, dim);
            },
            ids, scores, counts);
}
// QuantizedFlatScanAdapter.selectApproximateCandidates over ScalarQuantizedVectors
// (QuantizedFlatScanAdapter.java:97-113, ScalarQuantizedVectors.java:82-107).
void vo_sq_search(const int8_t* codes, const float* corr, int64_t n, int32_t dim, float min_q, float max_q,
                  int32_t max_value, int32_t metric, const float* queries, int32_t nq, int32_t k, int32_t policy,
                  int32_t nthreads, int32_t* ids, float* scores, int32_t* counts) {
  std::vector<int8_t> qc((size_t)nq * dim);
  std::vector<float> qcorr(nq);
  for (int q = 0; q < nq; q++)
    qcorr[q] = vo_sq_encode(min_q, max_q, max_value, queries + (int64_t)q * dim, dim, &qc[(size_t)q * dim]);
  scan_topk(n, nq, k, policy, nthreads,
            [&](int64_t q, int64_t r) {
              return vo_sq_score(metric, min_q, max_q, max_value, &qc[(size_t)q * dim], qcorr[q], codes + r * dim,
                                 corr[r], dim);
            },
            ids, scores, counts);
}
void vo_sq8_search(const int8_t* codes, const float* corr, int64_t n, int32_t dim, float min_q,
                   float max_q, int32_t metric, const float* queries, int32_t nq, int32_t k,
                   int32_t policy, int32_t nthreads, int32_t* ids, float* scores,
                   int32_t* counts) {
  vo_sq_search(codes, corr, n, dim, min_q, max_q, 127, metric, queries, nq, k, policy, nthreads, ids, scores, counts);
}
void vo_sq_encode_all(float min_q, float max_q, int32_t max_value, const float* data, int64_t n, int32_t dim,
                      int8_t* codes, float* corrections, int32_t nthreads) {
  parallel_for(n, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; i++)
      corrections[i] = vo_sq_encode(min_q, max_q, max_value, data + i * dim, dim, codes + i * dim);
  });
}
void vo_bq_search(const uint64_t* words, int64_t n, int32_t dim, int32_t metric,
                  const float* queries, int32_t nq, int32_t k, int32_t policy, int32_t nthreads,
                  int32_t* ids, float* scores, int32_t* counts) {
  int nw = (dim + 63) >> 6;
  std::vector<uint64_t> qw((size_t)nq * nw);
  for (int q = 0; q < nq; q++) vo_bq_encode(queries + (int64_t)q * dim, dim, &qw[(size_t)q * nw]);
  scan_topk(n, nq, k, policy, nthreads,
            [&](int64_t q, int64_t r) {
              int h = vo_hamming(&qw[(size_t)q * nw], words + r * nw, nw);
              return vo_bq_score(metric, h, dim);
            },
            ids, scores, counts);
}
// Fp16QuantizedVectors.scoreFunctionFor (Fp16QuantizedVectors.java:70-94).
void vo_fp16_search(const uint16_t* codes, int64_t n, int32_t dim, int32_t metric,
                    const float* queries, int32_t nq, int32_t k, int32_t policy, int32_t nthreads,
                    int32_t* ids, float* scores, int32_t* counts) {
  scan_topk(n, nq, k, policy, nthreads,
            [&](int64_t q, int64_t r) {
              thread_local std::vector<float> dec;
              dec.resize(dim);
              for (int d = 0; d < dim; d++) dec[d] = vo_f16_to_f32(codes[r * dim + d]);
              const float* qq = queries + q * dim;
              if (metric == VO_EUCLIDEAN) return 1.0f / (1.0f + vo_square_distance(qq, dec.data(), dim));
              float dot = vo_dot(qq, dec.data(), dim);
              if (metric == VO_MAXIMUM_INNER_PRODUCT) return vo_scale_mip(dot);
              return java_max((1.0f + dot) / 2.0f, 0.0f);
            },
            ids, scores, counts);
}
// PQVectors.scoreFunctionFor (PQVectors.java:104-191) behind QuantizedFlatScanAdapter's
// candidate heap: per query, ProductQuantizer.buildADCTable (ProductQuantizer.java:521-544) of
// the query minus the global centroid (subInPlace, when the quantizer has one): dotProduct
// entries for DOT_PRODUCT / COSINE / MAXIMUM_INNER_PRODUCT, squareDistance entries for
// EUCLIDEAN; per row the sequential fp32 sum of the M entries, then
//   DOT_PRODUCT  max((1 + sum) / 2, 0);  EUCLIDEAN  1 / (1 + sum);  MIP  scaleMaxInnerProductScore(sum);
//   COSINE  dot / (|q - gc| * sqrt(sum of centroidNormSq[m][code[m]])), 0 when either norm is 0,
//           then max((1 + cos) / 2, 0); centroidNormSq and |q - gc|^2 sequential sums of squares.
// Codebooks concatenated per subspace with computeSubspaceSizesAndOffsets' sizes.
void vo_pq_flat_search(const float* cb, const float* global_centroid, const uint8_t* codes, int64_t n, int32_t dim,
                       int32_t m, int32_t ks, int32_t metric, const float* queries, int32_t nq, int32_t k,
                       int32_t policy, int32_t nthreads, int32_t* ids, float* scores, int32_t* counts) {
  std::vector<int32_t> so;
  std::vector<int64_t> off = codebook_offsets(dim, m, ks, so);
  std::vector<float> cnorm((size_t)m * ks);  // PQVectors.precomputeCentroidNormsSq (:73-89)
  for (int s = 0; s < m; s++) {
    const int sub = so[2 * s];
    for (int c = 0; c < ks; c++) {
      const float* cc = cb + off[s] + (size_t)c * sub;
      float norm = 0.0f;
      for (int d = 0; d < sub; d++) norm += cc[d] * cc[d];
      cnorm[(size_t)s * ks + c] = norm;
    }
  }
  const int kk = (int)std::min<int64_t>(k, n);
  parallel_for(nq, nthreads, [&](int64_t lo, int64_t hi) {
    std::vector<float> table((size_t)m * ks), qc(dim);
    for (int64_t q = lo; q < hi; q++) {
      const float* qq = queries + q * dim;
      for (int d = 0; d < dim; d++) qc[d] = global_centroid ? qq[d] - global_centroid[d] : qq[d];
      vo_pq_adc_table(qc.data(), dim, m, ks, cb, metric == VO_EUCLIDEAN ? 0 : 1, table.data());
      float qnorm_sq = 0.0f;
      for (int d = 0; d < dim; d++) qnorm_sq += qc[d] * qc[d];
      const float qnorm = (float)std::sqrt((double)qnorm_sq);
      auto score = [&](int64_t r) -> float {
        const uint8_t* code = codes + r * m;
        float sum = 0.0f, vsq = 0.0f;
        for (int s = 0; s < m; s++) sum += table[(size_t)s * ks + code[s]];
        switch (metric) {
          case VO_EUCLIDEAN: return 1.0f / (1.0f + sum);
          case VO_MAXIMUM_INNER_PRODUCT: return vo_scale_mip(sum);
          case VO_COSINE: {
            for (int s = 0; s < m; s++) vsq += cnorm[(size_t)s * ks + code[s]];
            const float vnorm = (float)std::sqrt((double)vsq);
            if (qnorm == 0.0f || vnorm == 0.0f) return 0.0f;
            const float cosv = sum / (qnorm * vnorm);
            return java_max((1.0f + cosv) / 2.0f, 0.0f);
          }
          default: return java_max((1.0f + sum) / 2.0f, 0.0f);
        }
      };
      int32_t* oi = ids + q * k;
      float* os = scores + q * k;
      if (kk <= 0) {
        counts[q] = 0;
      } else if (policy == VO_POLICY_REFERENCE_HEAP) {
        RefHeap h(kk);
        for (int64_t r = 0; r < n; r++) h.offer((int32_t)r, score(r));
        counts[q] = h.drain(oi, os);
      } else {
        CanonTopK h(kk);
        for (int64_t r = 0; r < n; r++) h.offer((int32_t)r, score(r));
        counts[q] = h.drain(oi, os);
      }
    }
  });
}
// QuantizedFlatScanAdapter.search (QuantizedFlatScanAdapter.java:59-95).
void vo_quantized_two_pass_search(int32_t kind, const void* qdata, const float* qcorr,
                                  float min_q, float max_q, const float* db, int64_t n,
                                  int32_t dim, int32_t metric, const float* queries, int32_t nq,
                                  int32_t k, float oqf, int32_t policy, int32_t nthreads,
                                  int32_t* ids, float* scores, int32_t* counts) {
  if (n == 0) {
    for (int q = 0; q < nq; q++) counts[q] = 0;
    return;
  }
  if (oqf <= 1.0f) {
    vo_flat_search(db, n, dim, metric, queries, nq, k, policy, nthreads, ids, scores, counts);
    return;
  }
  int64_t ck = std::min<int64_t>(n, std::max<int64_t>(k, (int64_t)std::ceil((double)((float)k * oqf))));
  std::vector<int32_t> cid((size_t)nq * ck), cnt(nq);
  std::vector<float> csc((size_t)nq * ck);
  if (kind == 0)
    vo_sq8_search((const int8_t*)qdata, qcorr, n, dim, min_q, max_q, metric, queries, nq, (int32_t)ck,
                  policy, nthreads, cid.data(), csc.data(), cnt.data());
  else if (kind == 1)
    vo_bq_search((const uint64_t*)qdata, n, dim, metric, queries, nq, (int32_t)ck, policy,
                 nthreads, cid.data(), csc.data(), cnt.data());
  else
    vo_fp16_search((const uint16_t*)qdata, n, dim, metric, queries, nq, (int32_t)ck, policy,
                   nthreads, cid.data(), csc.data(), cnt.data());
  vo_rescore_candidates(db, dim, metric, queries, nq, cid.data(), (int32_t)ck, cnt.data(), k, policy, nthreads, ids,
                        scores, counts);
}
// The exact second pass of QuantizedFlatScanAdapter.search (QuantizedFlatScanAdapter.java:79-94):
// every candidate re-scored with the full-precision SimilarityFunction.compare, k best kept.
void vo_rescore_candidates(const float* db, int32_t dim, int32_t metric, const float* queries, int32_t nq,
                           const int32_t* cid, int32_t stride, const int32_t* cnt, int32_t k, int32_t policy,
                           int32_t nthreads, int32_t* ids, float* scores, int32_t* counts) {
  parallel_for(nq, nthreads, [&](int64_t lo, int64_t hi) {
    for (int64_t q = lo; q < hi; q++) {
      int c = cnt[q];
      int kk = std::min(k, c);
      const float* qq = queries + q * dim;
      if (policy == VO_POLICY_REFERENCE_HEAP) {
        RefHeap h(std::max(kk, 1));
        for (int i = 0; i < c; i++) {
          int32_t o = cid[q * stride + i];
          h.offer(o, vo_compare(metric, qq, db + (int64_t)o * dim, dim));
        }
        counts[q] = kk > 0 ? h.drain(ids + q * k, scores + q * k) : 0;
      } else {
        CanonTopK h(std::max(kk, 1));
        for (int i = 0; i < c; i++) {
          int32_t o = cid[q * stride + i];
          h.offer(o, vo_compare(metric, qq, db + (int64_t)o * dim, dim));
        }
        counts[q] = kk > 0 ? h.drain(ids + q * k, scores + q * k) : 0;
      }
    }
  });
}
// CentroidIndex.routeWithSpillDistances, gamma == 0 (CentroidIndex.java:89-211).
// CentroidIndex.computeDistances (CentroidIndex.java:196-211): squared L2 (EUCLIDEAN), negated
// cosine via the l2-normalised query (COSINE), negated dot (dot-style metrics).
static void route_distances(const float* cent, int32_t nlist, int32_t dim, int32_t metric, const float* qq,
                            float* d, float* qn) {
  if (metric == VO_EUCLIDEAN) {
    vo_mat_vec_square_l2(qq, cent, nlist, dim, d);
  } else if (metric == VO_COSINE) {
    std::memcpy(qn, qq, sizeof(float) * dim);
    vo_l2normalize(qn, dim);
    vo_mat_vec_dot(qn, cent, nlist, dim, d);
    for (int i = 0; i < nlist; i++) d[i] = -d[i];
  } else {
    vo_mat_vec_dot(qq, cent, nlist, dim, d);
    for (int i = 0; i < nlist; i++) d[i] = -d[i];
  }
}
void vo_route(const float* cent, int32_t nlist, int32_t dim, int32_t metric, const float* queries,
              int32_t nq, int32_t nprobe, int32_t policy, int32_t nthreads, int32_t* list_ids,
              float* dists) {
  int probes = std::min(nprobe, nlist);
  parallel_for(nq, nthreads, [&](int64_t lo, int64_t hi) {
    std::vector<float> d(nlist), qn(dim);
    std::vector<int32_t> tid(probes);
    std::vector<float> tds(probes);
    for (int64_t q = lo; q < hi; q++) {
      const float* qq = queries + q * dim;
      route_distances(cent, nlist, dim, metric, qq, d.data(), qn.data());
      int32_t* oi = list_ids + q * nprobe;
      float* od = dists + q * nprobe;
      if (policy == VO_POLICY_CANONICAL) {
        std::vector<int32_t> order(nlist);
        std::iota(order.begin(), order.end(), 0);
        std::partial_sort(order.begin(), order.begin() + probes, order.end(), [&](int a, int b) {
          if (d[a] != d[b]) return d[a] < d[b];
          return a < b;
        });
        for (int i = 0; i < probes; i++) {
          oi[i] = order[i];
          od[i] = d[order[i]];
        }
        continue;
      }
      int hs = 0;
      for (int i = 0; i < nlist; i++) {
        float di = d[i];
        if (hs < probes) {
          tid[hs] = i;
          tds[hs] = di;
          hs++;
          int idx = hs - 1;
          while (idx > 0) {
            int p = (idx - 1) >> 1;
            if (tds[idx] > tds[p]) {
              std::swap(tds[idx], tds[p]);
              std::swap(tid[idx], tid[p]);
              idx = p;
            } else break;
          }
        } else if (di < tds[0]) {
          tid[0] = i;
          tds[0] = di;
          int idx = 0, half = hs >> 1;
          while (idx < half) {
            int l = 2 * idx + 1, r = l + 1, lg = l;
            if (r < hs && tds[r] > tds[l]) lg = r;
            if (tds[idx] >= tds[lg]) break;
            std::swap(tds[idx], tds[lg]);
            std::swap(tid[idx], tid[lg]);
            idx = lg;
          }
        }
      }
      for (int i = 1; i < hs; i++) {
        float dd = tds[i];
        int id = tid[i], j = i - 1;
        while (j >= 0 && tds[j] > dd) {
          tds[j + 1] = tds[j];
          tid[j + 1] = tid[j];
          j--;
        }
        tds[j + 1] = dd;
        tid[j + 1] = id;
      }
      for (int i = 0; i < probes; i++) {
        oi[i] = tid[i];
        od[i] = tds[i];
      }
    }
  });
}
// CentroidIndex.routeWithSpillDistances with gamma > 0 (CentroidIndex.java:89-187,213-220): the
// nprobe nearest in ascending order (reference heap, as vo_route), then, walking them in that
// order while a primary's distance is within spillBoundary(nearest, gamma), each one's spill
// target when it is a valid list not yet included, appended with its own distance.
// spillBoundary: nearest * (1 + gamma) for EUCLIDEAN; otherwise -(s - |s| * gamma) with
// s = -nearest.  Writes up to 2 * nprobe lists per query and their count.
void vo_route_spill(const float* cent, int32_t nlist, int32_t dim, int32_t metric, const float* queries,
                    int32_t nq, int32_t nprobe, float gamma, const int32_t* spill_targets, int32_t nthreads,
                    int32_t* list_ids, float* dists, int32_t* counts) {
  const int probes = std::min(nprobe, nlist);
  const int width = 2 * nprobe;
  std::vector<int32_t> prim((size_t)nq * probes);
  std::vector<float> pd((size_t)nq * probes);
  vo_route(cent, nlist, dim, metric, queries, nq, probes, VO_POLICY_REFERENCE_HEAP, nthreads, prim.data(), pd.data());
  parallel_for(nq, nthreads, [&](int64_t lo, int64_t hi) {
    std::vector<float> d(nlist), qn(dim);
    std::vector<char> included(nlist);
    for (int64_t q = lo; q < hi; q++) {
      route_distances(cent, nlist, dim, metric, queries + q * dim, d.data(), qn.data());
      std::fill(included.begin(), included.end(), 0);
      int32_t* oi = list_ids + q * width;
      float* od = dists + q * width;
      int count = 0;
      for (int r = 0; r < probes; r++) {
        oi[count] = prim[(size_t)q * probes + r];
        od[count] = pd[(size_t)q * probes + r];
        included[oi[count]] = 1;
        count++;
      }
      if (gamma > 0.0f && spill_targets && count > 0) {
        const float nearest = pd[(size_t)q * probes];
        float boundary;
        if (metric == VO_EUCLIDEAN) {
          boundary = nearest * (1.0f + gamma);
        } else {
          const float ns = -nearest;
          const float thr = ns - std::fabs(ns) * gamma;
          boundary = -thr;
        }
        for (int r = 0; r < probes; r++) {
          if (pd[(size_t)q * probes + r] > boundary) break;
          const int32_t sp = spill_targets[prim[(size_t)q * probes + r]];
          if (sp >= 0 && sp < nlist && !included[sp]) {
            oi[count] = sp;
            od[count] = d[sp];
            included[sp] = 1;
            count++;
          }
        }
      }
      counts[q] = count;
    }
  });
}
// IvfIndex.pqSearch (IvfIndex.java:539-619) with TopKHeap semantics (TopKHeap.java:60-95).
// The probed clusters of every query, in the order IvfIndex visits them: the min(nprobe, nlist)
// nearest (CentroidIndex.routeWithSpillDistances, ascending), then with gamma > 0 and spill
// targets the SOAR additions (vo_route_spill).  width slots per query, cnt[q] of them used.
struct IvfRoute {
  int width = 0;
  std::vector<int32_t> lids, cnt;
  std::vector<float> ld;
};
static IvfRoute ivf_route(const float* cent, int32_t nlist, int32_t dim, int32_t metric, const float* queries,
                          int32_t nq, int32_t nprobe, float gamma, const int32_t* spill, int32_t policy,
                          int32_t nthreads) {
  IvfRoute r;
  const int probes = std::min(nprobe, nlist);
  if (gamma > 0.0f && spill) {
    r.width = 2 * nprobe;
    r.lids.assign((size_t)nq * r.width, -1);
    r.ld.assign((size_t)nq * r.width, 0.0f);
    r.cnt.assign(nq, 0);
    vo_route_spill(cent, nlist, dim, metric, queries, nq, nprobe, gamma, spill, nthreads, r.lids.data(), r.ld.data(),
                   r.cnt.data());
  } else {
    r.width = probes;
    r.lids.resize((size_t)nq * probes);
    r.ld.resize((size_t)nq * probes);
    r.cnt.assign(nq, probes);
    vo_route(cent, nlist, dim, metric, queries, nq, probes, policy, nthreads, r.lids.data(), r.ld.data());
  }
  return r;
}

static void ivfpq_search(const float* cent, int32_t nlist, int32_t dim, const int64_t* loff, const int32_t* lord,
                         int32_t m, int32_t ks, const float* cb, const uint8_t* codes, int64_t n, int32_t metric,
                         const float* queries, int32_t nq, int32_t k, int32_t nprobe, float gamma,
                         const int32_t* spill, int32_t rescore, const float* vectors, int32_t policy,
                         int32_t nthreads, int32_t* ids, float* scores, int32_t* counts) {
  const IvfRoute route = ivf_route(cent, nlist, dim, metric, queries, nq, nprobe, gamma, spill, policy, nthreads);
  int64_t wide = std::min<int64_t>((int64_t)k * rescore, n);
  if (wide < 1) wide = 1;
  bool euclid = metric == VO_EUCLIDEAN;
  parallel_for(nq, nthreads, [&](int64_t lo, int64_t hi) {
    std::vector<float> table((size_t)m * ks), resid(dim);
    std::vector<int32_t> wi(wide);
    std::vector<float> ws(wide);
    for (int64_t q = lo; q < hi; q++) {
      const float* qq = queries + q * dim;
      RefHeap rh((int)wide);
      CanonTopK ch((int)wide);
      auto offer = [&](int32_t o, float s) {
        if (policy == VO_POLICY_REFERENCE_HEAP) {
          // TopKHeap rejects score <= root when full (TopKHeap.java:68)
          if (rh.size < rh.cap) rh.offer(o, s);
          else if (s > rh.sc[0]) rh.offer(o, s);
        } else {
          ch.offer(o, s);
        }
      };
      for (int p = 0; p < route.cnt[q]; p++) {
        int cid = route.lids[(size_t)q * route.width + p];
        int64_t b = loff[cid], e = loff[cid + 1];
        if (b == e) continue;
        const float* c = cent + (size_t)cid * dim;
        float base = 0.0f;
        if (euclid) {
          for (int d = 0; d < dim; d++) resid[d] = qq[d] - c[d];
          vo_pq_adc_table(resid.data(), dim, m, ks, cb, 0, table.data());
        } else {
          vo_pq_adc_table(qq, dim, m, ks, cb, 1, table.data());
          base = metric == VO_COSINE ? 0.0f : vo_dot(qq, c, dim);
        }
        for (int64_t i = b; i < e; i++) {
          int32_t o = lord[i];
          const uint8_t* code = codes + (int64_t)o * m;
          float sum = 0.0f;
          for (int s = 0; s < m; s++) sum += table[(size_t)s * ks + code[s]];
          offer(o, euclid ? -sum : base + sum);
        }
      }
      int cnt = policy == VO_POLICY_REFERENCE_HEAP ? rh.drain(wi.data(), ws.data())
                                                   : ch.drain(wi.data(), ws.data());
      int32_t* oi = ids + q * k;
      float* os = scores + q * k;
      if (rescore == 1) {
        int c2 = 0;
        for (int i = 0; i < cnt && c2 < k; i++) {
          if (ws[i] < -3.4028235e38f) continue;  // minScore = -Float.MAX_VALUE
          oi[c2] = wi[i];
          os[c2] = ws[i];
          c2++;
        }
        counts[q] = c2;
      } else {
        auto exact = [&](int32_t o) {
          const float* v = vectors + (int64_t)o * dim;
          switch (metric) {
            case VO_EUCLIDEAN: return -vo_square_distance(qq, v, dim);
            case VO_COSINE: return vo_cosine(qq, v, dim);
            default: return vo_dot(qq, v, dim);
          }
        };
        if (policy == VO_POLICY_REFERENCE_HEAP) {
          RefHeap fh(k);
          for (int i = 0; i < cnt; i++) {
            float s = exact(wi[i]);
            if (fh.size < fh.cap) fh.offer(wi[i], s);
            else if (s > fh.sc[0]) fh.offer(wi[i], s);
          }
          counts[q] = fh.drain(oi, os);
        } else {
          CanonTopK fh(k);
          for (int i = 0; i < cnt; i++) fh.offer(wi[i], exact(wi[i]));
          counts[q] = fh.drain(oi, os);
        }
      }
    }
  });
}
void vo_ivfpq_search(const float* cent, int32_t nlist, int32_t dim, const int64_t* loff,
                     const int32_t* lord, int32_t m, int32_t ks, const float* cb,
                     const uint8_t* codes, int64_t n, int32_t metric, const float* queries,
                     int32_t nq, int32_t k, int32_t nprobe, int32_t rescore, const float* vectors,
                     int32_t policy, int32_t nthreads, int32_t* ids, float* scores,
                     int32_t* counts) {
  ivfpq_search(cent, nlist, dim, loff, lord, m, ks, cb, codes, n, metric, queries, nq, k, nprobe, 0.0f, nullptr,
               rescore, vectors, policy, nthreads, ids, scores, counts);
}
// IvfIndex.pqSearch with IvfSearchRequest.gamma > 0: the clusters of routeWithSpillDistances,
// SOAR spill targets appended (IvfIndex.java:545-547, CentroidIndex.java:168-187).
void vo_ivfpq_search_spill(const float* cent, int32_t nlist, int32_t dim, const int64_t* loff, const int32_t* lord,
                           int32_t m, int32_t ks, const float* cb, const uint8_t* codes, int64_t n, int32_t metric,
                           const float* queries, int32_t nq, int32_t k, int32_t nprobe, float gamma,
                           const int32_t* spill_targets, int32_t rescore, const float* vectors, int32_t nthreads,
                           int32_t* ids, float* scores, int32_t* counts) {
  ivfpq_search(cent, nlist, dim, loff, lord, m, ks, cb, codes, n, metric, queries, nq, k, nprobe, gamma,
               spill_targets, rescore, vectors, VO_POLICY_CANONICAL, nthreads, ids, scores, counts);
}
// IvfIndex.search without PQ (IvfIndex.java:170-226): route, then every probed cluster's
// ordinals in batches of BATCH_ROWS = 64 through batchSquaredL2 / batchDotProduct
// (scanPartitionBulk, :244-277 -- matVecSquaredL2 / matVecDot over the batch: groups of four
// rows on the 8-lane accumulators, the batch's last count % 4 rows through squareDistance /
// dotProduct); score -d (EUCLIDEAN), dot (DOT_PRODUCT, MAXIMUM_INNER_PRODUCT) or
// (float)(dot / sqrt((double)|q|^2 * (double)|v|^2)) with both norms from dotProduct (COSINE,
// computeNormsSq :83-89); scores < minScore (-Float.MAX_VALUE) skipped; TopKHeap of k.
// The EUCLIDEAN triangle-inequality early exit (:190-200) is restated by
// vo_ivfflat_search_early_exit (radii given): once the heap is full, the first cluster in route
// order whose bound (max(0, (float) sqrt(centroid distance) - radius))^2 reaches the heap's
// worst distance ends the scan, and every later cluster is skipped with it -- including one whose
// larger radius leaves a smaller bound, so it can miss a closer row that scanning every probed
// cluster (vo_ivfflat_search) finds.  Not restated: the HARMONY key-dimension path (:207-212,
// scanPartitionWithHarmony :279-289) of partitions built with key dimensions.
// HARMONY (kd_off / kd: each partition's key dimensions as CSR, nullable): for EUCLIDEAN, a
// partition with key dimensions met with a full heap is scanned by scanPartitionWithHarmony
// (IvfIndex.java:214-216,279-289): each row's partialSquaredDistance over the key dimensions
// (DimensionAnalysis.java:96-104, sequential) skips it when >= the heap's worst distance, else its
// score is -squareDistance(query, row) (not the batched order).
static void ivfflat_search(const float* cent, int32_t nlist, int32_t dim, const int64_t* loff, const int32_t* lord,
                           const float* vectors, int32_t metric, const float* radii, const float* queries,
                           int32_t nq, int32_t k, int32_t nprobe, float gamma, const int32_t* spill, int32_t policy,
                           int32_t nthreads, int32_t* ids, float* scores, int32_t* counts,
                           const int64_t* kd_off = nullptr, const int32_t* kd = nullptr) {
  const IvfRoute route = ivf_route(cent, nlist, dim, metric, queries, nq, nprobe, gamma, spill, policy, nthreads);
  const bool euclid = metric == VO_EUCLIDEAN, cosine = metric == VO_COSINE;
  parallel_for(nq, nthreads, [&](int64_t lo, int64_t hi) {
    std::vector<float> batch((size_t)64 * dim), out(64);
    for (int64_t q = lo; q < hi; q++) {
      const float* qq = queries + q * dim;
      const float qn = cosine ? vo_dot(qq, qq, dim) : 0.0f;
      RefHeap rh(k);
      CanonTopK ch(k);
      for (int p = 0; p < route.cnt[q]; p++) {
        int cid = route.lids[(size_t)q * route.width + p];
        if (euclid && radii) {
          const bool ref = policy == VO_POLICY_REFERENCE_HEAP;
          const bool full = ref ? rh.size == rh.cap : (int)ch.v.size() == ch.cap;
          if (full) {
            const float worst = ref ? rh.sc[0] : ch.v.front().first;
            const float centroid_l2 = (float)std::sqrt((double)route.ld[(size_t)q * route.width + p]);
            const float lb = centroid_l2 - radii[cid];
            if (lb > 0.0f) {
              const float lb_sq = lb * lb;
              if (lb_sq >= -worst) break;  // route order is ascending: no later cluster is scanned
            }
          }
        }
        int64_t b = loff[cid], e = loff[cid + 1];
        const bool ref_heap = policy == VO_POLICY_REFERENCE_HEAP;
        const bool full_now = ref_heap ? rh.size == rh.cap : (int)ch.v.size() == ch.cap;
        if (euclid && kd_off && kd_off[cid + 1] > kd_off[cid] && full_now) {
          for (int64_t i = b; i < e; i++) {
            const int32_t o = lord[i];
            const float* v = vectors + (int64_t)o * dim;
            float partial = 0.0f;
            for (int64_t t = kd_off[cid]; t < kd_off[cid + 1]; t++) {
              const float df = qq[kd[t]] - v[kd[t]];
              partial += df * df;
            }
            const float worst = ref_heap ? rh.sc[0] : ch.v.front().first;
            if (partial >= -worst) continue;
            const float sc = -vo_square_distance(qq, v, dim);
            if (sc < -3.4028235e38f) continue;
            if (ref_heap) {
              if (sc > rh.sc[0]) rh.offer(o, sc);
            } else {
              ch.offer(o, sc);
            }
          }
          continue;
        }
        for (int64_t s0 = b; s0 < e; s0 += 64) {
          const int cnt = (int)std::min<int64_t>(64, e - s0);
          for (int j = 0; j < cnt; j++)
            std::memcpy(&batch[(size_t)j * dim], vectors + (int64_t)lord[s0 + j] * dim, sizeof(float) * dim);
          if (euclid) vo_mat_vec_square_l2(qq, batch.data(), cnt, dim, out.data());
          else vo_mat_vec_dot(qq, batch.data(), cnt, dim, out.data());
          for (int j = 0; j < cnt; j++) {
            const int32_t o = lord[s0 + j];
            float sc;
            if (euclid) {
              sc = -out[j];
            } else if (cosine) {
              const float* v = vectors + (int64_t)o * dim;
              sc = (float)(out[j] / std::sqrt((double)qn * (double)vo_dot(v, v, dim)));
            } else {
              sc = out[j];
            }
            if (sc < -3.4028235e38f) continue;
            if (policy == VO_POLICY_REFERENCE_HEAP) {
              if (rh.size < rh.cap) rh.offer(o, sc);
              else if (sc > rh.sc[0]) rh.offer(o, sc);
            } else {
              ch.offer(o, sc);
            }
          }
        }
      }
      counts[q] = policy == VO_POLICY_REFERENCE_HEAP ? rh.drain(ids + q * k, scores + q * k)
                                                     : ch.drain(ids + q * k, scores + q * k);
    }
  });
}
void vo_ivfflat_search(const float* cent, int32_t nlist, int32_t dim, const int64_t* loff, const int32_t* lord,
                       const float* vectors, int64_t n, int32_t metric, const float* queries, int32_t nq,
                       int32_t k, int32_t nprobe, int32_t policy, int32_t nthreads, int32_t* ids, float* scores,
                       int32_t* counts) {
  (void)n;
  ivfflat_search(cent, nlist, dim, loff, lord, vectors, metric, nullptr, queries, nq, k, nprobe, 0.0f, nullptr,
                 policy, nthreads, ids, scores, counts);
}
void vo_ivfflat_search_early_exit(const float* cent, int32_t nlist, int32_t dim, const int64_t* loff,
                                  const int32_t* lord, const float* vectors, int64_t n, int32_t metric,
                                  const float* radii, const float* queries, int32_t nq, int32_t k, int32_t nprobe,
                                  int32_t policy, int32_t nthreads, int32_t* ids, float* scores, int32_t* counts) {
  (void)n;
  ivfflat_search(cent, nlist, dim, loff, lord, vectors, metric, radii, queries, nq, k, nprobe, 0.0f, nullptr,
                 policy, nthreads, ids, scores, counts);
}
// IvfIndex.search (no PQ) as the reference runs it in full: clusters of routeWithSpillDistances
// (SOAR spill targets appended when gamma > 0), and for EUCLIDEAN the early exit against radii.
void vo_ivfflat_search_spill(const float* cent, int32_t nlist, int32_t dim, const int64_t* loff, const int32_t* lord,
                             const float* vectors, int32_t metric, const float* radii, const float* queries,
                             int32_t nq, int32_t k, int32_t nprobe, float gamma, const int32_t* spill_targets,
                             const int64_t* kd_off, const int32_t* kd, int32_t nthreads, int32_t* ids, float* scores,
                             int32_t* counts) {
  ivfflat_search(cent, nlist, dim, loff, lord, vectors, metric, radii, queries, nq, k, nprobe, gamma, spill_targets,
                 VO_POLICY_CANONICAL, nthreads, ids, scores, counts, kd_off, kd);
}
// BuoyIndex.computeRadii / euclideanDist (BuoyIndex.java:175-183,220-227).
void vo_ivf_radii(const float* cent, int32_t nlist, int32_t dim, const int64_t* loff, const int32_t* lord,
                  const float* vectors, float* radii) {
  for (int l = 0; l < nlist; l++) {
    float r = 0.0f;
    const float* c = cent + (size_t)l * dim;
    for (int64_t i = loff[l]; i < loff[l + 1]; i++) {
      const float* v = vectors + (int64_t)lord[i] * dim;
      float sum = 0.0f;
      for (int d = 0; d < dim; d++) {
        const float x = v[d] - c[d];
        sum += x * x;
      }
      const float dist = (float)std::sqrt((double)sum);
      if (dist > r) r = dist;
    }
    radii[l] = r;
  }
}
// IndexShards.mergeWithOffsets (IndexShards.java:168-211).
void vo_merge_shards(int32_t ns, const int64_t* offsets, const int32_t* sids, const float* ssc,
                     const int32_t* scnt, int32_t kin, int32_t nq, int32_t k, int32_t policy,
                     int32_t* ids, float* scores, int32_t* counts) {
  for (int q = 0; q < nq; q++) {
    std::vector<int32_t> id;
    std::vector<float> sc;
    for (int s = 0; s < ns; s++) {
      int c = scnt[(size_t)s * nq + q];
      for (int j = 0; j < c; j++) {
        size_t at = ((size_t)s * nq + q) * kin + j;
        id.push_back((int32_t)(sids[at] + offsets[s]));
        sc.push_back(ssc[at]);
      }
    }
    int total = (int)id.size();
    int fk = std::min(k, total);
    if (policy == VO_POLICY_REFERENCE_HEAP) {
      for (int i = 0; i < fk; i++) {
        int bi = i;
        float bs = sc[i];
        for (int j = i + 1; j < total; j++)
          if (sc[j] > bs) {
            bs = sc[j];
            bi = j;
          }
        if (bi != i) {
          std::swap(sc[i], sc[bi]);
          std::swap(id[i], id[bi]);
        }
      }
    } else {
      std::vector<int> ord(total);
      std::iota(ord.begin(), ord.end(), 0);
      std::partial_sort(ord.begin(), ord.begin() + fk, ord.end(), [&](int a, int b) {
        if (sc[a] != sc[b]) return sc[a] > sc[b];
        return id[a] < id[b];
      });
      std::vector<int32_t> id2(fk);
      std::vector<float> sc2(fk);
      for (int i = 0; i < fk; i++) {
        id2[i] = id[ord[i]];
        sc2[i] = sc[ord[i]];
      }
      for (int i = 0; i < fk; i++) {
        id[i] = id2[i];
        sc[i] = sc2[i];
      }
    }
    for (int i = 0; i < fk; i++) {
      ids[(size_t)q * k + i] = id[i];
      scores[(size_t)q * k + i] = sc[i];
    }
    counts[q] = fk;
  }
}
// TopK.select (TopK.java:58-116): NaN rejected with a -1 return.
int32_t vo_topk_select(const float* scores, int32_t n, int32_t k, int32_t* out) {
  if (k <= 0 || n == 0) return 0;
  for (int i = 0; i < n; i++)
    if (std::isnan(scores[i])) return -1;
  CanonTopK h(std::min(k, n));
  for (int i = 0; i < n; i++) h.offer(i, scores[i]);
  std::vector<float> tmp(std::min(k, n));
  return h.drain(out, tmp.data());
}

}  // extern "C"
