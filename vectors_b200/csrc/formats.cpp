// formats.cpp -- readers for the reference's persistent index files, feeding the device builds.
//
//   quantized.bin  QuantizedVectorsCodec.decode (vectors-db/.../storage/QuantizedVectorsCodec.java:
//                  131-192): little-endian; 20-byte header magic 'VQTZ' (FileFormat.java:77),
//                  version 1 (FileFormat.java:112), QuantizerKind ordinal, dimension, vectorCount;
//                  then per kind the quantizer state and the per-vector records: SQ8/SQ4
//                  (:257-296, ScalarBits ordinal + quantiles, then codes + one float correction per
//                  vector), BQ (:475-518, BinaryMode ordinal [+ centroid for BBQ], then the words
//                  [+ 3 corrections for BBQ]), FP16 (:211-221, binary16 codes only).
//   graph.bin      of IVF generations: IvfIndex.encode (vectors-ivf/.../IvfIndex.java:354-400;
//                  decode :408-442; PQ trailer :450-500) around BuoyIndex.encode
//                  (BuoyIndex.java:130-167), big-endian (ByteBuffer's default order and
//                  DataOutputStream).
//
// The checks and their messages follow the Java decoders, so a file the reference rejects is
// rejected here with the same reason (VX_ERR_FORMAT for its IOExceptions and buffer underflows).
// Parsing runs on the host; the arrays then go to the existing build entry points.
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/vx.h"
#include "internal.h"

namespace vx {
namespace {

constexpr uint32_t kMagicQuantized = 0x5A545156u;  // FileFormat.MAGIC_QUANTIZED
constexpr int32_t kVersionQuantized = 1;            // FileFormat.VERSION_QUANTIZED
constexpr int kQuantizedHeader = 20;                // QuantizedVectorsCodec.COMMON_HEADER_SIZE

// QuantizerKind ordinals (vectors-db/.../QuantizerKind.java)
enum QuantizerKind { kNone, kSq8, kSq4, kPq, kBq, kRabitq, kNvq, kTurboquant, kFp16, kExtRabitq, kKinds };
const char* const kKindNames[kKinds] = {"NONE", "SQ8",  "SQ4",        "PQ",  "BQ",
                                        "RABITQ", "NVQ", "TURBOQUANT", "FP16", "EXTENDED_RABITQ"};
// SimilarityFunction names as BuoyIndex.encode writes them (writeUTF(metric.name()))
const char* const kMetricNames[4] = {"EUCLIDEAN", "DOT_PRODUCT", "COSINE", "MAXIMUM_INNER_PRODUCT"};

int failf(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int failf(int status, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return record_failure(status, buf);
}

// Bounds-checked cursor over the file bytes.
struct Cursor {
  const uint8_t* p;
  uint64_t len;
  bool big;  // big-endian fields
  uint64_t pos = 0;
  uint64_t remaining() const { return len - pos; }
  uint32_t u32() {
    uint32_t v;
    if (big) {
      v = (uint32_t)p[pos] << 24 | (uint32_t)p[pos + 1] << 16 | (uint32_t)p[pos + 2] << 8 | p[pos + 3];
    } else {
      std::memcpy(&v, p + pos, 4);
    }
    pos += 4;
    return v;
  }
  int32_t i32() { return (int32_t)u32(); }
  float f32() {
    const uint32_t b = u32();
    float f;
    std::memcpy(&f, &b, 4);
    return f;
  }
  uint16_t u16() {  // big-endian only (DataOutputStream.writeUTF length)
    const uint16_t v = (uint16_t)(p[pos] << 8 | p[pos + 1]);
    pos += 2;
    return v;
  }
  uint8_t u8() { return p[pos++]; }
};

// ---------------------------------------------------------------- quantized.bin
struct QuantizedFile {
  int kind = kNone;
  int32_t dim = 0, count = 0;
  float min_q = 0, max_q = 0;  // SQ
  int bq_mode = 0;             // BinaryMode ordinal: 0 SIGN_BIT, 1 BBQ
  // PQ: numSubspaces, numClusters, the global centroid's offset (0: none), the codebooks
  // concatenated per subspace, and whether the subspaces are computeSubspaceSizesAndOffsets'
  int32_t pq_m = 0, pq_ks = 0;
  uint64_t pq_gc = 0;
  std::vector<float> pq_codebooks;
  bool pq_standard = true;
  uint64_t data = 0;           // offset of the per-vector records
};

// ensureRemaining (QuantizedVectorsCodec.java:1056-1066)
int ensure(const Cursor& c, uint64_t needed, const char* what) {
  if (c.remaining() < needed)
    return failf(VX_ERR_FORMAT, "quantized.bin truncated while reading %s: need %llu bytes, have %llu", what,
                 (unsigned long long)needed, (unsigned long long)c.remaining());
  return VX_OK;
}

int parse_quantized(const uint8_t* bytes, int64_t len, QuantizedFile& f) {
  if (!bytes) return failf(VX_ERR_NULL_POINTER, "bytes must not be null");
  if (len < kQuantizedHeader)
    return failf(VX_ERR_FORMAT, "quantized.bin truncated: expected at least %d header bytes, got %lld",
                 kQuantizedHeader, (long long)len);
  Cursor c{bytes, (uint64_t)len, false};
  const uint32_t magic = c.u32();
  if (magic != kMagicQuantized)
    return failf(VX_ERR_FORMAT, "quantized.bin magic mismatch: expected 0x%08x, got 0x%08x", kMagicQuantized, magic);
  const int32_t version = c.i32();
  if (version != kVersionQuantized)
    return failf(VX_ERR_FORMAT, "quantized.bin version mismatch: expected %d, got %d", kVersionQuantized, version);
  const int32_t kind = c.i32();
  if (kind < 0 || kind >= kKinds) return failf(VX_ERR_FORMAT, "quantized.bin invalid quantizerKind ordinal: %d", kind);
  if (kind == kNone) return failf(VX_ERR_FORMAT, "quantized.bin cannot have quantizerKind NONE");
  f.kind = kind;
  f.dim = c.i32();
  if (f.dim <= 0) return failf(VX_ERR_FORMAT, "quantized.bin dimension must be positive, got %d", f.dim);
  f.count = c.i32();
  if (f.count < 0) return failf(VX_ERR_FORMAT, "quantized.bin vectorCount must be >= 0, got %d", f.count);
  const uint64_t n = (uint64_t)f.count, d = (uint64_t)f.dim;
  switch (kind) {
    case kSq8:
    case kSq4: {  // decodeSQ (:257-296)
      if (int s = ensure(c, 12, "SQ quantizer state")) return s;
      const int32_t bits = c.i32();  // ScalarBits ordinal: 0 INT8, 1 INT4
      if (bits < 0 || bits > 1) return failf(VX_ERR_FORMAT, "quantized.bin invalid ScalarBits ordinal: %d", bits);
      if (kind == kSq8 && bits != 0) return failf(VX_ERR_FORMAT, "quantized.bin SQ8 kind but ScalarBits is INT4");
      if (kind == kSq4 && bits != 1) return failf(VX_ERR_FORMAT, "quantized.bin SQ4 kind but ScalarBits is INT8");
      f.min_q = c.f32();
      f.max_q = c.f32();
      const uint64_t code_bytes = bits == 0 ? d : (d + 1) / 2;  // ScalarBits.encodedByteSize
      if (int s = ensure(c, (code_bytes + 4) * n, "SQ vector data")) return s;
      break;
    }
    case kBq: {  // decodeBQ (:475-518)
      if (int s = ensure(c, 4, "BQ mode ordinal")) return s;
      const int32_t mode = c.i32();
      if (mode < 0 || mode > 1) return failf(VX_ERR_FORMAT, "quantized.bin invalid BinaryMode ordinal: %d", mode);
      f.bq_mode = mode;
      if (mode == 1) {
        if (int s = ensure(c, d * 4, "BQ centroid")) return s;
        c.pos += d * 4;
      }
      const uint64_t per = ((d + 63) / 64) * 8 + (mode == 1 ? 12 : 0);
      if (int s = ensure(c, per * n, "BQ vector data")) return s;
      break;
    }
    case kFp16:  // decodeFp16 (:211-221)
      if (int s = ensure(c, d * 2 * n, "FP16 vector data")) return s;
      break;
    case kPq: {  // decodePQ (:367-420)
      if (int s = ensure(c, 12, "PQ quantizer state header")) return s;
      f.pq_m = c.i32();
      f.pq_ks = c.i32();
      const int32_t has_gc = c.i32();
      if (f.pq_m <= 0) return failf(VX_ERR_FORMAT, "quantized.bin PQ numSubspaces must be positive: %d", f.pq_m);
      if (f.pq_ks <= 0 || f.pq_ks > 256)
        return failf(VX_ERR_FORMAT, "quantized.bin PQ numClusters must be in [1, 256]: %d", f.pq_ks);
      if (has_gc == 1) {
        if (int s = ensure(c, d * 4, "PQ globalCentroid")) return s;
        f.pq_gc = c.pos;
        c.pos += d * 4;
      } else if (has_gc != 0) {
        return failf(VX_ERR_FORMAT, "quantized.bin PQ hasGlobalCentroid must be 0 or 1: %d", has_gc);
      }
      const uint64_t m = (uint64_t)f.pq_m;
      if (int s = ensure(c, m * 8, "PQ subspaceSizesAndOffsets")) return s;
      std::vector<int32_t> sizes(m);
      const int base = f.dim / f.pq_m, rem = f.dim % f.pq_m;
      int expect_off = 0;
      for (uint64_t i = 0; i < m; i++) {
        sizes[i] = c.i32();
        const int32_t off = c.i32();
        if (sizes[i] != base + ((int)i < rem ? 1 : 0) || off != expect_off) f.pq_standard = false;
        expect_off += sizes[i];
      }
      for (uint64_t i = 0; i < m; i++) {
        if (sizes[i] < 0) return failf(VX_ERR_FORMAT, "quantized.bin PQ subspace %d has size %d", (int)i, sizes[i]);
        const uint64_t len = (uint64_t)f.pq_ks * (uint64_t)sizes[i];
        char what[48];
        snprintf(what, sizeof(what), "PQ codebook %d", (int)i);
        if (int s = ensure(c, len * 4, what)) return s;
        for (uint64_t j = 0; j < len; j++) f.pq_codebooks.push_back(c.f32());
      }
      if (int s = ensure(c, n * m, "PQ vector data")) return s;
      break;
    }
    default:
      break;  // validated by the kinds this library serves only
  }
  f.data = c.pos;
  return VX_OK;
}

int unsupported_kind(const QuantizedFile& f) {
  if (f.kind == kBq && f.bq_mode == 1 && f.dim > 2048)
    return failf(VX_ERR_UNSUPPORTED, "quantized.bin BQ in BBQ mode is served up to 2048 dimensions, not %d", f.dim);
  if (f.kind == kPq && (!f.pq_standard || f.pq_m > f.dim))
    return failf(VX_ERR_UNSUPPORTED, "quantized.bin PQ subspaces differ from computeSubspaceSizesAndOffsets");
  if (f.kind != kSq8 && f.kind != kSq4 && f.kind != kBq && f.kind != kFp16 && f.kind != kPq)
    return failf(VX_ERR_UNSUPPORTED,
                 "quantized.bin kind %s is not served here (SQ8, SQ4, BQ SIGN_BIT and BBQ, FP16 and PQ are)",
                 kKindNames[f.kind]);
  return VX_OK;
}

// ---------------------------------------------------------------- graph.bin (IVF)
struct IvfFile {
  int32_t nlist = 0, dim = 0, metric = -1;
  std::vector<float> centroids;       // [nlist][dim]
  std::vector<int32_t> spill;         // [nlist] SOAR spill targets (-1: none)
  std::vector<float> radii;           // [nlist] cluster radii (the EUCLIDEAN early exit)
  std::vector<int64_t> offsets;       // [nlist + 1]
  std::vector<int32_t> ordinals;      // partitions, concatenated
  std::vector<int32_t> key_dims;      // [nlist] HARMONY key dimension count of each partition
  bool pq = false;
  int32_t m = 0, ks = 0;
  bool global_centroid = false;
  bool subspaces_standard = true;     // sizes / offsets as computeSubspaceSizesAndOffsets gives them
  std::vector<float> codebooks;       // concatenated per subspace
  int32_t count = 0;                  // coded rows
  const uint8_t* codes = nullptr;     // [count][m], ordinal order
};

int underflow(const char* what) {
  return failf(VX_ERR_FORMAT, "graph.bin truncated while reading %s", what);
}

// BuoyIndex.decode (BuoyIndex.java:150-167): k, dim, metric name, centroids, spill targets,
// cluster sizes, radii.
int parse_buoy(Cursor& c, IvfFile& f) {
  if (c.remaining() < 8) return underflow("the buoy header");
  f.nlist = c.i32();
  f.dim = c.i32();
  if (f.nlist <= 0 || f.dim <= 0)
    return failf(VX_ERR_FORMAT, "graph.bin buoy shape must be positive, got k=%d dim=%d", f.nlist, f.dim);
  if (c.remaining() < 2) return underflow("the buoy metric");
  const uint16_t nlen = c.u16();
  if (c.remaining() < nlen) return underflow("the buoy metric");
  const std::string name(reinterpret_cast<const char*>(c.p + c.pos), nlen);
  c.pos += nlen;
  f.metric = -1;
  for (int i = 0; i < 4; i++)
    if (name == kMetricNames[i]) f.metric = i;
  if (f.metric < 0) return failf(VX_ERR_FORMAT, "graph.bin unknown SimilarityFunction %s", name.c_str());
  const uint64_t k = (uint64_t)f.nlist, d = (uint64_t)f.dim;
  if (c.remaining() / 4 < k * d + 3 * k) return underflow("the buoy vectors");
  f.centroids.resize(k * d);
  for (uint64_t i = 0; i < k * d; i++) f.centroids[i] = c.f32();
  f.spill.resize(k);
  for (uint64_t i = 0; i < k; i++) f.spill[i] = c.i32();
  c.pos += k * 4;  // cluster sizes: not used by the search
  f.radii.resize(k);
  for (uint64_t i = 0; i < k; i++) f.radii[i] = c.f32();
  return VX_OK;
}

int parse_ivf(const uint8_t* bytes, int64_t len, IvfFile& f) {
  if (!bytes) return failf(VX_ERR_NULL_POINTER, "bytes must not be null");
  if (len < 4) return underflow("the buoy length");
  Cursor c{bytes, (uint64_t)len, true};
  const int32_t buoy_len = c.i32();
  if (buoy_len < 0 || (uint64_t)buoy_len > c.remaining()) return underflow("the buoy index");
  {
    Cursor b{bytes + c.pos, (uint64_t)buoy_len, true};
    if (int s = parse_buoy(b, f)) return s;
  }
  c.pos += (uint64_t)buoy_len;
  if (c.remaining() < 4) return underflow("the partition count");
  const int32_t k = c.i32();
  if (k != f.nlist)
    return failf(VX_ERR_FORMAT, "graph.bin holds %d partitions for %d centroids", k, f.nlist);
  f.offsets.assign((size_t)k + 1, 0);
  for (int32_t p = 0; p < k; p++) {
    if (c.remaining() < 4) return underflow("a partition size");
    const int32_t size = c.i32();
    if (size < 0) return failf(VX_ERR_FORMAT, "graph.bin partition %d has negative size %d", p, size);
    if (c.remaining() / 4 < (uint64_t)size + 1) return underflow("partition ordinals");
    const size_t at = f.ordinals.size();
    f.ordinals.resize(at + (size_t)size);  // grows geometrically (an exact reserve per partition would not)
    for (int32_t i = 0; i < size; i++) f.ordinals[at + (size_t)i] = c.i32();
    f.offsets[(size_t)p + 1] = f.offsets[(size_t)p] + size;
    const int32_t kd = c.i32();  // HARMONY key dimensions (0 = none): IVF-flat only, pqSearch ignores them
    if (kd < 0 || c.remaining() / 4 < (uint64_t)kd) return underflow("partition key dimensions");
    c.pos += (uint64_t)kd * 4;
    f.key_dims.push_back(kd);
  }
  // pqFlag: absent on files written before IVF-PQ (treated as 0), else 0 or 1
  const int flag = c.remaining() > 0 ? c.u8() : 0;
  if (flag != 0 && flag != 1) return failf(VX_ERR_INVALID_ARGUMENT, "Unknown IVF pqFlag byte: %d", (int)(int8_t)flag);
  f.pq = flag == 1;
  if (!f.pq) return VX_OK;
  // PQ trailer (IvfIndex.decodePqTrailer, IvfIndex.java:476-500)
  if (c.remaining() < 17) return underflow("the PQ trailer");
  const int32_t pdim = c.i32();
  f.m = c.i32();
  f.ks = c.i32();
  c.f32();  // anisotropic threshold: encoding only
  f.global_centroid = c.u8() == 1;
  if (pdim != f.dim) return failf(VX_ERR_FORMAT, "graph.bin PQ dimension %d differs from the centroids' %d", pdim, f.dim);
  if (f.m <= 0 || f.m > f.dim || f.ks <= 0)
    return failf(VX_ERR_FORMAT, "graph.bin PQ shape M=%d Ks=%d is invalid", f.m, f.ks);
  if (f.global_centroid) {
    if (c.remaining() / 4 < (uint64_t)f.dim) return underflow("the PQ global centroid");
    c.pos += (uint64_t)f.dim * 4;
  }
  // computeSubspaceSizesAndOffsets (ProductQuantizer.java:686-700): the first dim % M
  // subspaces take one extra dimension
  const int base = f.dim / f.m, rem = f.dim % f.m;
  int expect_off = 0;
  for (int32_t s = 0; s < f.m; s++) {
    if (c.remaining() < 8) return underflow("a PQ subspace");
    const int32_t size = c.i32(), off = c.i32();
    if (size != base + (s < rem ? 1 : 0) || off != expect_off) f.subspaces_standard = false;
    if (size <= 0 || size > f.dim) return failf(VX_ERR_FORMAT, "graph.bin PQ subspace %d has size %d", s, size);
    expect_off += size;
    const uint64_t nv = (uint64_t)f.ks * (uint64_t)size;
    if (c.remaining() / 4 < nv) return underflow("a PQ codebook");
    for (uint64_t i = 0; i < nv; i++) f.codebooks.push_back(c.f32());
  }
  if (c.remaining() < 4) return underflow("the PQ code count");
  f.count = c.i32();
  if (f.count < 0) return failf(VX_ERR_FORMAT, "graph.bin PQ code count %d is negative", f.count);
  if (c.remaining() / (uint64_t)f.m < (uint64_t)f.count) return underflow("the PQ codes");
  f.codes = bytes + c.pos;
  for (int32_t o : f.ordinals)
    if (o < 0 || o >= f.count) return failf(VX_ERR_FORMAT, "graph.bin partition ordinal %d outside [0, %d)", o, f.count);
  return VX_OK;
}

int unsupported_ivf(const IvfFile& f) {
  if (!f.pq) return VX_OK;  // IVF-flat
  if (f.global_centroid) return failf(VX_ERR_UNSUPPORTED, "graph.bin PQ with a global centroid is not served here");
  if (!f.subspaces_standard)
    return failf(VX_ERR_UNSUPPORTED, "graph.bin PQ subspaces differ from computeSubspaceSizesAndOffsets");
  if (f.ks > 256) return failf(VX_ERR_UNSUPPORTED, "graph.bin PQ with %d centroids per subspace (at most 256)", f.ks);
  return VX_OK;
}

template <class F>
int guarded_parse(F&& fn) {
  try {
    return fn();
  } catch (const std::bad_alloc&) {
    return failf(VX_ERR_OUT_OF_MEMORY, "host allocation failed while reading the file");
  } catch (...) {
    return failf(VX_ERR_CUDA, "unexpected failure while reading the file");
  }
}

}  // namespace
}  // namespace vx

using namespace vx;

extern "C" {

int vx_quantized_bin_info(const uint8_t* bytes, int64_t len, int32_t* kind_ordinal, int32_t* dim, int64_t* count) {
  return guarded_parse([&]() -> int {
    QuantizedFile f;
    if (int s = parse_quantized(bytes, len, f)) return s;
    if (kind_ordinal) *kind_ordinal = f.kind;
    if (dim) *dim = f.dim;
    if (count) *count = f.count;
    return unsupported_kind(f);
  });
}

int vx_quantized_bin_build(int32_t device, const uint8_t* bytes, int64_t len, int32_t metric,
                           const float* vectors, int64_t row_stride, vx_index** out) {
  return guarded_parse([&]() -> int {
    if (!out) return failf(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    QuantizedFile f;
    if (int s = parse_quantized(bytes, len, f)) return s;
    if (int s = unsupported_kind(f)) return s;
    const uint8_t* data = bytes + f.data;
    const size_t n = (size_t)f.count, d = (size_t)f.dim;
    if (f.kind == kPq) {
      // little-endian floats, as the host; codes [count][numSubspaces] follow the codebooks
      std::vector<float> gc;
      if (f.pq_gc) {
        gc.resize(d);
        std::memcpy(gc.data(), bytes + f.pq_gc, d * 4);
      }
      return vx_pq_build(device, f.pq_codebooks.data(), f.pq_gc ? gc.data() : nullptr, n ? data : nullptr,
                         (int64_t)n, f.dim, f.pq_m, f.pq_ks, metric, vectors, row_stride, out);
    }
    if (f.kind == kSq8) {
      // records are (codes[dim], correction): split into the two arrays vx_sq8_build takes
      std::vector<int8_t> codes(n * d);
      std::vector<float> corr(n);
      for (size_t i = 0; i < n; i++) {
        const uint8_t* r = data + i * (d + 4);
        std::memcpy(&codes[i * d], r, d);
        std::memcpy(&corr[i], r + d, 4);  // little-endian float, as the host
      }
      return vx_sq8_build(device, codes.data(), corr.data(), (int64_t)n, f.dim, f.min_q, f.max_q, metric, vectors,
                          row_stride, out);
    }
    if (f.kind == kSq4) {
      // records are (ceil(dim/2) packed bytes, correction)
      const size_t nb = (d + 1) / 2;
      std::vector<uint8_t> packed(n * nb);
      std::vector<float> corr(n);
      for (size_t i = 0; i < n; i++) {
        const uint8_t* r = data + i * (nb + 4);
        std::memcpy(&packed[i * nb], r, nb);
        std::memcpy(&corr[i], r + nb, 4);
      }
      return vx_sq4_build(device, packed.data(), corr.data(), (int64_t)n, f.dim, f.min_q, f.max_q, metric, vectors,
                          row_stride, out);
    }
    if (f.kind == kBq && f.bq_mode == 1) {
      // BBQ: the centroid after the mode ordinal, then (words, 3 corrections) per vector
      const size_t nw = (d + 63) / 64;
      std::vector<float> cent(d);
      std::memcpy(cent.data(), bytes + kQuantizedHeader + 4, d * 4);
      std::vector<uint64_t> words(n * nw);
      std::vector<float> corr(n * 3);
      for (size_t i = 0; i < n; i++) {
        const uint8_t* r = data + i * (nw * 8 + 12);
        std::memcpy(&words[i * nw], r, nw * 8);
        std::memcpy(&corr[i * 3], r + nw * 8, 12);
      }
      return vx_bbq_build(device, words.data(), corr.data(), cent.data(), (int64_t)n, f.dim, metric, vectors,
                          row_stride, out);
    }
    if (f.kind == kBq) {
      const size_t nw = (d + 63) / 64;
      std::vector<uint64_t> words(n * nw);  // an aligned copy of the little-endian longs
      if (n) std::memcpy(words.data(), data, n * nw * 8);
      return vx_bq_build(device, words.data(), (int64_t)n, f.dim, metric, vectors, row_stride, out);
    }
    std::vector<uint16_t> codes(n * d);  // FP16
    if (n) std::memcpy(codes.data(), data, n * d * 2);
    return vx_fp16_build(device, codes.data(), (int64_t)n, f.dim, metric, vectors, row_stride, out);
  });
}

int vx_ivf_graph_info(const uint8_t* bytes, int64_t len, int32_t* nlist, int32_t* dim, int64_t* count, int32_t* m,
                      int32_t* metric) {
  return guarded_parse([&]() -> int {
    IvfFile f;
    if (int s = parse_ivf(bytes, len, f)) return s;
    if (nlist) *nlist = f.nlist;
    if (dim) *dim = f.dim;
    if (count) *count = f.pq ? (int64_t)f.count : (int64_t)f.ordinals.size();
    if (m) *m = f.pq ? f.m : 0;
    if (metric) *metric = f.metric;
    return unsupported_ivf(f);
  });
}

int vx_ivf_graph_build(int32_t device, const uint8_t* bytes, int64_t len, int32_t metric, const float* vectors,
                       int64_t vector_count, int64_t row_stride, int32_t nprobe, int32_t rescore_factor,
                       vx_index** out) {
  return guarded_parse([&]() -> int {
    if (!out) return failf(VX_ERR_NULL_POINTER, "out must not be null");
    *out = nullptr;
    IvfFile f;
    if (int s = parse_ivf(bytes, len, f)) return s;
    if (int s = unsupported_ivf(f)) return s;
    if (metric == -1) metric = f.metric;
    if (metric != f.metric)
      return failf(VX_ERR_UNSUPPORTED, "graph.bin routes by %s; the index metric %d differs", kMetricNames[f.metric],
                   metric);
    int st;
    if (!f.pq) {  // IVF-flat: IvfIndex.decode scores the caller's vectors
      if (!vectors) return failf(VX_ERR_NULL_POINTER, "an IVF-flat graph.bin needs the vectors");
      st = vx_ivfflat_build(device, f.centroids.data(), f.nlist, f.dim, f.offsets.data(),
                            f.ordinals.empty() ? nullptr : f.ordinals.data(), vectors, vector_count, row_stride,
                            metric, nprobe, out);
    } else {
      if (vectors && vector_count != f.count)
        return failf(VX_ERR_INVALID_ARGUMENT, "%lld vectors for %d PQ codes", (long long)vector_count, f.count);
      st = ivfpq_build_strided(device, f.centroids.data(), f.nlist, f.dim, f.offsets.data(),
                               f.ordinals.empty() ? nullptr : f.ordinals.data(), f.m, f.ks, f.codebooks.data(),
                               f.count ? f.codes : nullptr, f.count, metric, vectors,
                               vectors ? row_stride : f.dim, nprobe, rescore_factor, out);
    }
    if (st != VX_OK) return st;
    // the buoy's own radii and spill targets, as IvfIndex.decode restores them (BuoyIndex.decode),
    // and which IVF-flat partitions carry HARMONY key dimensions
    st = vx_ivf_set_buoy(*out, f.radii.data(), f.spill.data());
    if (st == VX_OK && !f.pq) st = vx_ivf_set_key_dims(*out, f.key_dims.data());
    if (st != VX_OK) {
      vx_index_free(*out);
      *out = nullptr;
    }
    return st;
  });
}

}  // extern "C"
