// GGUF v3 reader (hy-mt-rs src/gguf.rs:50-210): the memory-mapped model file,
// its metadata and tensor table, with the reference's bounds checks and
// type-id profiles; tensors go to the device unchanged through hyq_upload.
// Host code only.
//
// Checks, as gguf.rs: magic and version 3; header counts bounded by the
// bytes left (gguf.rs:304-311); strings at most 64 MiB, arrays at most 16 M
// items; non-finite float metadata rejected; no duplicate keys; alignment a
// power of two <= 65536 (default 32); split files rejected; tensor rank 1-4,
// no zero dimension, offsets aligned; a data section inside the file; legacy
// type ids 40/42 need a Tencent profile, given or recognised by the file's
// SHA-256 (gguf.rs:113-126), and then the architecture, file type and the
// set of types of a Tencent export (gguf.rs:130-151); whole blocks per row;
// no truncated or overlapping tensors.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/hyq.h"
#include "hyq_kernels.h"

namespace {

// ---------------------------------------------------------------------------
// SHA-256 (FIPS 180-4), for recognising the Tencent legacy exports.
// ---------------------------------------------------------------------------
struct Sha256 {
  uint32_t h[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                   0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
  static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
  void block(const uint8_t* p) {
    static const uint32_t k[64] = {
        0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u, 0xab1c5ed5u,
        0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu, 0x9bdc06a7u, 0xc19bf174u,
        0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu, 0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau,
        0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u, 0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u,
        0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu, 0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u,
        0xa2bfe8a1u, 0xa81a664bu, 0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u,
        0x19a4c116u, 0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
        0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u, 0xc67178f2u};
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 | p[4 * i + 3];
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t t1 = hh + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[i] + w[i];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      hh = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h[0] += a;
    h[1] += b;
    h[2] += c;
    h[3] += d;
    h[4] += e;
    h[5] += f;
    h[6] += g;
    h[7] += hh;
  }
  std::string hex(const uint8_t* data, size_t n) {
    size_t i = 0;
    for (; i + 64 <= n; i += 64) block(data + i);
    uint8_t tail[128] = {};
    const size_t r = n - i;
    memcpy(tail, data + i, r);
    tail[r] = 0x80;
    const size_t len = r + 9 <= 64 ? 64 : 128;
    const uint64_t bits = (uint64_t)n * 8;
    for (int b = 0; b < 8; ++b) tail[len - 1 - b] = (uint8_t)(bits >> (8 * b));
    block(tail);
    if (len == 128) block(tail + 64);
    static const char* d = "0123456789abcdef";
    std::string s;
    for (uint32_t v : h)
      for (int b = 28; b >= 0; b -= 4) s.push_back(d[(v >> b) & 15]);
    return s;
  }
};

constexpr const char* kStqSha256 = "cc497fe8f033b52b3b8b00a7669e9661435432f9d4cd43f7ed24400c01507a93";
constexpr const char* kQ2cSha256 = "dcc33bbae9b28d923c8c76a64f6157840841d26f8774f3dfd770d5fabeeb1cd7";

// ---------------------------------------------------------------------------
// Metadata values (the GGUF value types 0-12)
// ---------------------------------------------------------------------------
struct Value {
  int type = -1;           // GGUF type id (9: array)
  bool is_signed = false;  // integer types: the value fits int64
  uint64_t u = 0;
  int64_t i = 0;
  double f = 0;
  bool b = false;
  std::string s;
  std::vector<Value> items;
};

struct Tensor {
  std::string name;
  std::vector<int64_t> dims;
  uint32_t type_id = 0;
  int dtype = 0;
  uint64_t offset = 0, byte_len = 0;
};

struct Fail {
  int code;
  std::string msg;
};

struct Reader {
  const uint8_t* bytes;
  size_t len, pos = 0;
  const uint8_t* take(size_t n) {
    if (n > len - pos) throw Fail{HYQ_E_SHAPE, "truncated GGUF header"};
    const uint8_t* p = bytes + pos;
    pos += n;
    return p;
  }
  uint32_t u32() {
    uint32_t v;
    memcpy(&v, take(4), 4);
    return v;
  }
  uint64_t u64() {
    uint64_t v;
    memcpy(&v, take(8), 8);
    return v;
  }
  uint64_t count(size_t minimum_bytes) {
    const uint64_t n = u64();
    if (n > (len - pos) / minimum_bytes) throw Fail{HYQ_E_SHAPE, "GGUF count exceeds file bounds"};
    return n;
  }
  std::string string() {
    const uint64_t n = count(1);
    if (n > 64ull * 1024 * 1024) throw Fail{HYQ_E_SHAPE, "GGUF string exceeds 64 MiB limit"};
    return std::string(reinterpret_cast<const char*>(take(n)), n);
  }
  Value value(uint32_t kind, int depth = 0) {
    Value v;
    v.type = (int)kind;
    switch (kind) {
      case 0: v.u = *take(1); v.i = (int64_t)v.u; break;
      case 1: v.i = (int8_t)*take(1); v.is_signed = true; break;
      case 2: { uint16_t x; memcpy(&x, take(2), 2); v.u = x; v.i = x; break; }
      case 3: { int16_t x; memcpy(&x, take(2), 2); v.i = x; v.is_signed = true; break; }
      case 4: v.u = u32(); v.i = (int64_t)v.u; break;
      case 5: v.i = (int32_t)u32(); v.is_signed = true; break;
      case 6: {
        float x;
        const uint32_t bits = u32();
        memcpy(&x, &bits, 4);
        if (!std::isfinite(x)) throw Fail{HYQ_E_SHAPE, "non-finite GGUF metadata"};
        v.f = x;
        break;
      }
      case 7: {
        const uint8_t x = *take(1);
        if (x > 1) throw Fail{HYQ_E_SHAPE, "invalid GGUF boolean"};
        v.b = x == 1;
        break;
      }
      case 8: v.s = string(); break;
      case 9: {
        if (depth > 0) throw Fail{HYQ_E_SHAPE, "nested GGUF arrays are not supported"};
        const uint32_t et = u32();
        size_t minimum = 0;
        if (et == 0 || et == 1 || et == 7) minimum = 1;
        else if (et == 2 || et == 3) minimum = 2;
        else if (et >= 4 && et <= 6) minimum = 4;
        else if (et == 8 || (et >= 10 && et <= 12)) minimum = 8;
        else throw Fail{HYQ_E_SHAPE, "unsupported GGUF array element type " + std::to_string(et)};
        const uint64_t n = count(minimum);
        if (n > 16000000) throw Fail{HYQ_E_SHAPE, "GGUF array is too large"};
        v.items.reserve(n);
        for (uint64_t k = 0; k < n; ++k) v.items.push_back(value(et, depth + 1));
        break;
      }
      case 10: v.u = u64(); v.i = (int64_t)v.u; break;
      case 11: v.i = (int64_t)u64(); v.is_signed = true; break;
      case 12: {
        double x;
        const uint64_t bits = u64();
        memcpy(&x, &bits, 8);
        if (!std::isfinite(x)) throw Fail{HYQ_E_SHAPE, "non-finite GGUF metadata"};
        v.f = x;
        break;
      }
      default: throw Fail{HYQ_E_SHAPE, "unsupported GGUF metadata type " + std::to_string(kind)};
    }
    return v;
  }
};

// serde_json's as_u64 / as_f64 on the reference's JSON values
bool as_u64(const Value& v, uint64_t& out) {
  if (v.type == 0 || v.type == 2 || v.type == 4 || v.type == 10) {
    out = v.u;
    return true;
  }
  if (v.type == 1 || v.type == 3 || v.type == 5 || v.type == 11) {
    if (v.i < 0) return false;
    out = (uint64_t)v.i;
    return true;
  }
  return false;
}

bool as_f64(const Value& v, double& out) {
  if (v.type == 6 || v.type == 12) {
    out = v.f;
    return true;
  }
  uint64_t u;
  if (as_u64(v, u)) {
    out = (double)u;
    return true;
  }
  if (v.type == 1 || v.type == 3 || v.type == 5 || v.type == 11) {
    out = (double)v.i;
    return true;
  }
  return false;
}

}  // namespace

struct hyq_gguf {
  const uint8_t* data = nullptr;
  size_t len = 0;
  int profile = HYQ_PROFILE_STANDARD;
  std::map<std::string, Value> metadata;
  std::vector<std::string> keys;  // in file order
  std::map<std::string, Tensor> tensors;
  std::vector<std::string> names;  // in file order
};

namespace {

void parse(hyq_gguf& g, int requested) {
  Reader r{g.data, g.len};
  if (memcmp(r.take(4), "GGUF", 4) != 0) throw Fail{HYQ_E_SHAPE, "not a GGUF file"};
  if (r.u32() != 3) throw Fail{HYQ_E_UNSUPPORTED, "only GGUF v3 is supported"};
  const uint64_t tensor_count = r.count(24);
  const uint64_t kv_count = r.count(13);
  for (uint64_t k = 0; k < kv_count; ++k) {
    std::string key = r.string();
    const uint32_t kind = r.u32();
    Value v = r.value(kind);
    if (!g.metadata.emplace(key, std::move(v)).second) throw Fail{HYQ_E_SHAPE, "duplicate metadata key " + key};
    g.keys.push_back(key);
  }
  uint64_t alignment = 32;
  auto it = g.metadata.find("general.alignment");
  if (it != g.metadata.end() && !as_u64(it->second, alignment)) throw Fail{HYQ_E_SHAPE, "invalid GGUF alignment"};
  if (alignment == 0 || (alignment & (alignment - 1)) || alignment > 65536)
    throw Fail{HYQ_E_SHAPE, "invalid GGUF alignment " + std::to_string(alignment)};
  it = g.metadata.find("split.count");
  if (it != g.metadata.end()) {
    uint64_t n = 0;
    if (!as_u64(it->second, n) || n != 1)
      throw Fail{HYQ_E_UNSUPPORTED, "split GGUF files are not supported; supply a merged file"};
  }
  struct Raw {
    std::string name;
    std::vector<int64_t> dims;
    uint32_t type_id;
    uint64_t offset;
  };
  std::vector<Raw> raw;
  raw.reserve(tensor_count);
  for (uint64_t t = 0; t < tensor_count; ++t) {
    Raw x;
    x.name = r.string();
    const uint32_t rank = r.u32();
    if (rank < 1 || rank > 4) throw Fail{HYQ_E_SHAPE, "invalid rank for tensor " + x.name};
    for (uint32_t d = 0; d < rank; ++d) {
      const uint64_t dim = r.u64();
      if (dim == 0) throw Fail{HYQ_E_SHAPE, "zero dimension in tensor " + x.name};
      if (dim > (uint64_t)INT64_MAX) throw Fail{HYQ_E_SHAPE, "tensor dimension too large"};
      x.dims.push_back((int64_t)dim);
    }
    x.type_id = r.u32();
    x.offset = r.u64();
    if (x.offset % alignment) throw Fail{HYQ_E_SHAPE, "unaligned tensor " + x.name};
    raw.push_back(std::move(x));
  }
  if (r.pos > SIZE_MAX - (alignment - 1)) throw Fail{HYQ_E_SHAPE, "offset overflow"};
  const uint64_t data_start = (r.pos + alignment - 1) & ~(alignment - 1);
  if (data_start > g.len) throw Fail{HYQ_E_SHAPE, "missing tensor data"};
  const bool legacy = std::any_of(raw.begin(), raw.end(), [](const Raw& x) { return x.type_id == 40 || x.type_id == 42; });
  int profile = requested;
  if (requested == HYQ_PROFILE_AUTO) {
    if (legacy) {
      const std::string digest = Sha256().hex(g.data, g.len);
      if (digest == kQ2cSha256) profile = HYQ_PROFILE_TENCENT_Q2_0C;
      else if (digest == kStqSha256) profile = HYQ_PROFILE_TENCENT_STQ1;
      else
        throw Fail{HYQ_E_INVALID, "ambiguous GGUF type 40/42 in an unrecognized file (SHA256 " + digest +
                                      "); open it with the Tencent profile of a known legacy export"};
    } else {
      profile = HYQ_PROFILE_STANDARD;
    }
  }
  if (profile == HYQ_PROFILE_TENCENT_Q2_0C || profile == HYQ_PROFILE_TENCENT_STQ1) {
    it = g.metadata.find("general.architecture");
    if (it == g.metadata.end() || it->second.type != 8 || it->second.s != "hunyuan-dense")
      throw Fail{HYQ_E_INVALID, "Tencent low-bit profiles require hunyuan-dense"};
    const uint32_t id = profile == HYQ_PROFILE_TENCENT_Q2_0C ? 40 : 42;
    const uint64_t file_type = profile == HYQ_PROFILE_TENCENT_Q2_0C ? 39 : 41;
    uint64_t ft = 0;
    it = g.metadata.find("general.file_type");
    if (it == g.metadata.end() || !as_u64(it->second, ft) || ft != file_type)
      throw Fail{HYQ_E_INVALID, "incompatible Tencent general.file_type"};
    if (!std::any_of(raw.begin(), raw.end(), [&](const Raw& x) { return x.type_id == id; }))
      throw Fail{HYQ_E_INVALID, "file has no tensors for selected Tencent profile"};
    for (const Raw& x : raw)
      if (x.type_id != 0 && x.type_id != 14 && x.type_id != id)
        throw Fail{HYQ_E_INVALID, "unexpected mixed types in Tencent legacy export"};
  }
  g.profile = profile;
  std::vector<std::pair<uint64_t, uint64_t>> extents;
  std::vector<std::string> extent_names;
  for (Raw& x : raw) {
    int dtype = 0;
    if (hyq_dtype_from_id(x.type_id, profile, &dtype) != HYQ_OK)
      throw Fail{HYQ_E_UNSUPPORTED, "tensor " + x.name + ": unsupported GGUF tensor type " + std::to_string(x.type_id)};
    const int64_t bl = hyq_block_len(dtype), bb = hyq_block_bytes(dtype);
    if (x.dims[0] % bl) throw Fail{HYQ_E_SHAPE, "tensor " + x.name + " has a partial quantization block in its row"};
    uint64_t elements = 1;
    for (int64_t d : x.dims) {
      if (elements > UINT64_MAX / (uint64_t)d) throw Fail{HYQ_E_SHAPE, "tensor element count overflow"};
      elements *= (uint64_t)d;
    }
    if (elements / bl > UINT64_MAX / bb) throw Fail{HYQ_E_SHAPE, "tensor byte count overflow"};
    const uint64_t byte_len = elements / bl * bb;
    if (x.offset > UINT64_MAX - data_start) throw Fail{HYQ_E_SHAPE, "tensor offset overflow"};
    const uint64_t offset = data_start + x.offset;
    if (byte_len > UINT64_MAX - offset) throw Fail{HYQ_E_SHAPE, "tensor end overflow"};
    const uint64_t end = offset + byte_len;
    if (end > g.len)
      throw Fail{HYQ_E_SHAPE, "truncated tensor " + x.name + ": end " + std::to_string(end) + ", file length " +
                                  std::to_string(g.len)};
    extents.push_back({offset, end});
    extent_names.push_back(x.name);
    Tensor t;
    t.name = x.name;
    t.dims = x.dims;
    t.type_id = x.type_id;
    t.dtype = dtype;
    t.offset = offset;
    t.byte_len = byte_len;
    if (!g.tensors.emplace(x.name, t).second) throw Fail{HYQ_E_SHAPE, "duplicate tensor " + x.name};
    g.names.push_back(x.name);
  }
  std::vector<size_t> order(extents.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = i;
  std::sort(order.begin(), order.end(), [&](size_t a, size_t b) { return extents[a].first < extents[b].first; });
  for (size_t i = 1; i < order.size(); ++i)
    if (extents[order[i - 1]].second > extents[order[i]].first)
      throw Fail{HYQ_E_SHAPE, "overlapping tensors " + extent_names[order[i - 1]] + " and " + extent_names[order[i]]};
}

const Value* meta(const hyq_gguf* g, const char* key) {
  if (!g || !key) return nullptr;
  auto it = g->metadata.find(key);
  return it == g->metadata.end() ? nullptr : &it->second;
}

}  // namespace

extern "C" {

int hyq_gguf_open(const char* path, int profile, hyq_gguf** out) {
  if (!path || !out) return hyq::api_fail(HYQ_E_INVALID, "gguf_open: null pointer");
  *out = nullptr;
  if (profile < 0 || profile > HYQ_PROFILE_TENCENT_STQ1) return hyq::api_fail(HYQ_E_INVALID, "gguf_open: profile");
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return hyq::api_fail(HYQ_E_INVALID, "opening %s: %s", path, strerror(errno));
  struct stat st {};
  if (fstat(fd, &st) != 0) {
    close(fd);
    return hyq::api_fail(HYQ_E_INVALID, "stat %s: %s", path, strerror(errno));
  }
  std::unique_ptr<hyq_gguf> g(new hyq_gguf());
  g->len = (size_t)st.st_size;
  if (g->len > 0) {
    void* m = mmap(nullptr, g->len, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
      close(fd);
      return hyq::api_fail(HYQ_E_INVALID, "mapping %s: %s", path, strerror(errno));
    }
    g->data = static_cast<const uint8_t*>(m);
  }
  close(fd);
  try {
    parse(*g, profile);
  } catch (const Fail& f) {
    if (g->data) munmap(const_cast<uint8_t*>(g->data), g->len);
    return hyq::api_fail(f.code, "%s: %s", path, f.msg.c_str());
  } catch (const std::exception& e) {
    if (g->data) munmap(const_cast<uint8_t*>(g->data), g->len);
    return hyq::api_fail(HYQ_E_INVALID, "%s: %s", path, e.what());
  }
  *out = g.release();
  return HYQ_OK;
}

void hyq_gguf_close(hyq_gguf* g) {
  if (!g) return;
  if (g->data) munmap(const_cast<uint8_t*>(g->data), g->len);
  delete g;
}

int hyq_gguf_profile(const hyq_gguf* g) { return g ? g->profile : HYQ_E_INVALID; }

int64_t hyq_gguf_tensor_count(const hyq_gguf* g) { return g ? (int64_t)g->names.size() : HYQ_E_INVALID; }

int hyq_gguf_tensor_name(const hyq_gguf* g, int64_t index, const char** name) {
  if (!g || !name || index < 0 || index >= (int64_t)g->names.size())
    return hyq::api_fail(HYQ_E_INVALID, "gguf_tensor_name: bad argument");
  *name = g->names[(size_t)index].c_str();
  return HYQ_OK;
}

int hyq_gguf_tensor_info(const hyq_gguf* g, const char* name, int* dtype, uint32_t* type_id, int* ndim,
                         int64_t* dims, uint64_t* offset, uint64_t* byte_len) {
  if (!g || !name) return hyq::api_fail(HYQ_E_INVALID, "gguf_tensor_info: null pointer");
  auto it = g->tensors.find(name);
  if (it == g->tensors.end()) return hyq::api_fail(HYQ_E_INVALID, "missing tensor %s", name);
  const Tensor& t = it->second;
  if (dtype) *dtype = t.dtype;
  if (type_id) *type_id = t.type_id;
  if (ndim) *ndim = (int)t.dims.size();
  if (dims)
    for (size_t d = 0; d < 4; ++d) dims[d] = d < t.dims.size() ? t.dims[d] : 0;
  if (offset) *offset = t.offset;
  if (byte_len) *byte_len = t.byte_len;
  return HYQ_OK;
}

int hyq_gguf_tensor_data(const hyq_gguf* g, const char* name, const void** data, size_t* bytes) {
  if (!g || !name || !data) return hyq::api_fail(HYQ_E_INVALID, "gguf_tensor_data: null pointer");
  auto it = g->tensors.find(name);
  if (it == g->tensors.end()) return hyq::api_fail(HYQ_E_INVALID, "missing tensor %s", name);
  *data = g->data + it->second.offset;
  if (bytes) *bytes = (size_t)it->second.byte_len;
  return HYQ_OK;
}

int hyq_gguf_upload(const hyq_gguf* g, const char* name, hyq_weight** out) {
  if (!g || !name || !out) return hyq::api_fail(HYQ_E_INVALID, "gguf_upload: null pointer");
  auto it = g->tensors.find(name);
  if (it == g->tensors.end()) return hyq::api_fail(HYQ_E_INVALID, "missing tensor %s", name);
  const Tensor& t = it->second;
  if (t.dims.size() > 3) return hyq::api_fail(HYQ_E_UNSUPPORTED, "tensor %s: rank %d", name, (int)t.dims.size());
  return hyq_upload(g->data + t.offset, (size_t)t.byte_len, t.dtype, (int)t.dims.size(), t.dims.data(), out);
}

int64_t hyq_gguf_meta_count(const hyq_gguf* g) { return g ? (int64_t)g->keys.size() : HYQ_E_INVALID; }

int hyq_gguf_meta_key(const hyq_gguf* g, int64_t index, const char** key, int* type) {
  if (!g || !key || index < 0 || index >= (int64_t)g->keys.size())
    return hyq::api_fail(HYQ_E_INVALID, "gguf_meta_key: bad argument");
  *key = g->keys[(size_t)index].c_str();
  if (type) *type = g->metadata.at(g->keys[(size_t)index]).type;
  return HYQ_OK;
}

int hyq_gguf_meta_u64(const hyq_gguf* g, const char* key, uint64_t* out) {
  const Value* v = meta(g, key);
  if (!v || !out || !as_u64(*v, *out))
    return hyq::api_fail(HYQ_E_INVALID, "missing or invalid integer metadata %s", key ? key : "");
  return HYQ_OK;
}

int hyq_gguf_meta_f64(const hyq_gguf* g, const char* key, double* out) {
  const Value* v = meta(g, key);
  if (!v || !out || !as_f64(*v, *out))
    return hyq::api_fail(HYQ_E_INVALID, "missing or invalid float metadata %s", key ? key : "");
  return HYQ_OK;
}

int hyq_gguf_meta_bool(const hyq_gguf* g, const char* key, int* out) {
  const Value* v = meta(g, key);
  if (!v || !out || v->type != 7)
    return hyq::api_fail(HYQ_E_INVALID, "missing or invalid boolean metadata %s", key ? key : "");
  *out = v->b ? 1 : 0;
  return HYQ_OK;
}

int hyq_gguf_meta_str(const hyq_gguf* g, const char* key, const char** s, size_t* len) {
  const Value* v = meta(g, key);
  if (!v || !s || v->type != 8)
    return hyq::api_fail(HYQ_E_INVALID, "missing or invalid string metadata %s", key ? key : "");
  *s = v->s.c_str();
  if (len) *len = v->s.size();
  return HYQ_OK;
}

int hyq_gguf_meta_array_len(const hyq_gguf* g, const char* key, int64_t* n) {
  const Value* v = meta(g, key);
  if (!v || !n || v->type != 9)
    return hyq::api_fail(HYQ_E_INVALID, "missing or invalid array metadata %s", key ? key : "");
  *n = (int64_t)v->items.size();
  return HYQ_OK;
}

}  // extern "C"
