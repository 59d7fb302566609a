// GGUF file reader for the Q8_0 linears: header, metadata key/values, tensor infos and
// tensor bytes, and the upload of a Q8_0 tensor into a device weight.
//
// Replaces the reader the reference gets from candle's `quantized::gguf_file`
// (candle-core 0.11.0, not vendored): `Content::read` at
// crates/voxcpm/src/weights.rs:31-33, `content.tensor(file, name, device)` at :100 and
// `content.metadata.get(name)` at :117-123, with the typed checks of :124-137.  The
// format follows the published GGUF specification (versions 2 and 3, little-endian):
//   u32 magic "GGUF" | u32 version | u64 tensor_count | u64 kv_count
//   kv_count x { string key | u32 value_type | value }
//   tensor_count x { string name | u32 n_dims | u64 ne[n_dims] | u32 ggml_type | u64 offset }
//   padding to general.alignment (default 32) | tensor data (offsets relative to here)
// where a string is { u64 length | bytes } and an array value is
// { u32 element_type | u64 count | elements }.
//
// The file is memory-mapped read-only; every length, count, dimension and offset is
// checked against the mapping before it is used, so a truncated or malformed file
// yields Q8LIN_ERR_FORMAT, never an out-of-bounds read.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "internal.h"
#include "q8lin.h"

struct q8lin_gguf {
  const uint8_t* base = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  uint64_t alignment = 32;
  uint64_t data_start = 0;
  struct Value {
    uint32_t type = 0;
    uint64_t u = 0;  // unsigned / bool payload
    int64_t i = 0;   // signed payload
    double f = 0.0;  // float payload
    uint64_t str_off = 0, str_len = 0;           // string: bytes in the mapping
    uint32_t elem_type = 0;                       // array
    uint64_t count = 0, elems_off = 0, elems_bytes = 0;
  };
  std::unordered_map<std::string, Value> kv;
  struct Tensor {
    std::string name;
    uint32_t type = 0;
    uint32_t n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint64_t offset = 0;  // absolute, in the mapping
    uint64_t nbytes = 0;
  };
  std::vector<Tensor> tensors;
  std::unordered_map<std::string, int64_t> by_name;
};

namespace q8lin {
namespace {

enum : uint32_t {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
  kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};

constexpr uint32_t kMagic = 0x46554747u;  // "GGUF" read as a little-endian u32
constexpr int kMaxDims = 4;
constexpr int kMaxArrayDepth = 8;

size_t scalar_size(uint32_t t) {
  switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return 0;
  }
}

// Bytes of a ggml tensor type: (elements per block, bytes per block) from the published
// block definitions; 0 for types this reader cannot size.
bool type_block(uint32_t t, int64_t* elems, int64_t* bytes) {
  switch (t) {
    case Q8LIN_GGML_F32: *elems = 1; *bytes = 4; return true;
    case Q8LIN_GGML_F16: *elems = 1; *bytes = 2; return true;
    case 2: *elems = 32; *bytes = 18; return true;    // Q4_0 {f16 d; u8 qs[16]}
    case 3: *elems = 32; *bytes = 20; return true;    // Q4_1 {f16 d, m; u8 qs[16]}
    case 6: *elems = 32; *bytes = 22; return true;    // Q5_0 {f16 d; u8 qh[4]; u8 qs[16]}
    case 7: *elems = 32; *bytes = 24; return true;    // Q5_1 {f16 d, m; u8 qh[4]; u8 qs[16]}
    case Q8LIN_GGML_Q8_0: *elems = 32; *bytes = 34; return true;  // {f16 d; i8 qs[32]}
    case 9: *elems = 32; *bytes = 36; return true;    // Q8_1 {f16 d, s; i8 qs[32]}
    case 10: *elems = 256; *bytes = 84; return true;  // Q2_K
    case 11: *elems = 256; *bytes = 110; return true; // Q3_K
    case 12: *elems = 256; *bytes = 144; return true; // Q4_K
    case 13: *elems = 256; *bytes = 176; return true; // Q5_K
    case 14: *elems = 256; *bytes = 210; return true; // Q6_K
    case 15: *elems = 256; *bytes = 292; return true; // Q8_K
    case 24: *elems = 1; *bytes = 1; return true;     // I8
    case 25: *elems = 1; *bytes = 2; return true;     // I16
    case 26: *elems = 1; *bytes = 4; return true;     // I32
    case 27: *elems = 1; *bytes = 8; return true;     // I64
    case 28: *elems = 1; *bytes = 8; return true;     // F64
    case Q8LIN_GGML_BF16: *elems = 1; *bytes = 2; return true;
    default: return false;
  }
}

class Cursor {
 public:
  Cursor(const uint8_t* b, size_t n) : b_(b), n_(n) {}
  bool take(size_t k, const uint8_t** p) {
    if (k > n_ - pos_) return false;
    *p = b_ + pos_;
    pos_ += k;
    return true;
  }
  template <typename T>
  bool get(T* v) {
    const uint8_t* p;
    if (!take(sizeof(T), &p)) return false;
    std::memcpy(v, p, sizeof(T));
    return true;
  }
  bool str(uint64_t* off, uint64_t* len) {
    uint64_t l;
    const uint8_t* p;
    if (!get(&l) || l > n_ - pos_) return false;
    *off = pos_;
    *len = l;
    return take((size_t)l, &p);
  }
  size_t pos() const { return pos_; }

 private:
  const uint8_t* b_;
  size_t n_;
  size_t pos_ = 0;
};

bool skip_value(Cursor& c, uint32_t t, int depth);

bool skip_array(Cursor& c, int depth, uint32_t* et, uint64_t* count, uint64_t* off, uint64_t* bytes) {
  if (depth > kMaxArrayDepth) return false;
  if (!c.get(et) || !c.get(count)) return false;
  *off = c.pos();
  const size_t es = scalar_size(*et);
  if (es) {
    const uint8_t* p;
    if (*count > (SIZE_MAX / es)) return false;
    if (!c.take((size_t)(*count * es), &p)) return false;
  } else if (*et == kString || *et == kArray) {
    for (uint64_t i = 0; i < *count; ++i)
      if (!skip_value(c, *et, depth + 1)) return false;
  } else {
    return false;
  }
  *bytes = c.pos() - *off;
  return true;
}

bool skip_value(Cursor& c, uint32_t t, int depth) {
  if (t == kString) {
    uint64_t o, l;
    return c.str(&o, &l);
  }
  if (t == kArray) {
    uint32_t et;
    uint64_t n, o, b;
    return skip_array(c, depth, &et, &n, &o, &b);
  }
  const size_t es = scalar_size(t);
  const uint8_t* p;
  return es && c.take(es, &p);
}

bool read_value(Cursor& c, uint32_t t, q8lin_gguf::Value* v) {
  v->type = t;
  switch (t) {
    case kU8: { uint8_t x; if (!c.get(&x)) return false; v->u = x; v->i = x; v->f = x; return true; }
    case kI8: { int8_t x; if (!c.get(&x)) return false; v->i = x; v->u = (uint64_t)(int64_t)x; v->f = x; return true; }
    case kU16: { uint16_t x; if (!c.get(&x)) return false; v->u = x; v->i = x; v->f = x; return true; }
    case kI16: { int16_t x; if (!c.get(&x)) return false; v->i = x; v->u = (uint64_t)(int64_t)x; v->f = x; return true; }
    case kU32: { uint32_t x; if (!c.get(&x)) return false; v->u = x; v->i = x; v->f = x; return true; }
    case kI32: { int32_t x; if (!c.get(&x)) return false; v->i = x; v->u = (uint64_t)(int64_t)x; v->f = x; return true; }
    case kU64: { uint64_t x; if (!c.get(&x)) return false; v->u = x; v->i = (int64_t)x; v->f = (double)x; return true; }
    case kI64: { int64_t x; if (!c.get(&x)) return false; v->i = x; v->u = (uint64_t)x; v->f = (double)x; return true; }
    case kF32: { float x; if (!c.get(&x)) return false; v->f = x; return true; }
    case kF64: { double x; if (!c.get(&x)) return false; v->f = x; return true; }
    case kBool: {
      uint8_t x;
      if (!c.get(&x) || x > 1) return false;
      v->u = x;
      v->i = x;
      return true;
    }
    case kString: return c.str(&v->str_off, &v->str_len);
    case kArray: return skip_array(c, 0, &v->elem_type, &v->count, &v->elems_off, &v->elems_bytes);
    default: return false;
  }
}

bool is_integer(uint32_t t) {
  return t == kU8 || t == kI8 || t == kU16 || t == kI16 || t == kU32 || t == kI32 || t == kU64 || t == kI64;
}
bool is_signed(uint32_t t) { return t == kI8 || t == kI16 || t == kI32 || t == kI64; }

int format_error(const std::string& path, const std::string& what) {
  return fail(Q8LIN_ERR_FORMAT, "GGUF " + path + ": " + what);
}

int parse(q8lin_gguf* g, const std::string& path) {
  Cursor c(g->base, g->size);
  uint32_t magic = 0;
  uint64_t n_tensors = 0, n_kv = 0;
  if (!c.get(&magic) || magic != kMagic) return format_error(path, "not a GGUF file (bad magic)");
  if (!c.get(&g->version)) return format_error(path, "truncated header");
  if (g->version != 2 && g->version != 3)
    return format_error(path, "unsupported GGUF version " + std::to_string(g->version) + " (2 and 3 are read)");
  if (!c.get(&n_tensors) || !c.get(&n_kv)) return format_error(path, "truncated header");
  // every key/value takes at least 12 bytes and every tensor info at least 24
  if (n_kv > g->size / 12 || n_tensors > g->size / 24) return format_error(path, "counts exceed the file size");
  for (uint64_t i = 0; i < n_kv; ++i) {
    uint64_t ko, kl;
    uint32_t t;
    if (!c.str(&ko, &kl)) return format_error(path, "truncated metadata key " + std::to_string(i));
    std::string key(reinterpret_cast<const char*>(g->base + ko), (size_t)kl);
    q8lin_gguf::Value v;
    if (!c.get(&t) || !read_value(c, t, &v))
      return format_error(path, "malformed metadata value for key '" + key + "'");
    if (!g->kv.emplace(key, v).second) return format_error(path, "duplicate metadata key '" + key + "'");
  }
  auto al = g->kv.find("general.alignment");
  if (al != g->kv.end()) {
    const q8lin_gguf::Value& v = al->second;
    if (!is_integer(v.type) || (is_signed(v.type) && v.i <= 0) || v.u == 0 || v.u > (1u << 30) ||
        (v.u & (v.u - 1)))
      return format_error(path, "general.alignment must be a positive power of two");
    g->alignment = v.u;
  }
  g->tensors.reserve((size_t)n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    q8lin_gguf::Tensor t;
    uint64_t no, nl;
    if (!c.str(&no, &nl)) return format_error(path, "truncated tensor info " + std::to_string(i));
    t.name.assign(reinterpret_cast<const char*>(g->base + no), (size_t)nl);
    if (!c.get(&t.n_dims) || t.n_dims == 0 || t.n_dims > kMaxDims)
      return format_error(path, "tensor '" + t.name + "' has an invalid dimension count");
    int64_t numel = 1;
    for (uint32_t d = 0; d < t.n_dims; ++d) {
      uint64_t ne;
      if (!c.get(&ne)) return format_error(path, "truncated tensor info '" + t.name + "'");
      if (ne == 0 || ne > ((uint64_t)1 << 40) || (uint64_t)numel > ((uint64_t)1 << 42) / ne)
        return format_error(path, "tensor '" + t.name + "' has an invalid shape");
      t.ne[d] = (int64_t)ne;
      numel *= (int64_t)ne;
    }
    if (!c.get(&t.type) || !c.get(&t.offset)) return format_error(path, "truncated tensor info '" + t.name + "'");
    int64_t be = 0, bb = 0;
    if (type_block(t.type, &be, &bb)) {
      if (t.ne[0] % be) return format_error(path, "tensor '" + t.name + "': ne[0] is not a multiple of the block size");
      t.nbytes = (uint64_t)(numel / be) * (uint64_t)bb;
    } else {
      t.nbytes = 0;  // unknown type: listed, but its bytes cannot be read
    }
    if (t.offset % g->alignment) return format_error(path, "tensor '" + t.name + "' offset is not aligned");
    if (!g->by_name.emplace(t.name, (int64_t)g->tensors.size()).second)
      return format_error(path, "duplicate tensor name '" + t.name + "'");
    g->tensors.push_back(std::move(t));
  }
  g->data_start = (c.pos() + g->alignment - 1) / g->alignment * g->alignment;
  for (q8lin_gguf::Tensor& t : g->tensors) {
    if (t.offset > g->size || g->data_start > g->size - t.offset ||
        t.nbytes > g->size - g->data_start - t.offset)
      return format_error(path, "tensor '" + t.name + "' extends past the end of the file");
    t.offset += g->data_start;
  }
  return Q8LIN_OK;
}

const q8lin_gguf::Value* lookup(const q8lin_gguf* g, const char* key) {
  if (!g || !key) return nullptr;
  auto it = g->kv.find(key);
  return it == g->kv.end() ? nullptr : &it->second;
}

int missing_key(const char* key) {
  return fail(Q8LIN_ERR_NOT_FOUND, std::string("missing GGUF metadata ") + (key ? key : "(null)"));
}

}  // namespace
}  // namespace q8lin

using namespace q8lin;

extern "C" {

int q8lin_gguf_open(const char* path, q8lin_gguf** out) {
  if (!out) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "out is null");
  *out = nullptr;
  if (!path) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "path is null");
  const int fd = ::open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return fail(Q8LIN_ERR_IO, std::string("cannot open ") + path + ": " + std::strerror(errno));
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    ::close(fd);
    return fail(Q8LIN_ERR_FORMAT, std::string("GGUF ") + path + ": empty or unreadable file");
  }
  void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (m == MAP_FAILED) return fail(Q8LIN_ERR_IO, std::string("cannot map ") + path + ": " + std::strerror(errno));
  q8lin_gguf* g = new q8lin_gguf();
  g->base = static_cast<const uint8_t*>(m);
  g->size = (size_t)st.st_size;
  const int rc = parse(g, path);
  if (rc != Q8LIN_OK) {
    munmap(const_cast<uint8_t*>(g->base), g->size);
    delete g;
    return rc;
  }
  *out = g;
  return Q8LIN_OK;
}

int q8lin_gguf_close(q8lin_gguf* g) {
  if (!g) return Q8LIN_OK;
  munmap(const_cast<uint8_t*>(g->base), g->size);
  delete g;
  return Q8LIN_OK;
}

int q8lin_gguf_version(const q8lin_gguf* g, uint32_t* version) {
  if (!g || !version) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "null argument");
  *version = g->version;
  return Q8LIN_OK;
}

int64_t q8lin_gguf_tensor_count(const q8lin_gguf* g) { return g ? (int64_t)g->tensors.size() : -1; }

int64_t q8lin_gguf_metadata_count(const q8lin_gguf* g) { return g ? (int64_t)g->kv.size() : -1; }

int q8lin_gguf_find_tensor(const q8lin_gguf* g, const char* name, int64_t* index) {
  if (!g || !name || !index) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "null argument");
  auto it = g->by_name.find(name);
  if (it == g->by_name.end()) return fail(Q8LIN_ERR_NOT_FOUND, std::string("cannot find tensor info for ") + name);
  *index = it->second;
  return Q8LIN_OK;
}

int q8lin_gguf_tensor_info(const q8lin_gguf* g, int64_t index, const char** name, uint32_t* ggml_type,
                           uint32_t* n_dims, int64_t* dims, uint64_t* nbytes) {
  if (!g) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "gguf handle is null");
  if (index < 0 || index >= (int64_t)g->tensors.size()) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "tensor index out of range");
  const q8lin_gguf::Tensor& t = g->tensors[(size_t)index];
  if (name) *name = t.name.c_str();
  if (ggml_type) *ggml_type = t.type;
  if (n_dims) *n_dims = t.n_dims;
  if (dims)
    for (int d = 0; d < kMaxDims; ++d) dims[d] = t.ne[d];
  if (nbytes) *nbytes = t.nbytes;
  return Q8LIN_OK;
}

int q8lin_gguf_tensor_data(const q8lin_gguf* g, int64_t index, const void** data, uint64_t* nbytes) {
  if (!g || !data) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "null argument");
  if (index < 0 || index >= (int64_t)g->tensors.size()) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "tensor index out of range");
  const q8lin_gguf::Tensor& t = g->tensors[(size_t)index];
  if (t.nbytes == 0)
    return fail(Q8LIN_ERR_FORMAT, "tensor '" + t.name + "' has ggml type " + std::to_string(t.type) + ", which this reader cannot size");
  *data = g->base + t.offset;
  if (nbytes) *nbytes = t.nbytes;
  return Q8LIN_OK;
}

int q8lin_gguf_metadata_type(const q8lin_gguf* g, const char* key, uint32_t* value_type) {
  if (!g || !key || !value_type) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "null argument");
  const q8lin_gguf::Value* v = lookup(g, key);
  if (!v) return missing_key(key);
  *value_type = v->type;
  return Q8LIN_OK;
}

int q8lin_gguf_metadata_u32(const q8lin_gguf* g, const char* key, uint32_t* value) {
  if (!g || !key || !value) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "null argument");
  const q8lin_gguf::Value* v = lookup(g, key);
  if (!v) return missing_key(key);
  if (v->type != kU32) return fail(Q8LIN_ERR_FORMAT, std::string("GGUF metadata ") + key + " is not a u32");
  *value = (uint32_t)v->u;
  return Q8LIN_OK;
}

int q8lin_gguf_metadata_i64(const q8lin_gguf* g, const char* key, int64_t* value) {
  if (!g || !key || !value) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "null argument");
  const q8lin_gguf::Value* v = lookup(g, key);
  if (!v) return missing_key(key);
  if (!is_integer(v->type) && v->type != kBool)
    return fail(Q8LIN_ERR_FORMAT, std::string("GGUF metadata ") + key + " is not an integer");
  if (v->type == kU64 && v->u > (uint64_t)INT64_MAX)
    return fail(Q8LIN_ERR_FORMAT, std::string("GGUF metadata ") + key + " does not fit in an i64");
  *value = v->i;
  return Q8LIN_OK;
}

int q8lin_gguf_metadata_f64(const q8lin_gguf* g, const char* key, double* value) {
  if (!g || !key || !value) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "null argument");
  const q8lin_gguf::Value* v = lookup(g, key);
  if (!v) return missing_key(key);
  if (v->type == kString || v->type == kArray)
    return fail(Q8LIN_ERR_FORMAT, std::string("GGUF metadata ") + key + " is not a number");
  *value = v->f;
  return Q8LIN_OK;
}

int q8lin_gguf_metadata_string(const q8lin_gguf* g, const char* key, const char** data, uint64_t* len) {
  if (!g || !key || !data || !len) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "null argument");
  const q8lin_gguf::Value* v = lookup(g, key);
  if (!v) return missing_key(key);
  if (v->type != kString) return fail(Q8LIN_ERR_FORMAT, std::string("GGUF metadata ") + key + " is not a string");
  *data = reinterpret_cast<const char*>(g->base + v->str_off);
  *len = v->str_len;
  return Q8LIN_OK;
}

int q8lin_gguf_metadata_array(const q8lin_gguf* g, const char* key, uint32_t* elem_type, uint64_t* count,
                              const void** data, uint64_t* nbytes) {
  if (!g || !key || !elem_type || !count) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "null argument");
  const q8lin_gguf::Value* v = lookup(g, key);
  if (!v) return missing_key(key);
  if (v->type != kArray) return fail(Q8LIN_ERR_FORMAT, std::string("GGUF metadata ") + key + " is not an array");
  *elem_type = v->elem_type;
  *count = v->count;
  if (data) *data = g->base + v->elems_off;
  if (nbytes) *nbytes = v->elems_bytes;
  return Q8LIN_OK;
}

int q8lin_gguf_weight_create(const q8lin_gguf* g, const char* tensor_name, int device, q8lin_stream_t stream,
                             q8lin_weight** out) {
  if (!out) return fail(Q8LIN_ERR_INVALID_ARGUMENT, "out is null");
  *out = nullptr;
  int64_t idx = 0;
  int st = q8lin_gguf_find_tensor(g, tensor_name, &idx);
  if (st != Q8LIN_OK) return st;
  const q8lin_gguf::Tensor& t = g->tensors[(size_t)idx];
  if (t.type != Q8LIN_GGML_Q8_0)
    return fail(Q8LIN_ERR_FORMAT, "tensor '" + t.name + "' has ggml type " + std::to_string(t.type) +
                                      "; the quantized linear takes Q8_0 (type 8)");
  if (t.n_dims != 2 && !(t.n_dims > 2 && t.ne[2] == 1 && t.ne[3] == 1))
    return fail(Q8LIN_ERR_SHAPE, "tensor '" + t.name + "' is not a matrix");
  // GGUF ne = [in, out]: ne[0] = K (contiguous), ne[1] = N rows of K/32 blocks.
  return q8lin_weight_create(g->base + t.offset, t.ne[1], t.ne[0], device, stream, out);
}

}  // extern "C"
