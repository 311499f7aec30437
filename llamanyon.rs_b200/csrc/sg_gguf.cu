// sg_gguf.cu -- GGUF file reader and the upload path from a GGUF tensor to a
// registered device weight (host code; part of the libswamp_gpu.so unity
// build, after sg_api.cu).
//
// Replaces swamp-gguf's GgufFile (swamp-gguf/src/mmap.rs:26-120), its
// metadata reader (metadata.rs:118-236) and TensorInfo
// (tensor_info.rs:8-38), as the engine uses them to find a tensor and its raw
// blocks before every forward_linear (swamp-engine/src/linear.rs:24,
// executor.rs:436-438). The format rules follow the reference exactly:
//   - magic "GGUF", version 1..3 (mmap.rs:38-46); counts and dimensions are
//     u32 in version 1 and u64 from version 2 (:48-49,:64-66);
//   - a string is a u64 byte length and the bytes, decoded as UTF-8 with
//     each invalid sequence replaced by U+FFFD (metadata.rs:185-191, Rust's
//     from_utf8_lossy), in every version;
//   - metadata value types 0..12, arrays of any of them except arrays
//     (metadata.rs:201-236); a repeated key keeps its last value (HashMap
//     insert, mmap.rs:53-58);
//   - tensor types must be known ggml types (dtype.rs:43-75: 0-3, 6-30);
//   - tensor data starts at the end of the tensor table rounded up to 32
//     bytes; general.alignment is not consulted (mmap.rs:13,78-89);
//   - a tensor's bytes are ceil(elements / block) * block bytes
//     (dtype.rs:78-140, in wrapping u64 arithmetic as the reference's
//     release build computes them), checked against the file only when read
//     (mmap.rs:111-118).
// The file is mapped read-only; tensor data is never copied until a tensor is
// registered (sg_gguf_register), which hands the mapped blocks to
// sg_weight_register.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

struct SgKv {
  std::string key;
  int type = 0, elem_type = -1;  // GGUF value type; element type of an array
  int64_t count = 1;             // elements (1 for a scalar)
  std::vector<int64_t> ints;     // integer and bool values (u64 stored as its bits)
  std::vector<double> floats;    // f32 / f64 values
  std::vector<std::string> strs; // string values
};

struct SgTensorInfo {
  std::string name;
  std::vector<int64_t> dims;  // u64 bit patterns
  int dtype = 0;
  uint64_t offset = 0;  // absolute, in the file
  uint64_t nbytes = 0;  // u64 arithmetic wraps as the reference's release build does
};

struct sg_gguf_s {
  const uint8_t* data = nullptr;
  size_t size = 0;
  bool mapped = false;
  uint32_t version = 0;
  int64_t data_offset = 0;
  std::vector<SgKv> kv;  // in file order
  std::vector<SgTensorInfo> tensors;
};

namespace {

// ggml element block and block bytes by type (dtype.rs:78-140); 0 = unknown
void gguf_type_shape(int t, int64_t* block, int64_t* bytes) {
  static const int64_t kBlock[31] = {1, 1, 32, 32, 0, 0, 32, 32, 32, 32, 256, 256, 256, 256, 256, 256,
                                     256, 256, 256, 256, 32, 256, 256, 32, 1, 1, 1, 1, 1, 256, 1};
  static const int64_t kBytes[31] = {4, 2, 18, 20, 0, 0, 22, 24, 34, 40, 84, 110, 144, 176, 210, 292,
                                     66, 74, 98, 50, 18, 110, 82, 136, 1, 2, 4, 8, 8, 56, 2};
  *block = (t >= 0 && t < 31) ? kBlock[t] : 0;
  *bytes = (t >= 0 && t < 31) ? kBytes[t] : 0;
}

// UTF-8 decode with each maximal invalid subsequence replaced by U+FFFD, the
// rule of Rust's String::from_utf8_lossy
std::string utf8_lossy(const uint8_t* p, size_t n) {
  std::string out;
  out.reserve(n);
  size_t i = 0;
  while (i < n) {
    const uint8_t c = p[i];
    if (c < 0x80) {
      out.push_back((char)c);
      ++i;
      continue;
    }
    int need = 0;
    uint8_t lo = 0x80, hi = 0xBF;
    if (c >= 0xC2 && c <= 0xDF) need = 1;
    else if (c == 0xE0) need = 2, lo = 0xA0;
    else if (c >= 0xE1 && c <= 0xEC) need = 2;
    else if (c == 0xED) need = 2, hi = 0x9F;
    else if (c >= 0xEE && c <= 0xEF) need = 2;
    else if (c == 0xF0) need = 3, lo = 0x90;
    else if (c >= 0xF1 && c <= 0xF3) need = 3;
    else if (c == 0xF4) need = 3, hi = 0x8F;
    size_t j = i + 1;
    int got = 0;
    if (need > 0) {
      // the first continuation byte has the lead byte's range, the rest 80..BF
      while (got < need && j < n) {
        const uint8_t b = p[j];
        const uint8_t l = got == 0 ? lo : 0x80, h = got == 0 ? hi : 0xBF;
        if (b < l || b > h) break;
        ++j;
        ++got;
      }
    }
    if (need > 0 && got == need) {
      out.append(reinterpret_cast<const char*>(p + i), j - i);
    } else {
      out.append("\xEF\xBF\xBD");
    }
    i = (need > 0 && got == need) ? j : (need > 0 ? i + 1 + got : i + 1);
  }
  return out;
}

// little-endian reader over the file image; every read is bounds-checked
struct GgufReader {
  const uint8_t* p;
  size_t n, pos = 0;
  bool ok = true;
  const char* what = nullptr;  // first failing read
  bool take(size_t k, const char* w) {
    if (!ok) return false;
    if (k > n - pos) {
      ok = false;
      what = w;
      return false;
    }
    return true;
  }
  uint64_t uint(int bytes, const char* w) {
    if (!take((size_t)bytes, w)) return 0;
    uint64_t v = 0;
    for (int i = 0; i < bytes; ++i) v |= (uint64_t)p[pos + i] << (8 * i);
    pos += (size_t)bytes;
    return v;
  }
  std::string str(const char* w) {
    const uint64_t len = uint(8, w);
    if (!ok) return std::string();
    if (!take(len > n ? n + 1 : (size_t)len, w)) return std::string();
    std::string s = utf8_lossy(p + pos, (size_t)len);
    pos += (size_t)len;
    return s;
  }
};

// one metadata value of type t into kv (elements appended)
bool gguf_value(GgufReader& r, int t, SgKv& kv) {
  switch (t) {
    case 0: kv.ints.push_back((int64_t)(uint8_t)r.uint(1, "read_u8")); break;
    case 1: kv.ints.push_back((int64_t)(int8_t)r.uint(1, "read_u8")); break;
    case 2: kv.ints.push_back((int64_t)(uint16_t)r.uint(2, "read_u16")); break;
    case 3: kv.ints.push_back((int64_t)(int16_t)r.uint(2, "read_u16")); break;
    case 4: kv.ints.push_back((int64_t)(uint32_t)r.uint(4, "read_u32")); break;
    case 5: kv.ints.push_back((int64_t)(int32_t)r.uint(4, "read_u32")); break;
    case 6: {
      const uint32_t b = (uint32_t)r.uint(4, "read_u32");
      float f;
      memcpy(&f, &b, 4);
      kv.floats.push_back((double)f);
      break;
    }
    case 7: kv.ints.push_back(r.uint(1, "read_u8") != 0 ? 1 : 0); break;
    case 8: kv.strs.push_back(r.str("read_string")); break;
    case 10: kv.ints.push_back((int64_t)r.uint(8, "read_u64")); break;
    case 11: kv.ints.push_back((int64_t)r.uint(8, "read_u64")); break;
    case 12: {
      const uint64_t b = r.uint(8, "read_u64");
      double d;
      memcpy(&d, &b, 8);
      kv.floats.push_back(d);
      break;
    }
    default: return false;
  }
  return r.ok;
}

int gguf_parse(sg_gguf_s* g) {
  GgufReader r{g->data, g->size};
  if (g->size < 4) return fail(SG_ERR_FORMAT, "gguf: unexpected end of file (read_bytes)");
  if (memcmp(g->data, "GGUF", 4) != 0) return fail(SG_ERR_FORMAT, "gguf: invalid magic");
  r.pos = 4;
  g->version = (uint32_t)r.uint(4, "read_u32");
  if (!r.ok) return fail(SG_ERR_FORMAT, "gguf: unexpected end of file (%s)", r.what);
  if (g->version < 1 || g->version > 3) return fail(SG_ERR_FORMAT, "gguf: unsupported version %u", g->version);
  const int cw = g->version >= 2 ? 8 : 4;  // width of counts and dimensions
  const uint64_t n_t = r.uint(cw, cw == 8 ? "read_u64" : "read_u32");
  const uint64_t n_kv = r.uint(cw, cw == 8 ? "read_u64" : "read_u32");
  for (uint64_t i = 0; r.ok && i < n_kv; ++i) {
    SgKv kv;
    kv.key = r.str("read_string");
    kv.type = (int)(uint32_t)r.uint(4, "read_u32");
    if (!r.ok) break;
    if (kv.type == 9) {
      kv.elem_type = (int)(uint32_t)r.uint(4, "read_u32");
      const uint64_t cnt = r.uint(8, "read_u64");
      if (!r.ok) break;
      if (kv.elem_type == 9 || kv.elem_type < 0 || kv.elem_type > 12)
        return fail(SG_ERR_FORMAT, "gguf: unknown metadata type %u", (uint32_t)kv.elem_type);
      kv.count = (int64_t)cnt;
      for (uint64_t e = 0; r.ok && e < cnt; ++e)
        if (!gguf_value(r, kv.elem_type, kv) && r.ok)
          return fail(SG_ERR_FORMAT, "gguf: unknown metadata type %u", (uint32_t)kv.elem_type);
    } else if (!gguf_value(r, kv.type, kv) && r.ok) {
      return fail(SG_ERR_FORMAT, "gguf: unknown metadata type %u", (uint32_t)kv.type);
    }
    if (r.ok) g->kv.push_back(std::move(kv));
  }
  for (uint64_t i = 0; r.ok && i < n_t; ++i) {
    SgTensorInfo t;
    t.name = r.str("read_string");
    const uint32_t nd = (uint32_t)r.uint(4, "read_u32");
    for (uint32_t d = 0; r.ok && d < nd; ++d) t.dims.push_back((int64_t)r.uint(cw, cw == 8 ? "read_u64" : "read_u32"));
    t.dtype = (int)(uint32_t)r.uint(4, "read_u32");
    if (!r.ok) break;
    int64_t block, bytes;
    gguf_type_shape(t.dtype, &block, &bytes);
    if (block == 0) return fail(SG_ERR_FORMAT, "gguf: unknown tensor type %u", (uint32_t)t.dtype);
    t.offset = r.uint(8, "read_u64");
    if (!r.ok) break;
    uint64_t elems = 1;
    for (int64_t d : t.dims) elems *= (uint64_t)d;  // tensor_info.rs:19-21, wrapping
    t.nbytes = (elems + (uint64_t)block - 1) / (uint64_t)block * (uint64_t)bytes;  // dtype.rs:136-140
    g->tensors.push_back(std::move(t));
  }
  if (!r.ok) return fail(SG_ERR_FORMAT, "gguf: unexpected end of file (%s)", r.what);
  g->data_offset = (int64_t)((r.pos + 31) / 32 * 32);
  for (auto& t : g->tensors) t.offset += (uint64_t)g->data_offset;
  return SG_OK;
}

int gguf_check(sg_gguf_t g) { return g ? SG_OK : fail(SG_ERR_INVALID_ARG, "null gguf handle"); }

}  // namespace

int sg_gguf_open(const char* path, sg_gguf_t* out) {
  if (!path || !out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return fail(SG_ERR_INVALID_ARG, "gguf: cannot open %s", path);
  struct stat st;
  if (fstat(fd, &st) != 0) {
    close(fd);
    return fail(SG_ERR_INVALID_ARG, "gguf: cannot stat %s", path);
  }
  auto* g = new sg_gguf_s();
  g->size = (size_t)st.st_size;
  if (g->size > 0) {
    void* m = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
      close(fd);
      delete g;
      return fail(SG_ERR_OOM, "gguf: cannot map %s", path);
    }
    g->data = static_cast<const uint8_t*>(m);
    g->mapped = true;
  }
  close(fd);
  const int rc = gguf_parse(g);
  if (rc != SG_OK) {
    sg_gguf_close(g);
    return rc;
  }
  *out = g;
  return SG_OK;
}

int sg_gguf_open_memory(const void* data, size_t size, sg_gguf_t* out) {
  if (!out || (!data && size)) return fail(SG_ERR_INVALID_ARG, "null pointer");
  *out = nullptr;
  auto* g = new sg_gguf_s();
  g->data = static_cast<const uint8_t*>(data);
  g->size = size;
  const int rc = gguf_parse(g);
  if (rc != SG_OK) {
    delete g;
    return rc;
  }
  *out = g;
  return SG_OK;
}

int sg_gguf_close(sg_gguf_t g) {
  if (!g) return SG_OK;
  if (g->mapped) munmap(const_cast<uint8_t*>(g->data), g->size);
  delete g;
  return SG_OK;
}

int sg_gguf_header(sg_gguf_t g, uint32_t* version, int64_t* n_tensors, int64_t* n_kv, int64_t* data_offset,
                   int64_t* file_size) {
  if (int rc = gguf_check(g)) return rc;
  if (version) *version = g->version;
  if (n_tensors) *n_tensors = (int64_t)g->tensors.size();
  if (n_kv) *n_kv = (int64_t)g->kv.size();
  if (data_offset) *data_offset = g->data_offset;
  if (file_size) *file_size = (int64_t)g->size;
  return SG_OK;
}

int sg_gguf_find_tensor(sg_gguf_t g, const char* name, int64_t* index) {
  if (int rc = gguf_check(g)) return rc;
  if (!name || !index) return fail(SG_ERR_INVALID_ARG, "null pointer");
  for (size_t i = 0; i < g->tensors.size(); ++i)  // first match (mmap.rs:96-98)
    if (g->tensors[i].name == name) {
      *index = (int64_t)i;
      return SG_OK;
    }
  return fail(SG_ERR_NOT_FOUND, "gguf: tensor not found: %s", name);
}

int sg_gguf_tensor_info(sg_gguf_t g, int64_t index, const char** name, int* dtype, int* n_dims, int64_t* dims,
                        int dims_cap, int64_t* offset, int64_t* nbytes) {
  if (int rc = gguf_check(g)) return rc;
  if (index < 0 || index >= (int64_t)g->tensors.size()) return fail(SG_ERR_INVALID_ARG, "gguf: tensor index %lld", (long long)index);
  const SgTensorInfo& t = g->tensors[(size_t)index];
  if (name) *name = t.name.c_str();
  if (dtype) *dtype = t.dtype;
  if (n_dims) *n_dims = (int)t.dims.size();
  for (int d = 0; dims && d < dims_cap && d < (int)t.dims.size(); ++d) dims[d] = t.dims[(size_t)d];
  if (offset) *offset = (int64_t)t.offset;
  if (nbytes) *nbytes = (int64_t)t.nbytes;
  return SG_OK;
}

int sg_gguf_tensor_data(sg_gguf_t g, int64_t index, const void** data, int64_t* nbytes) {
  if (int rc = gguf_check(g)) return rc;
  if (index < 0 || index >= (int64_t)g->tensors.size()) return fail(SG_ERR_INVALID_ARG, "gguf: tensor index %lld", (long long)index);
  const SgTensorInfo& t = g->tensors[(size_t)index];
  if (t.offset > g->size || t.nbytes > g->size - t.offset)
    return fail(SG_ERR_FORMAT, "gguf: %s: range %llu..%llu outside the file (%zu bytes)", t.name.c_str(),
                (unsigned long long)t.offset, (unsigned long long)(t.offset + t.nbytes), g->size);
  if (data) *data = g->data + t.offset;
  if (nbytes) *nbytes = (int64_t)t.nbytes;
  return SG_OK;
}

int sg_gguf_find_kv(sg_gguf_t g, const char* key, int64_t* index) {
  if (int rc = gguf_check(g)) return rc;
  if (!key || !index) return fail(SG_ERR_INVALID_ARG, "null pointer");
  for (size_t i = g->kv.size(); i-- > 0;)  // a repeated key keeps its last value
    if (g->kv[i].key == key) {
      *index = (int64_t)i;
      return SG_OK;
    }
  return fail(SG_ERR_NOT_FOUND, "gguf: metadata key not found: %s", key);
}

int sg_gguf_kv_info(sg_gguf_t g, int64_t index, const char** key, int* type, int* elem_type, int64_t* count) {
  if (int rc = gguf_check(g)) return rc;
  if (index < 0 || index >= (int64_t)g->kv.size()) return fail(SG_ERR_INVALID_ARG, "gguf: metadata index %lld", (long long)index);
  const SgKv& kv = g->kv[(size_t)index];
  if (key) *key = kv.key.c_str();
  if (type) *type = kv.type;
  if (elem_type) *elem_type = kv.elem_type;
  if (count) *count = kv.count;
  return SG_OK;
}

namespace {
int kv_elem(sg_gguf_t g, int64_t index, int64_t elem, const SgKv** kv, int* t) {
  if (int rc = gguf_check(g)) return rc;
  if (index < 0 || index >= (int64_t)g->kv.size()) return fail(SG_ERR_INVALID_ARG, "gguf: metadata index %lld", (long long)index);
  *kv = &g->kv[(size_t)index];
  *t = (*kv)->type == 9 ? (*kv)->elem_type : (*kv)->type;
  if (elem < 0 || elem >= (*kv)->count) return fail(SG_ERR_INVALID_ARG, "gguf: element %lld of %s", (long long)elem, (*kv)->key.c_str());
  return SG_OK;
}
}  // namespace

int sg_gguf_kv_int(sg_gguf_t g, int64_t index, int64_t elem, int64_t* value) {
  const SgKv* kv;
  int t;
  if (int rc = kv_elem(g, index, elem, &kv, &t)) return rc;
  if (t == 6 || t == 8 || t == 12) return fail(SG_ERR_INVALID_ARG, "gguf: %s is not an integer", kv->key.c_str());
  if (value) *value = kv->ints[(size_t)elem];
  return SG_OK;
}

int sg_gguf_kv_float(sg_gguf_t g, int64_t index, int64_t elem, double* value) {
  const SgKv* kv;
  int t;
  if (int rc = kv_elem(g, index, elem, &kv, &t)) return rc;
  if (t != 6 && t != 12) return fail(SG_ERR_INVALID_ARG, "gguf: %s is not a float", kv->key.c_str());
  if (value) *value = kv->floats[(size_t)elem];
  return SG_OK;
}

int sg_gguf_kv_string(sg_gguf_t g, int64_t index, int64_t elem, const char** str, int64_t* len) {
  const SgKv* kv;
  int t;
  if (int rc = kv_elem(g, index, elem, &kv, &t)) return rc;
  if (t != 8) return fail(SG_ERR_INVALID_ARG, "gguf: %s is not a string", kv->key.c_str());
  const std::string& s = kv->strs[(size_t)elem];
  if (str) *str = s.c_str();
  if (len) *len = (int64_t)s.size();
  return SG_OK;
}

int sg_gguf_register(sg_gguf_t g, int64_t index, int tp_mode, sg_weight_t* out) {
  if (int rc = gguf_check(g)) return rc;
  if (!out) return fail(SG_ERR_INVALID_ARG, "null pointer");
  if (index < 0 || index >= (int64_t)g->tensors.size()) return fail(SG_ERR_INVALID_ARG, "gguf: tensor index %lld", (long long)index);
  const SgTensorInfo& t = g->tensors[(size_t)index];
  if (t.dtype != SG_DTYPE_Q4_0 && t.dtype != SG_DTYPE_Q4_K && t.dtype != SG_DTYPE_Q6_K)
    return fail(SG_ERR_UNSUPPORTED, "gguf: %s has type %d; the device path takes Q4_0 (2), Q4_K (12) and Q6_K (14)",
                t.name.c_str(), t.dtype);
  // a linear weight: shape[0] = n_cols (K, contiguous), shape[1] = n_rows (N);
  // trailing dimensions of 1 are allowed
  if (t.dims.size() < 2) return fail(SG_ERR_UNSUPPORTED, "gguf: %s is not a matrix", t.name.c_str());
  for (size_t d = 2; d < t.dims.size(); ++d)
    if (t.dims[d] != 1) return fail(SG_ERR_UNSUPPORTED, "gguf: %s has more than two non-unit dimensions", t.name.c_str());
  const void* blocks = nullptr;
  if (int rc = sg_gguf_tensor_data(g, index, &blocks, nullptr)) return rc;
  return sg_weight_register(blocks, t.dtype, t.dims[1], t.dims[0], tp_mode, out);
}
