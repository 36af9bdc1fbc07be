// GGUF (version 2/3) reader of libunltd_gpu: the file is mapped read-only
// and its tensors are handed to the upload path as zero-copy views, the way
// the reference opens a model (gguf.rs:353-520 parse, weights.rs:32-92
// tensor views). Every field is bounds-checked against the mapping (the file
// is untrusted input); nothing is read past its end.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "unltd_host.h"
#include "unltd_internal.cuh"

using namespace unltd;

namespace {

// GGUF metadata value types
enum : uint32_t {
  GT_U8 = 0, GT_I8, GT_U16, GT_I16, GT_U32, GT_I32, GT_F32, GT_BOOL, GT_STRING, GT_ARRAY, GT_U64, GT_I64, GT_F64
};

// ggml tensor types this path uses -> unltd dtype (lib.rs:19-31 ordinals)
int dtype_of_ggml(uint32_t t) {
  switch (t) {
    case 0: return F32;
    case 1: return F16;
    case 30: return BF16;
    case 8: return Q8_0;
    case 12: return Q4K;
    case 14: return Q6K;
    default: return -1;
  }
}

// bytes of n elements of an unltd dtype (0: not a whole number of blocks)
size_t dtype_bytes(int dt, uint64_t n) {
  switch (dt) {
    case F32: return n * 4;
    case F16:
    case BF16: return n * 2;
    case Q8_0: return n % kQ80Elems ? 0 : n / kQ80Elems * kQ80Bytes;
    case Q4K: return n % kQK ? 0 : n / kQK * kQ4Bytes;
    case Q6K: return n % kQK ? 0 : n / kQK * kQ6Bytes;
    default: return 0;
  }
}

struct Cursor {
  const uint8_t *p, *end;
  bool ok = true;
  bool take(void *dst, size_t n) {
    if (!ok || (size_t)(end - p) < n) return ok = false;
    memcpy(dst, p, n);
    p += n;
    return true;
  }
  template <class T> T get() {
    T v{};
    take(&v, sizeof(T));
    return v;
  }
  bool skip(size_t n) {
    if (!ok || (size_t)(end - p) < n) return ok = false;
    p += n;
    return true;
  }
  std::string str(size_t limit) {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > limit || (size_t)(end - p) < n) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char *>(p), n);
    p += n;
    return s;
  }
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case GT_U8: case GT_I8: case GT_BOOL: return 1;
    case GT_U16: case GT_I16: return 2;
    case GT_U32: case GT_I32: case GT_F32: return 4;
    case GT_U64: case GT_I64: case GT_F64: return 8;
    default: return 0;
  }
}

}  // namespace

struct GgufValue {
  uint32_t type = 0;      // scalar type, or GT_ARRAY
  uint32_t elem = 0;      // array element type
  std::vector<int64_t> i; // integer scalars / arrays (bool as 0/1)
  std::vector<double> f;  // float scalars / arrays
  std::string s;          // string scalar
  size_t count = 0;       // array length (strings in arrays are skipped)
};

struct unltd_gguf_s {
  int fd = -1;
  const uint8_t *map = nullptr;
  size_t size = 0;
  uint32_t version = 0;
  size_t alignment = 32, data_off = 0;
  std::map<std::string, GgufValue> kv;
  struct Tensor {
    std::string name;
    uint32_t ndims = 0, ggml = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    int dtype = -1;
    uint64_t offset = 0;
    size_t nbytes = 0;
  };
  std::vector<Tensor> tensors;
  std::map<std::string, size_t> index;
};

namespace {

int32_t parse(unltd_gguf g) {
  Cursor c{g->map, g->map + g->size};
  char magic[4];
  if (!c.take(magic, 4) || memcmp(magic, "GGUF", 4) != 0) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: bad magic");
  g->version = c.get<uint32_t>();
  if (!c.ok || (g->version != 2 && g->version != 3))
    return set_error(UNLTD_ERR_UNSUPPORTED, "gguf: version " + std::to_string(g->version) + " (2 or 3 expected)");
  const uint64_t nt = c.get<uint64_t>(), nkv = c.get<uint64_t>();
  if (!c.ok || nt > (1u << 20) || nkv > (1u << 20)) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: bad counts");
  for (uint64_t k = 0; k < nkv && c.ok; k++) {
    std::string key = c.str(1 << 16);
    GgufValue v;
    v.type = c.get<uint32_t>();
    if (!c.ok) break;
    if (v.type == GT_STRING) {
      v.s = c.str(1 << 24);
    } else if (v.type == GT_ARRAY) {
      v.elem = c.get<uint32_t>();
      const uint64_t n = c.get<uint64_t>();
      if (!c.ok || n > (1ull << 26)) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: array of '" + key + "' too long");
      v.count = (size_t)n;
      if (v.elem == GT_STRING) {  // e.g. a tokenizer vocabulary: skipped
        for (uint64_t j = 0; j < n && c.ok; j++) c.str(1 << 20);
      } else {
        const size_t es = scalar_size(v.elem);
        if (!es) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: bad array element type of '" + key + "'");
        if (n <= 64) {  // small arrays are kept (rope sections, ...)
          for (uint64_t j = 0; j < n && c.ok; j++) {
            if (v.elem == GT_F32) v.f.push_back(c.get<float>());
            else if (v.elem == GT_F64) v.f.push_back(c.get<double>());
            else {
              int64_t x = 0;
              switch (v.elem) {
                case GT_U8: x = c.get<uint8_t>(); break;
                case GT_I8: x = c.get<int8_t>(); break;
                case GT_BOOL: x = c.get<uint8_t>() != 0; break;
                case GT_U16: x = c.get<uint16_t>(); break;
                case GT_I16: x = c.get<int16_t>(); break;
                case GT_U32: x = c.get<uint32_t>(); break;
                case GT_I32: x = c.get<int32_t>(); break;
                case GT_U64: x = (int64_t)c.get<uint64_t>(); break;
                default: x = c.get<int64_t>(); break;
              }
              v.i.push_back(x);
            }
          }
        } else if (!c.skip(es * (size_t)n)) {
          break;
        }
      }
    } else {
      switch (v.type) {
        case GT_U8: v.i.push_back(c.get<uint8_t>()); break;
        case GT_I8: v.i.push_back(c.get<int8_t>()); break;
        case GT_BOOL: v.i.push_back(c.get<uint8_t>() != 0); break;
        case GT_U16: v.i.push_back(c.get<uint16_t>()); break;
        case GT_I16: v.i.push_back(c.get<int16_t>()); break;
        case GT_U32: v.i.push_back(c.get<uint32_t>()); break;
        case GT_I32: v.i.push_back(c.get<int32_t>()); break;
        case GT_U64: v.i.push_back((int64_t)c.get<uint64_t>()); break;
        case GT_I64: v.i.push_back(c.get<int64_t>()); break;
        case GT_F32: v.f.push_back(c.get<float>()); break;
        case GT_F64: v.f.push_back(c.get<double>()); break;
        default: return set_error(UNLTD_ERR_INVALID_ARG, "gguf: bad value type of '" + key + "'");
      }
    }
    if (c.ok) g->kv[key] = std::move(v);
  }
  if (!c.ok) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: metadata runs past the end of the file");
  auto al = g->kv.find("general.alignment");
  if (al != g->kv.end() && !al->second.i.empty()) {
    const int64_t a = al->second.i[0];
    if (a <= 0 || (a & (a - 1)) || a > 65536) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: bad general.alignment");
    g->alignment = (size_t)a;
  }
  for (uint64_t k = 0; k < nt && c.ok; k++) {
    unltd_gguf_s::Tensor t;
    t.name = c.str(1 << 12);
    t.ndims = c.get<uint32_t>();
    if (!c.ok || t.ndims < 1 || t.ndims > 4) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: bad tensor rank");
    uint64_t n = 1;
    for (uint32_t d = 0; d < t.ndims; d++) {
      const uint64_t ne = c.get<uint64_t>();
      if (ne == 0 || ne > (1ull << 40) || n > (1ull << 40) / ne) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: bad dims of '" + t.name + "'");
      t.ne[d] = (int64_t)ne;
      n *= ne;
    }
    t.ggml = c.get<uint32_t>();
    t.offset = c.get<uint64_t>();
    if (!c.ok) break;
    t.dtype = dtype_of_ggml(t.ggml);
    t.nbytes = t.dtype >= 0 ? dtype_bytes(t.dtype, n) : 0;
    if (g->index.count(t.name)) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: duplicate tensor '" + t.name + "'");
    g->index[t.name] = g->tensors.size();
    g->tensors.push_back(std::move(t));
  }
  if (!c.ok) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: tensor table runs past the end of the file");
  const size_t hdr = (size_t)(c.p - g->map);
  g->data_off = (hdr + g->alignment - 1) / g->alignment * g->alignment;
  for (const auto &t : g->tensors) {
    if (t.dtype < 0) continue;  // a type this path does not read: never handed out
    if (t.offset % g->alignment || g->data_off > g->size || t.offset > g->size - g->data_off ||
        t.nbytes > g->size - g->data_off - t.offset)
      return set_error(UNLTD_ERR_INVALID_ARG, "gguf: tensor '" + t.name + "' lies outside the file or is misaligned");
  }
  return UNLTD_OK;
}

const GgufValue *find_kv(unltd_gguf g, const char *key) {
  auto it = g->kv.find(key);
  return it == g->kv.end() ? nullptr : &it->second;
}

}  // namespace

namespace unltd {

bool gguf_tensor(unltd_gguf g, const std::string &name, GgufTensorView *out) {
  auto it = g->index.find(name);
  if (it == g->index.end()) return false;
  const auto &t = g->tensors[it->second];
  out->data = t.dtype >= 0 ? g->map + g->data_off + t.offset : nullptr;
  out->nbytes = t.nbytes;
  out->dtype = t.dtype;
  out->ndims = t.ndims;
  for (int d = 0; d < 4; d++) out->ne[d] = t.ne[d];
  return true;
}

}  // namespace unltd

extern "C" {

int32_t unltd_gguf_open(const char *path, unltd_gguf *out) {
  if (!path || !out) return set_error(UNLTD_ERR_INVALID_ARG, "gguf_open: NULL argument");
  *out = nullptr;
  const int fd = open(path, O_RDONLY | O_CLOEXEC);
  if (fd < 0) return set_error(UNLTD_ERR_INVALID_ARG, std::string("gguf_open: cannot open ") + path);
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    close(fd);
    return set_error(UNLTD_ERR_INVALID_ARG, std::string("gguf_open: ") + path + " is too short for a GGUF header");
  }
  void *m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  if (m == MAP_FAILED) {
    close(fd);
    return set_error(UNLTD_ERR_INVALID_ARG, std::string("gguf_open: cannot map ") + path);
  }
  auto *g = new unltd_gguf_s;
  g->fd = fd;
  g->map = static_cast<const uint8_t *>(m);
  g->size = (size_t)st.st_size;
  if (int32_t rc = parse(g)) {
    unltd_gguf_close(g);
    return rc;
  }
  *out = g;
  return UNLTD_OK;
}

int32_t unltd_gguf_close(unltd_gguf g) {
  if (!g) return UNLTD_OK;
  if (g->map) munmap(const_cast<uint8_t *>(g->map), g->size);
  if (g->fd >= 0) close(g->fd);
  delete g;
  return UNLTD_OK;
}

int64_t unltd_gguf_tensor_count(unltd_gguf g) { return g ? (int64_t)g->tensors.size() : -1; }

int32_t unltd_gguf_tensor_info(unltd_gguf g, int64_t i, const char **name, int32_t *dtype, int64_t *ne,
                               int32_t *ndims, const void **data, size_t *nbytes) {
  if (!g || i < 0 || i >= (int64_t)g->tensors.size()) return set_error(UNLTD_ERR_INVALID_ARG, "gguf_tensor_info: bad index");
  const auto &t = g->tensors[(size_t)i];
  if (name) *name = t.name.c_str();
  if (dtype) *dtype = t.dtype;
  if (ne)
    for (int d = 0; d < 4; d++) ne[d] = t.ne[d];
  if (ndims) *ndims = (int32_t)t.ndims;
  if (data) *data = t.dtype >= 0 ? g->map + g->data_off + t.offset : nullptr;
  if (nbytes) *nbytes = t.nbytes;
  return UNLTD_OK;
}

int32_t unltd_gguf_find_tensor(unltd_gguf g, const char *name, int64_t *index) {
  if (!g || !name || !index) return set_error(UNLTD_ERR_INVALID_ARG, "gguf_find_tensor: NULL argument");
  auto it = g->index.find(name);
  if (it == g->index.end()) return set_error(UNLTD_ERR_INVALID_ARG, std::string("gguf: no tensor '") + name + "'");
  *index = (int64_t)it->second;
  return UNLTD_OK;
}

int32_t unltd_gguf_get_int(unltd_gguf g, const char *key, int64_t *out) {
  if (!g || !key || !out) return set_error(UNLTD_ERR_INVALID_ARG, "gguf_get_int: NULL argument");
  const GgufValue *v = find_kv(g, key);
  if (!v || v->type == GT_ARRAY || v->i.empty()) return set_error(UNLTD_ERR_INVALID_ARG, std::string("gguf: no integer '") + key + "'");
  *out = v->i[0];
  return UNLTD_OK;
}

int32_t unltd_gguf_get_float(unltd_gguf g, const char *key, double *out) {
  if (!g || !key || !out) return set_error(UNLTD_ERR_INVALID_ARG, "gguf_get_float: NULL argument");
  const GgufValue *v = find_kv(g, key);
  if (!v || v->type == GT_ARRAY || v->f.empty()) return set_error(UNLTD_ERR_INVALID_ARG, std::string("gguf: no float '") + key + "'");
  *out = v->f[0];
  return UNLTD_OK;
}

int32_t unltd_gguf_get_string(unltd_gguf g, const char *key, const char **out) {
  if (!g || !key || !out) return set_error(UNLTD_ERR_INVALID_ARG, "gguf_get_string: NULL argument");
  const GgufValue *v = find_kv(g, key);
  if (!v || v->type != GT_STRING) return set_error(UNLTD_ERR_INVALID_ARG, std::string("gguf: no string '") + key + "'");
  *out = v->s.c_str();
  return UNLTD_OK;
}

// Qwen35Config::from_gguf (qwen35.rs:23-42 required keys, 130-200 extraction
// and checks): every key must be present with its type; vocab from the
// token embedding's row count.
int32_t unltd_qwen35_config_from_gguf(unltd_gguf g, unltd_qwen35_config *cfg) {
  if (!g || !cfg) return set_error(UNLTD_ERR_INVALID_ARG, "qwen35_config_from_gguf: NULL argument");
  const GgufValue *arch = find_kv(g, "general.architecture");
  if (!arch || arch->type != GT_STRING || arch->s != "qwen35")
    return set_error(UNLTD_ERR_UNSUPPORTED, "gguf: general.architecture is not qwen35");
  auto u32 = [&](const char *suffix, int32_t *out) -> int32_t {
    const std::string key = std::string("qwen35.") + suffix;
    const GgufValue *v = find_kv(g, key.c_str());
    if (!v || v->type != GT_U32) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: missing u32 " + key);
    if (v->i[0] > 0x7fffffff) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: " + key + " out of range");
    *out = (int32_t)v->i[0];
    return UNLTD_OK;
  };
  auto f32 = [&](const char *suffix, float *out) -> int32_t {
    const std::string key = std::string("qwen35.") + suffix;
    const GgufValue *v = find_kv(g, key.c_str());
    if (!v || v->type != GT_F32) return set_error(UNLTD_ERR_INVALID_ARG, "gguf: missing f32 " + key);
    *out = (float)v->f[0];
    return UNLTD_OK;
  };
  unltd_qwen35_config c{};
  int32_t ctx_len = 0;
  int32_t rc = UNLTD_OK;
  if (!rc) rc = u32("block_count", &c.n_layer);
  if (!rc) rc = u32("context_length", &ctx_len);
  if (!rc) rc = u32("embedding_length", &c.n_embd);
  if (!rc) rc = u32("feed_forward_length", &c.n_ff);
  if (!rc) rc = u32("attention.head_count", &c.n_head);
  if (!rc) rc = u32("attention.head_count_kv", &c.n_head_kv);
  if (!rc) rc = u32("attention.key_length", &c.head_dim);
  if (!rc) rc = u32("attention.value_length", &c.head_dim_v);
  if (!rc) rc = f32("attention.layer_norm_rms_epsilon", &c.rms_eps);
  if (!rc) rc = u32("rope.dimension_count", &c.n_rot);
  if (!rc) rc = f32("rope.freq_base", &c.freq_base);
  if (!rc) rc = u32("ssm.conv_kernel", &c.conv_kernel);
  if (!rc) rc = u32("ssm.state_size", &c.state_size);
  if (!rc) rc = u32("ssm.group_count", &c.group_count);
  if (!rc) rc = u32("ssm.time_step_rank", &c.time_step_rank);
  if (!rc) rc = u32("ssm.inner_size", &c.d_inner);
  if (!rc) rc = u32("full_attention_interval", &c.full_attn_interval);
  if (rc) return rc;
  const GgufValue *sec = find_kv(g, "qwen35.rope.dimension_sections");
  if (!sec || sec->type != GT_ARRAY || sec->elem != GT_I32 || sec->count != 4)
    return set_error(UNLTD_ERR_INVALID_ARG, "gguf: qwen35.rope.dimension_sections must be i32[4] (IMROPE)");
  GgufTensorView emb;
  if (!gguf_tensor(g, "token_embd.weight", &emb) || emb.ndims != 2)
    return set_error(UNLTD_ERR_INVALID_ARG, "gguf: no 2-D token_embd.weight");
  if (emb.ne[0] != c.n_embd || emb.ne[1] > 0x7fffffff)
    return set_error(UNLTD_ERR_INVALID_ARG, "gguf: token_embd.weight does not match embedding_length");
  c.vocab = (int32_t)emb.ne[1];
  *cfg = c;  // structural checks run in unltd_qwen35_create
  return UNLTD_OK;
}

}  // extern "C"
