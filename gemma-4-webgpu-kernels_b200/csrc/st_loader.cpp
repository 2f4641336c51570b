// st_loader.cpp — the reference's checkpoint loader for the quantized weights, on
// the host side of libgq: safetensors header parse and memory map
// (rust/src/safetensors.rs:52-72, :131-180), the float decodes (safetensors.rs:74-110),
// the logical-to-on-disk name resolution (rust/src/weights.rs:37-48), the bit-width
// table (rust/src/config.rs:161-169) and the quantized-tensor construction
// (rust/src/weights.rs:86-110): U8 / I8 payload + f32 scale -> QuantWeight with
// bits, signed_i8 and group_size = K / scale_cols, uploaded with gq_qweight_upload.
//
// The file is memory-mapped read-only; a tensor's bytes are touched only when it is
// uploaded (the packed payload goes from the mapping to the device in the upload's
// copy; the scales are decoded to f32 on the host first).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <map>
#include <regex>
#include <string>
#include <vector>

#include "gq_host.h"

struct StMeta {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // data_offsets, relative to the payload
};

struct gq_st_file {
  const uint8_t *base = nullptr;  // whole file (mapped) or the caller's blob
  size_t size = 0;
  bool mapped = false;
  size_t data_start = 0;
  std::map<std::string, StMeta> tensors;  // sorted by name
  std::vector<const std::string *> names;
};

namespace {

// ---- a JSON reader for the safetensors header: objects, arrays, strings, numbers,
// true/false/null (everything the format and its __metadata__ may hold) ---------------
struct Json {
  const char *p, *e;
  bool ok = true;

  void ws() {
    while (p < e && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
  }
  bool eat(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    return false;
  }
  bool fail() { return ok = false; }
  bool str(std::string *out) {
    ws();
    if (p >= e || *p != '"') return fail();
    ++p;
    std::string s;
    while (p < e && *p != '"') {
      char c = *p++;
      if (c == '\\') {
        if (p >= e) return fail();
        const char x = *p++;
        switch (x) {
          case '"': case '\\': case '/': s += x; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'n': s += '\n'; break;
          case 'r': s += '\r'; break;
          case 't': s += '\t'; break;
          case 'u': {
            if (e - p < 4) return fail();
            unsigned v = 0;
            for (int i = 0; i < 4; ++i) {
              const char h = *p++;
              v <<= 4;
              if (h >= '0' && h <= '9') v |= h - '0';
              else if (h >= 'a' && h <= 'f') v |= h - 'a' + 10;
              else if (h >= 'A' && h <= 'F') v |= h - 'A' + 10;
              else return fail();
            }
            // tensor names are ASCII in practice; keep other code points as UTF-8
            if (v < 0x80) s += (char)v;
            else if (v < 0x800) { s += (char)(0xC0 | (v >> 6)); s += (char)(0x80 | (v & 0x3F)); }
            else { s += (char)(0xE0 | (v >> 12)); s += (char)(0x80 | ((v >> 6) & 0x3F)); s += (char)(0x80 | (v & 0x3F)); }
            break;
          }
          default: return fail();
        }
      } else {
        s += c;
      }
    }
    if (p >= e) return fail();
    ++p;
    if (out) *out = std::move(s);
    return true;
  }
  bool uint(uint64_t *out) {
    ws();
    if (p >= e || *p < '0' || *p > '9') return fail();
    uint64_t v = 0;
    while (p < e && *p >= '0' && *p <= '9') {
      const uint64_t d = (uint64_t)(*p++ - '0');
      if (v > (UINT64_MAX - d) / 10) return fail();
      v = v * 10 + d;
    }
    *out = v;
    return true;
  }
  bool skip(int depth = 0) {  // any value
    if (depth > 64) return fail();
    ws();
    if (p >= e) return fail();
    if (*p == '"') return str(nullptr);
    if (*p == '{') {
      ++p;
      if (eat('}')) return true;
      do {
        if (!str(nullptr) || !eat(':') || !skip(depth + 1)) return fail();
      } while (eat(','));
      return eat('}') || fail();
    }
    if (*p == '[') {
      ++p;
      if (eat(']')) return true;
      do {
        if (!skip(depth + 1)) return fail();
      } while (eat(','));
      return eat(']') || fail();
    }
    const char *q = p;
    while (p < e && (std::isalnum((unsigned char)*p) || *p == '-' || *p == '+' || *p == '.')) ++p;
    return p > q || fail();
  }
  bool uint_array(std::vector<uint64_t> *out) {
    if (!eat('[')) return fail();
    out->clear();
    if (eat(']')) return true;
    do {
      uint64_t v;
      if (!uint(&v)) return false;
      out->push_back(v);
    } while (eat(','));
    return eat(']') || fail();
  }
};

// parse_header (rust/src/safetensors.rs:52-72): [u64 LE header length][JSON header]
int parse(gq_st_file *f, std::string *why) {
  if (f->size < 8) return *why = "file shorter than 8 bytes", GQ_ERR_INVALID_ARGUMENT;
  uint64_t hlen = 0;
  for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | f->base[i];
  if (hlen == 0 || hlen > f->size - 8) return *why = "header length out of range", GQ_ERR_INVALID_ARGUMENT;
  Json j{reinterpret_cast<const char *>(f->base + 8), reinterpret_cast<const char *>(f->base + 8 + hlen)};
  if (!j.eat('{')) return *why = "header is not a JSON object", GQ_ERR_INVALID_ARGUMENT;
  if (!j.eat('}')) {
    do {
      std::string name;
      if (!j.str(&name) || !j.eat(':')) return *why = "malformed header", GQ_ERR_INVALID_ARGUMENT;
      if (name == "__metadata__") {
        if (!j.skip()) return *why = "malformed __metadata__", GQ_ERR_INVALID_ARGUMENT;
        continue;
      }
      StMeta m;
      bool have_dtype = false, have_shape = false, have_off = false;
      if (!j.eat('{')) return *why = name + ": entry is not an object", GQ_ERR_INVALID_ARGUMENT;
      if (!j.eat('}')) {
        do {
          std::string key;
          if (!j.str(&key) || !j.eat(':')) return *why = name + ": malformed entry", GQ_ERR_INVALID_ARGUMENT;
          if (key == "dtype") {
            have_dtype = j.str(&m.dtype);
          } else if (key == "shape") {
            std::vector<uint64_t> v;
            have_shape = j.uint_array(&v);
            for (uint64_t d : v) m.shape.push_back((int64_t)d);
          } else if (key == "data_offsets") {
            std::vector<uint64_t> v;
            have_off = j.uint_array(&v) && v.size() == 2;
            if (have_off) {
              m.begin = v[0];
              m.end = v[1];
            }
          } else if (!j.skip()) {
            return *why = name + ": malformed entry", GQ_ERR_INVALID_ARGUMENT;
          }
          if (!j.ok) return *why = name + ": malformed entry", GQ_ERR_INVALID_ARGUMENT;
        } while (j.eat(','));
        if (!j.eat('}')) return *why = name + ": malformed entry", GQ_ERR_INVALID_ARGUMENT;
      }
      if (!have_dtype || !have_shape || !have_off) return *why = name + ": dtype, shape and data_offsets required", GQ_ERR_INVALID_ARGUMENT;
      f->tensors[name] = std::move(m);
    } while (j.eat(','));
    if (!j.eat('}')) return *why = "malformed header", GQ_ERR_INVALID_ARGUMENT;
  }
  f->data_start = 8 + (size_t)hlen;
  for (auto &kv : f->tensors) f->names.push_back(&kv.first);
  return GQ_OK;
}

const StMeta *find(const gq_st_file *f, const char *name) {
  if (!f || !name) return nullptr;
  auto it = f->tensors.find(name);
  return it == f->tensors.end() ? nullptr : &it->second;
}

// raw_bytes (rust/src/safetensors.rs:154-163): the payload slice, bounds-checked
bool slice(const gq_st_file *f, const StMeta &m, const uint8_t **data, size_t *nbytes) {
  const uint64_t a = f->data_start + m.begin, b = f->data_start + m.end;
  if (m.begin > m.end || b > f->size || a < f->data_start) return false;
  *data = f->base + a;
  *nbytes = (size_t)(b - a);
  return true;
}

// f16_to_f32 (rust/src/safetensors.rs:75-86): the same formula, exact in f32
float f16_to_f32(uint16_t h) {
  const float s = (h & 0x8000) ? -1.0f : 1.0f;
  const int e = (h & 0x7c00) >> 10;
  const float fr = (float)(h & 0x03ff);
  if (e == 0) return s * std::ldexp(1.0f, -14) * (fr / 1024.0f);
  if (e == 0x1f) return fr != 0.0f ? NAN : s * INFINITY;
  return s * std::ldexp(1.0f, e - 15) * (1.0f + fr / 1024.0f);
}

float bf16_to_f32(uint16_t b) {
  const uint32_t u = (uint32_t)b << 16;
  float v;
  std::memcpy(&v, &u, 4);
  return v;
}

int64_t numel(const StMeta &m) {
  int64_t n = 1;
  for (int64_t d : m.shape) n *= d;
  return n;
}

}  // namespace

extern "C" {

int gq_st_open(const char *path, gq_st_file **out) {
  if (!path || !out) return GQ_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) return GQ_ERR_INVALID_ARGUMENT;
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size <= 0) {
    close(fd);
    return GQ_ERR_INVALID_ARGUMENT;
  }
  void *p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (p == MAP_FAILED) return GQ_ERR_OUT_OF_MEMORY;
  gq_st_file *f = new gq_st_file;
  f->base = static_cast<const uint8_t *>(p);
  f->size = (size_t)st.st_size;
  f->mapped = true;
  std::string why;
  const int rc = parse(f, &why);
  if (rc != GQ_OK) {
    munmap(const_cast<uint8_t *>(f->base), f->size);
    delete f;
    return rc;
  }
  *out = f;
  return GQ_OK;
}

int gq_st_open_memory(const uint8_t *bytes, size_t nbytes, gq_st_file **out) {
  if (!bytes || !out) return GQ_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  gq_st_file *f = new gq_st_file;
  f->base = bytes;
  f->size = nbytes;
  std::string why;
  const int rc = parse(f, &why);
  if (rc != GQ_OK) {
    delete f;
    return rc;
  }
  *out = f;
  return GQ_OK;
}

int gq_st_close(gq_st_file *f) {
  if (!f) return GQ_OK;
  if (f->mapped) munmap(const_cast<uint8_t *>(f->base), f->size);
  delete f;
  return GQ_OK;
}

int64_t gq_st_count(const gq_st_file *f) { return f ? (int64_t)f->names.size() : -1; }

const char *gq_st_name(const gq_st_file *f, int64_t i) {
  if (!f || i < 0 || i >= (int64_t)f->names.size()) return nullptr;
  return f->names[(size_t)i]->c_str();
}

int gq_st_info(const gq_st_file *f, const char *name, char *dtype16, int64_t *shape8, int32_t *ndim,
               const uint8_t **data, size_t *nbytes) {
  const StMeta *m = find(f, name);
  if (!m) return GQ_ERR_INVALID_ARGUMENT;
  if (m->shape.size() > 8 || m->dtype.size() >= 16) return GQ_ERR_UNSUPPORTED;
  const uint8_t *d = nullptr;
  size_t n = 0;
  if (!slice(f, *m, &d, &n)) return GQ_ERR_INVALID_ARGUMENT;
  if (dtype16) std::snprintf(dtype16, 16, "%s", m->dtype.c_str());
  if (shape8)
    for (size_t i = 0; i < m->shape.size(); ++i) shape8[i] = m->shape[i];
  if (ndim) *ndim = (int32_t)m->shape.size();
  if (data) *data = d;
  if (nbytes) *nbytes = n;
  return GQ_OK;
}

int gq_st_read_f32(const gq_st_file *f, const char *name, float *dst, size_t count) {
  const StMeta *m = find(f, name);
  if (!m || !dst) return GQ_ERR_INVALID_ARGUMENT;
  const uint8_t *d = nullptr;
  size_t n = 0;
  if (!slice(f, *m, &d, &n)) return GQ_ERR_INVALID_ARGUMENT;
  const size_t esz = m->dtype == "F32" ? 4 : ((m->dtype == "F16" || m->dtype == "BF16") ? 2 : 0);
  if (esz == 0) return GQ_ERR_UNSUPPORTED;
  if (n != count * esz || (int64_t)count != numel(*m)) return GQ_ERR_INVALID_ARGUMENT;
  for (size_t i = 0; i < count; ++i) {
    if (esz == 4) {
      std::memcpy(dst + i, d + 4 * i, 4);
    } else {
      const uint16_t h = (uint16_t)(d[2 * i] | (d[2 * i + 1] << 8));
      dst[i] = m->dtype == "F16" ? f16_to_f32(h) : bf16_to_f32(h);
    }
  }
  return GQ_OK;
}

int32_t gq_bits_for(const char *name, const char *const *patterns, const int32_t *bits, int32_t nrules) {
  if (!name || nrules < 0 || (nrules > 0 && (!patterns || !bits))) return -1;
  for (int32_t i = 0; i < nrules; ++i) {
    try {
      if (std::regex_search(name, std::regex(patterns[i], std::regex::ECMAScript))) return bits[i];
    } catch (const std::regex_error &) {
      return -1;
    }
  }
  return 16;
}

int gq_st_resolve(const char *logical, char *weight256, char *scale256, char *bare256) {
  if (!logical || !weight256 || !scale256 || !bare256) return GQ_ERR_INVALID_ARGUMENT;
  std::string base = logical;
  const std::string suf = ".weight";
  if (base.size() >= suf.size() && base.compare(base.size() - suf.size(), suf.size(), suf) == 0)
    base.resize(base.size() - suf.size());
  std::string w, s, b;
  auto ends = [&](const std::string &t) {
    return base.size() >= t.size() && base.compare(base.size() - t.size(), t.size(), t) == 0;
  };
  if (base == "lm_head") {
    w = "lm_head.weight";
    s = "lm_head.weight_scale";
  } else {
    const std::string real = "model." + base;
    if (ends("embed_tokens") || ends("embed_tokens_per_layer")) {
      w = real + ".embedding_quantized";
      s = real + ".embedding_scale";
    } else {
      w = real + ".weight";
      s = real + ".weight_scale";
      b = real;
    }
  }
  if (w.size() >= 256 || s.size() >= 256 || b.size() >= 256) return GQ_ERR_INVALID_ARGUMENT;
  std::snprintf(weight256, 256, "%s", w.c_str());
  std::snprintf(scale256, 256, "%s", s.c_str());
  std::snprintf(bare256, 256, "%s", b.c_str());
  return GQ_OK;
}

int gq_st_upload_quant(gq_ctx *ctx, const gq_st_file *f, const char *logical, int32_t bits_u8, gq_qweight **out) {
  if (!ctx) return GQ_ERR_INVALID_ARGUMENT;
  if (!f || !logical || !out) return gq_set_error(ctx, GQ_ERR_INVALID_ARGUMENT, "st_upload_quant: null argument");
  *out = nullptr;
  char wn[256], sn[256], bn[256];
  if (gq_st_resolve(logical, wn, sn, bn) != GQ_OK)
    return gq_set_error(ctx, GQ_ERR_INVALID_ARGUMENT, std::string("st_upload_quant: name too long: ") + logical);
  const StMeta *m = find(f, wn);
  if (!m && bn[0]) m = find(f, bn);  // tensors stored without the .weight suffix
  if (!m) return gq_set_error(ctx, GQ_ERR_INVALID_ARGUMENT, std::string("st_upload_quant: no tensor for ") + logical);
  if (m->dtype != "U8" && m->dtype != "I8")
    return gq_set_error(ctx, GQ_ERR_UNSUPPORTED, std::string("st_upload_quant: ") + logical + " is " + m->dtype +
                                                     ", not a quantized U8/I8 tensor");
  if (m->shape.size() != 2)
    return gq_set_error(ctx, GQ_ERR_INVALID_ARGUMENT, std::string("st_upload_quant: ") + logical + " is not 2-D");
  const bool signed_i8 = m->dtype == "I8";
  const int32_t bits = signed_i8 ? 8 : bits_u8;
  if (bits != 2 && bits != 4 && bits != 8)
    return gq_set_error(ctx, GQ_ERR_UNSUPPORTED, std::string("st_upload_quant: bit width for ") + logical +
                                                     " is not 2, 4 or 8");
  const int64_t per_byte = signed_i8 ? 1 : 8 / bits;
  const int64_t n = m->shape[0], stored_cols = m->shape[1], k = stored_cols * per_byte;
  const StMeta *sm = find(f, sn);
  if (!sm) return gq_set_error(ctx, GQ_ERR_INVALID_ARGUMENT, std::string("quantized tensor ") + wn +
                                                                 " is missing its scale tensor " + sn);
  const int64_t scale_cols = sm->shape.size() >= 2 ? sm->shape[1] : 1;
  if (scale_cols <= 0 || k % scale_cols != 0 || (sm->shape.empty() ? 1 : sm->shape[0]) != n)
    return gq_set_error(ctx, GQ_ERR_INVALID_ARGUMENT, std::string("st_upload_quant: scale shape of ") + logical);
  const int64_t group = k / scale_cols;
  std::vector<float> scales((size_t)(n * scale_cols));
  int rc = gq_st_read_f32(f, sn, scales.data(), scales.size());
  if (rc != GQ_OK) return gq_set_error(ctx, rc, std::string("st_upload_quant: decoding the scales of ") + logical);
  const uint8_t *qb = nullptr;
  size_t qn = 0;
  if (!slice(f, *m, &qb, &qn) || (int64_t)qn != n * stored_cols)
    return gq_set_error(ctx, GQ_ERR_INVALID_ARGUMENT, std::string("st_upload_quant: payload size of ") + logical);
  return gq_qweight_upload(ctx, qb, qn, scales.data(), scales.size(), n, k, bits, signed_i8 ? 1 : 0, group, out);
}

}  // extern "C"
