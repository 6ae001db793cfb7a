// Base-model loading from Hugging Face safetensors shards, the counterpart of
// load_base_model_safetensors (src/model_io_impl.inc:57-190):
//   * the path is one .safetensors file or a directory whose *.safetensors
//     files are read in sorted order; a tensor name is looked up in that order;
//   * names: model.embed_tokens.weight, model.layers.{l}.{input_layernorm,
//     self_attn.{q,k,v,o}_proj, post_attention_layernorm,
//     mlp.{gate,up,down}_proj}.weight, model.norm.weight, lm_head.weight;
//   * lm_head.weight missing -> tied to the embedding; stored [D, V] ->
//     transposed to [V, D];
//   * BF16 / F16 / F32 accepted; the model stores bf16 (F32 -> bf16 with
//     round-to-nearest-even, F16 -> exact widening then bf16 rounding).
// Files are memory-mapped; each tensor is converted into one host staging
// buffer and copied into the model's fused layout by Model::set_weight.
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

#include "common.cuh"
#include "model.cuh"

namespace glt {
namespace {

struct StTensor {
  std::string dtype;
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;
};

struct StFile {
  std::string path;
  const uint8_t* map = nullptr;
  size_t size = 0;
  const uint8_t* data = nullptr;  // start of the byte buffer
  size_t data_size = 0;
  std::unordered_map<std::string, StTensor> tensors;
  ~StFile() {
    if (map) munmap(const_cast<uint8_t*>(map), size);
  }
};

// Minimal JSON reader for the safetensors header: objects, arrays, strings,
// integers; other scalars are skipped.
struct Json {
  const char* p;
  const char* e;
  std::string err;
  void ws() {
    while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t')) ++p;
  }
  bool expect(char c) {
    ws();
    if (p < e && *p == c) {
      ++p;
      return true;
    }
    err = std::string("expected '") + c + "'";
    return false;
  }
  bool str(std::string* out) {
    ws();
    if (p >= e || *p != '"') {
      err = "expected string";
      return false;
    }
    ++p;
    std::string s;
    while (p < e && *p != '"') {
      if (*p == '\\') {
        if (++p >= e) break;
        const char c = *p++;
        switch (c) {
          case 'n': s += '\n'; break;
          case 't': s += '\t'; break;
          case 'r': s += '\r'; break;
          case 'b': s += '\b'; break;
          case 'f': s += '\f'; break;
          case 'u': {  // keep the escape verbatim; tensor names are ASCII
            s += "\\u";
            for (int k = 0; k < 4 && p < e; ++k) s += *p++;
            break;
          }
          default: s += c;
        }
      } else {
        s += *p++;
      }
    }
    if (p >= e) {
      err = "unterminated string";
      return false;
    }
    ++p;
    if (out) *out = s;
    return true;
  }
  bool integer(int64_t* out) {
    ws();
    const char* q = p;
    if (q < e && (*q == '-' || *q == '+')) ++q;
    if (q >= e || *q < '0' || *q > '9') {
      err = "expected integer";
      return false;
    }
    char tmp[24];  // the mapping is not NUL-terminated: parse a bounded copy
    size_t n = 0;
    while (p + n < e && n + 1 < sizeof(tmp) && (p[n] == '-' || p[n] == '+' || (p[n] >= '0' && p[n] <= '9'))) {
      tmp[n] = p[n];
      ++n;
    }
    tmp[n] = 0;
    char* endp = nullptr;
    const long long v = strtoll(tmp, &endp, 10);
    if (endp == tmp) {
      err = "bad integer";
      return false;
    }
    p += endp - tmp;
    *out = v;
    return true;
  }
  bool skip() {  // any value
    ws();
    if (p >= e) {
      err = "unexpected end";
      return false;
    }
    if (*p == '"') return str(nullptr);
    if (*p == '{' || *p == '[') {
      const char open = *p, close = open == '{' ? '}' : ']';
      ++p;
      ws();
      if (p < e && *p == close) {
        ++p;
        return true;
      }
      for (;;) {
        if (open == '{') {
          if (!str(nullptr) || !expect(':')) return false;
        }
        if (!skip()) return false;
        ws();
        if (p < e && *p == ',') {
          ++p;
          continue;
        }
        return expect(close);
      }
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;  // number / literal
    return true;
  }
  bool int_array(std::vector<int64_t>* out) {
    if (!expect('[')) return false;
    ws();
    if (p < e && *p == ']') {
      ++p;
      return true;
    }
    for (;;) {
      int64_t v = 0;
      if (!integer(&v)) return false;
      out->push_back(v);
      ws();
      if (p < e && *p == ',') {
        ++p;
        continue;
      }
      return expect(']');
    }
  }
  bool tensor(StTensor* t) {
    if (!expect('{')) return false;
    ws();
    if (p < e && *p == '}') {
      ++p;
      return true;
    }
    for (;;) {
      std::string key;
      if (!str(&key) || !expect(':')) return false;
      if (key == "dtype") {
        if (!str(&t->dtype)) return false;
      } else if (key == "shape") {
        if (!int_array(&t->shape)) return false;
      } else if (key == "data_offsets") {
        std::vector<int64_t> o;
        if (!int_array(&o)) return false;
        if (o.size() != 2 || o[0] < 0 || o[1] < o[0]) {
          err = "bad data_offsets";
          return false;
        }
        t->begin = static_cast<uint64_t>(o[0]);
        t->end = static_cast<uint64_t>(o[1]);
      } else if (!skip()) {
        return false;
      }
      ws();
      if (p < e && *p == ',') {
        ++p;
        continue;
      }
      return expect('}');
    }
  }
};

int elem_size(const std::string& dt) {
  if (dt == "BF16" || dt == "F16") return 2;
  if (dt == "F32") return 4;
  return 0;
}

int open_file(const std::string& path, StFile* f) {
  f->path = path;
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return fail(GLT_EIO, "cannot open %s", path.c_str());
  struct stat sb;
  if (fstat(fd, &sb) != 0) {
    close(fd);
    return fail(GLT_EIO, "cannot stat %s", path.c_str());
  }
  f->size = static_cast<size_t>(sb.st_size);
  if (f->size < 8) {
    close(fd);
    return fail(GLT_EIO, "%s: too short for a safetensors header", path.c_str());
  }
  void* m = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) return fail(GLT_EIO, "cannot map %s", path.c_str());
  f->map = static_cast<const uint8_t*>(m);
  uint64_t hlen = 0;
  memcpy(&hlen, f->map, 8);  // little-endian u64
  if (hlen > f->size - 8) return fail(GLT_EIO, "%s: header length %llu exceeds the file", path.c_str(),
                                      (unsigned long long)hlen);
  f->data = f->map + 8 + hlen;
  f->data_size = f->size - 8 - hlen;
  Json j{reinterpret_cast<const char*>(f->map + 8), reinterpret_cast<const char*>(f->map + 8 + hlen), {}};
  if (!j.expect('{')) return fail(GLT_EIO, "%s: header: %s", path.c_str(), j.err.c_str());
  j.ws();
  if (j.p < j.e && *j.p == '}') return GLT_OK;
  for (;;) {
    std::string name;
    if (!j.str(&name) || !j.expect(':')) return fail(GLT_EIO, "%s: header: %s", path.c_str(), j.err.c_str());
    if (name == "__metadata__") {
      if (!j.skip()) return fail(GLT_EIO, "%s: header: %s", path.c_str(), j.err.c_str());
    } else {
      StTensor t;
      if (!j.tensor(&t)) return fail(GLT_EIO, "%s: tensor %s: %s", path.c_str(), name.c_str(), j.err.c_str());
      const int es = elem_size(t.dtype);
      int64_t numel = 1;
      for (int64_t d : t.shape) numel *= d;
      if (es && (t.end > f->data_size || t.end - t.begin != static_cast<uint64_t>(numel) * es))
        return fail(GLT_EIO, "%s: tensor %s: data_offsets do not match its shape and dtype",
                    path.c_str(), name.c_str());
      f->tensors.emplace(name, std::move(t));
    }
    j.ws();
    if (j.p < j.e && *j.p == ',') {
      ++j.p;
      continue;
    }
    if (!j.expect('}')) return fail(GLT_EIO, "%s: header: %s", path.c_str(), j.err.c_str());
    return GLT_OK;
  }
}

int open_all(const char* path, std::vector<std::unique_ptr<StFile>>* files) {
  struct stat sb;
  if (!path || stat(path, &sb) != 0)
    return fail(GLT_EIO, "safetensors path '%s' is not a file or directory", path ? path : "(null)");
  std::vector<std::string> paths;
  if (S_ISREG(sb.st_mode)) {
    paths.push_back(path);
  } else if (S_ISDIR(sb.st_mode)) {
    DIR* d = opendir(path);
    if (!d) return fail(GLT_EIO, "cannot list %s", path);
    while (dirent* ent = readdir(d)) {
      const std::string n = ent->d_name;
      const std::string ext = ".safetensors";
      if (n.size() > ext.size() && n.compare(n.size() - ext.size(), ext.size(), ext) == 0)
        paths.push_back(std::string(path) + "/" + n);
    }
    closedir(d);
    std::sort(paths.begin(), paths.end());
  } else {
    return fail(GLT_EIO, "safetensors path '%s' is not a file or directory", path);
  }
  if (paths.empty()) return fail(GLT_EIO, "no .safetensors files found at '%s'", path);
  for (const auto& p : paths) {
    files->emplace_back(new StFile());
    GLT_TRY(open_file(p, files->back().get()));
  }
  return GLT_OK;
}

const StTensor* lookup(const std::vector<std::unique_ptr<StFile>>& files, const std::string& name,
                       const StFile** owner) {
  for (const auto& f : files) {
    auto it = f->tensors.find(name);
    if (it != f->tensors.end()) {
      *owner = f.get();
      return &it->second;
    }
  }
  return nullptr;
}

uint16_t f32_bits_to_bf16(uint32_t bits) {
  if ((bits & 0x7F800000u) == 0x7F800000u && (bits & 0x007FFFFFu))  // NaN stays NaN
    return static_cast<uint16_t>((bits >> 16) | 0x40u);
  bits += ((bits >> 16) & 1u) + 0x7FFFu;
  return static_cast<uint16_t>(bits >> 16);
}

float half_to_float(uint16_t h) {
  const uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  const int exp = (h >> 10) & 0x1F;
  uint32_t mant = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else {  // subnormal half -> normal float
      int e = -1;
      do {
        ++e;
        mant <<= 1;
      } while (!(mant & 0x400u));
      bits = sign | static_cast<uint32_t>(127 - 15 - e) << 23 | (mant & 0x3FFu) << 13;
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | mant << 13;
  } else {
    bits = sign | static_cast<uint32_t>(exp - 15 + 127) << 23 | mant << 13;
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// Converts a tensor to bf16 in `out` (row-major as stored).
void to_bf16(const StFile& f, const StTensor& t, std::vector<uint16_t>* out) {
  int64_t n = 1;
  for (int64_t d : t.shape) n *= d;
  out->resize(static_cast<size_t>(n));
  const uint8_t* src = f.data + t.begin;
  if (t.dtype == "BF16") {
    memcpy(out->data(), src, static_cast<size_t>(n) * 2);
  } else if (t.dtype == "F32") {
    for (int64_t i = 0; i < n; ++i) {
      uint32_t b;
      memcpy(&b, src + 4 * i, 4);
      (*out)[i] = f32_bits_to_bf16(b);
    }
  } else {  // F16
    for (int64_t i = 0; i < n; ++i) {
      uint16_t h;
      memcpy(&h, src + 2 * i, 2);
      const float v = half_to_float(h);
      uint32_t b;
      memcpy(&b, &v, 4);
      (*out)[i] = f32_bits_to_bf16(b);
    }
  }
}

}  // namespace

int Model::load_safetensors(const char* path, cudaStream_t st) {
  if (kind != GLT_MODEL_DECODER) return fail(GLT_ESTATE, "safetensors loading needs the decoder model");
  std::vector<std::unique_ptr<StFile>> files;
  GLT_TRY(open_all(path, &files));
  std::vector<uint16_t> buf, tr;
  auto load = [&](const std::string& name, int layer, int which, int64_t rows, int64_t cols,
                  bool required, bool* found) -> int {
    const StFile* f = nullptr;
    const StTensor* t = lookup(files, name, &f);
    if (found) *found = t != nullptr;
    if (!t) return required ? fail(GLT_EIO, "%s not found in safetensors", name.c_str()) : GLT_OK;
    if (!elem_size(t->dtype))
      return fail(GLT_EIO, "%s: unsupported safetensors dtype %s", name.c_str(), t->dtype.c_str());
    int64_t numel = 1;
    for (int64_t d : t->shape) numel *= d;
    const bool vec = cols == 0;
    const bool ok = vec ? (t->shape.size() == 1 && t->shape[0] == rows)
                        : (t->shape.size() == 2 && t->shape[0] == rows && t->shape[1] == cols);
    // lm_head stored [D, V] is transposed to [V, D] (model_io_impl.inc:128-133)
    const bool transposed = !ok && which == GLT_W_LM_HEAD && t->shape.size() == 2 &&
                            t->shape[0] == cols && t->shape[1] == rows && rows != cols;
    if (!ok && !transposed) {
      std::string got;
      for (size_t i = 0; i < t->shape.size(); ++i) got += (i ? ", " : "") + std::to_string(t->shape[i]);
      return fail(GLT_EINVAL, "%s has shape [%s], expected [%lld%s%s]", name.c_str(), got.c_str(),
                  (long long)rows, vec ? "" : ", ", vec ? "" : std::to_string(cols).c_str());
    }
    to_bf16(*f, *t, &buf);
    const uint16_t* src = buf.data();
    if (transposed) {
      tr.resize(buf.size());
      for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) tr[r * cols + c] = buf[c * rows + r];
      src = tr.data();
    }
    GLT_TRY(set_weight(layer, which, src, numel, 1, st));
    GLT_CUDA_TRY(cudaStreamSynchronize(st));  // the staging buffer is reused
    return GLT_OK;
  };
  GLT_TRY(load("model.embed_tokens.weight", -1, GLT_W_EMBED, V, D, true, nullptr));
  for (int l = 0; l < L; ++l) {
    const std::string p = "model.layers." + std::to_string(l) + ".";
    GLT_TRY(load(p + "input_layernorm.weight", l, GLT_W_IN_NORM, D, 0, true, nullptr));
    GLT_TRY(load(p + "self_attn.q_proj.weight", l, GLT_W_Q, static_cast<int64_t>(nh) * hd, D, true, nullptr));
    GLT_TRY(load(p + "self_attn.k_proj.weight", l, GLT_W_K, static_cast<int64_t>(nkv) * hd, D, true, nullptr));
    GLT_TRY(load(p + "self_attn.v_proj.weight", l, GLT_W_V, static_cast<int64_t>(nkv) * hd, D, true, nullptr));
    GLT_TRY(load(p + "self_attn.o_proj.weight", l, GLT_W_O, D, static_cast<int64_t>(nh) * hd, true, nullptr));
    GLT_TRY(load(p + "post_attention_layernorm.weight", l, GLT_W_POST_NORM, D, 0, true, nullptr));
    GLT_TRY(load(p + "mlp.gate_proj.weight", l, GLT_W_GATE, F, D, true, nullptr));
    GLT_TRY(load(p + "mlp.up_proj.weight", l, GLT_W_UP, F, D, true, nullptr));
    GLT_TRY(load(p + "mlp.down_proj.weight", l, GLT_W_DOWN, D, F, true, nullptr));
  }
  GLT_TRY(load("model.norm.weight", -1, GLT_W_FINAL_NORM, D, 0, true, nullptr));
  const StFile* f = nullptr;
  const bool has_head = lookup(files, "lm_head.weight", &f) != nullptr;
  if (has_head && cfg.tie_embeddings)
    return fail(GLT_EINVAL, "the safetensors hold a separate lm_head.weight; create the model with "
                "tie_embeddings = 0");
  if (!has_head && !cfg.tie_embeddings)
    return fail(GLT_EINVAL, "lm_head.weight not found (tied to the embedding); create the model with "
                "tie_embeddings = 1");
  if (has_head) GLT_TRY(load("lm_head.weight", -1, GLT_W_LM_HEAD, V, D, true, nullptr));
  return GLT_OK;
}

}  // namespace glt

extern "C" int glt_safetensors_tensor_info(const char* path, const char* name, int* found,
                                           int64_t* shape, int* ndim) {
  if (!name || !found) return glt::fail(GLT_EINVAL, "null argument");
  std::vector<std::unique_ptr<glt::StFile>> files;
  GLT_TRY(glt::open_all(path, &files));
  const glt::StFile* f = nullptr;
  const glt::StTensor* t = glt::lookup(files, name, &f);
  *found = t != nullptr;
  if (t) {
    if (ndim) *ndim = static_cast<int>(t->shape.size());
    if (shape)
      for (size_t i = 0; i < t->shape.size() && i < 8; ++i) shape[i] = t->shape[i];
  }
  return GLT_OK;
}

extern "C" int glt_model_load_safetensors(GltModel* m, const char* path, void* stream) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  return reinterpret_cast<glt::Model*>(m)->load_safetensors(path, static_cast<cudaStream_t>(stream));
}
