// Host-side I/O of the graft path: the GRFT checkpoint (src/checkpoint_impl.inc),
// the training-state file (fp32 graft + Adam moments + step, which the
// reference does not keep), the .bin token files and the seeded batch walk
// (src/data_impl.inc, grafting.hip:924-988).  Pure C++ (no device code)
// except for the optional device source/destination of the weights; these
// entry points work on GPU-less hosts when given host buffers.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/stat.h>

#include <map>
#include <string>
#include <vector>

#include "common.cuh"
#include "model.cuh"

namespace glt {
namespace {

constexpr uint32_t kGrftMagic = 0x54465247u;  // "GRFT" little endian
constexpr uint8_t kGrftVersion = 4;

bool is_dir(const char* p) {
  struct stat s;
  return stat(p, &s) == 0 && S_ISDIR(s.st_mode);
}

std::string parent_of(const std::string& p) {
  const size_t k = p.find_last_of('/');
  return k == std::string::npos ? std::string() : p.substr(0, k);
}

// The header text of build_safetensors_header (checkpoint_impl.inc:8-30),
// byte for byte (values are not escaped, as in the reference).
std::string grft_header(const char* session, int domain, int S, int H, int D, int L) {
  const long long total = 3LL * L;
  const long long nbytes = total * S * static_cast<long long>(H) * 2;
  char buf[1024];
  std::string s = "{\"__metadata__\":{\"session_id\":\"";
  s += session ? session : "";
  snprintf(buf, sizeof(buf),
           "\",\"domain_id\":\"%d\",\"slice_dim\":\"%d\",\"h_slice_dim\":\"%d\",\"hidden_dim\":\"%d\","
           "\"num_layers\":\"%d\"},\"delta_weights\":{\"dtype\":\"BF16\",\"shape\":[%lld,%d,%d],"
           "\"data_offsets\":[0,%lld]}}",
           domain, S, H, D, L, total, S, H, nbytes);
  s += buf;
  return s;
}

// ---- a small JSON reader, enough for safetensors headers ----
struct Json {
  const char* p;
  const char* e;
  bool ok = true;
  void ws() { while (p < e && (*p == ' ' || *p == '\n' || *p == '\r' || *p == '\t' || *p == '\0')) ++p; }
  bool eat(char c) { ws(); if (p < e && *p == c) { ++p; return true; } return false; }
  bool str(std::string& out) {
    ws();
    if (p >= e || *p != '"') return ok = false;
    ++p;
    out.clear();
    while (p < e && *p != '"') {
      if (*p == '\\' && p + 1 < e) { ++p; }
      out.push_back(*p++);
    }
    if (p >= e) return ok = false;
    ++p;
    return true;
  }
  bool num(long long& v) {
    ws();
    char* end = nullptr;
    v = strtoll(p, &end, 10);
    if (end == p) return ok = false;
    p = end;
    return true;
  }
  // Skips any value.
  bool skip() {
    ws();
    if (p >= e) return ok = false;
    if (*p == '"') { std::string t; return str(t); }
    if (*p == '{' || *p == '[') {
      const char open = *p, close = open == '{' ? '}' : ']';
      ++p;
      if (eat(close)) return true;
      while (ok) {
        if (open == '{') { std::string k; if (!str(k) || !eat(':')) return ok = false; }
        if (!skip()) return false;
        if (eat(',')) continue;
        if (eat(close)) return true;
        return ok = false;
      }
      return false;
    }
    while (p < e && *p != ',' && *p != '}' && *p != ']') ++p;
    return true;
  }
};

struct StHeader {
  std::string dtype;
  std::vector<long long> shape;
  long long off0 = -1, off1 = -1;
  bool has_tensor = false;
  std::string session;
  int domain = -1;
};

bool parse_header(const char* p, size_t n, StHeader& h) {
  Json j{p, p + n};
  if (!j.eat('{')) return false;
  if (j.eat('}')) return true;
  while (j.ok) {
    std::string key;
    if (!j.str(key) || !j.eat(':')) return false;
    if (key == "__metadata__") {
      if (!j.eat('{')) return false;
      if (!j.eat('}')) {
        while (j.ok) {
          std::string k, v;
          if (!j.str(k) || !j.eat(':') || !j.str(v)) return false;
          if (k == "session_id") h.session = v;
          if (k == "domain_id") h.domain = atoi(v.c_str());
          if (j.eat(',')) continue;
          if (j.eat('}')) break;
          return false;
        }
      }
    } else if (key == "delta_weights") {
      h.has_tensor = true;
      if (!j.eat('{')) return false;
      while (j.ok) {
        std::string k;
        if (!j.str(k) || !j.eat(':')) return false;
        if (k == "dtype") {
          if (!j.str(h.dtype)) return false;
        } else if (k == "shape" || k == "data_offsets") {
          if (!j.eat('[')) return false;
          std::vector<long long> v;
          if (!j.eat(']')) {
            while (true) {
              long long x;
              if (!j.num(x)) return false;
              v.push_back(x);
              if (j.eat(',')) continue;
              if (j.eat(']')) break;
              return false;
            }
          }
          if (k == "shape") h.shape = v;
          else if (v.size() == 2) { h.off0 = v[0]; h.off1 = v[1]; }
        } else if (!j.skip()) {
          return false;
        }
        if (j.eat(',')) continue;
        if (j.eat('}')) break;
        return false;
      }
    } else if (!j.skip()) {
      return false;
    }
    if (j.eat(',')) continue;
    if (j.eat('}')) return true;
    return false;
  }
  return false;
}

// ---- training state ("GLTS") ----
constexpr uint32_t kStateMagic = 0x53544C47u;  // "GLTS" little endian
constexpr uint8_t kStateVersion = 1;
const char* const kStateTensors[3] = {"weights", "adam_m", "adam_v"};

std::string json_escape(const char* s) {
  std::string o;
  for (; s && *s; ++s) {
    const unsigned char c = static_cast<unsigned char>(*s);
    if (c == '"' || c == '\\') { o.push_back('\\'); o.push_back(static_cast<char>(c)); }
    else if (c < 0x20) { char b[8]; snprintf(b, sizeof(b), "\\u%04x", c); o += b; }
    else o.push_back(static_cast<char>(c));
  }
  return o;
}

std::string state_header(const char* session, int domain, int S, int H, int D, int L, long long step) {
  const long long total = 3LL * L;
  const long long nb = total * S * static_cast<long long>(H) * 4;
  char buf[256];
  std::string s = "{\"__metadata__\":{\"format\":\"glt-train-state\",\"session_id\":\"";
  s += json_escape(session);
  snprintf(buf, sizeof(buf),
           "\",\"domain_id\":\"%d\",\"slice_dim\":\"%d\",\"h_slice_dim\":\"%d\",\"hidden_dim\":\"%d\","
           "\"num_layers\":\"%d\",\"step\":\"%lld\"}",
           domain, S, H, D, L, step);
  s += buf;
  for (int t = 0; t < 3; ++t) {
    snprintf(buf, sizeof(buf), ",\"%s\":{\"dtype\":\"F32\",\"shape\":[%lld,%d,%d],\"data_offsets\":[%lld,%lld]}",
             kStateTensors[t], total, S, H, nb * t, nb * (t + 1));
    s += buf;
  }
  return s + "}";
}

struct StTensor {
  std::string dtype;
  std::vector<long long> shape;
  long long off0 = -1, off1 = -1;
};

// Any safetensors-style header: string metadata and every tensor entry.
bool parse_header_all(const char* p, size_t n, std::map<std::string, std::string>& meta,
                      std::map<std::string, StTensor>& tensors) {
  Json j{p, p + n};
  if (!j.eat('{')) return false;
  if (j.eat('}')) return true;
  while (j.ok) {
    std::string key;
    if (!j.str(key) || !j.eat(':')) return false;
    if (key == "__metadata__") {
      if (!j.eat('{')) return false;
      if (!j.eat('}')) {
        while (j.ok) {
          std::string k, v;
          if (!j.str(k) || !j.eat(':') || !j.str(v)) return false;
          meta[k] = v;
          if (j.eat(',')) continue;
          if (j.eat('}')) break;
          return false;
        }
      }
    } else {
      StTensor t;
      if (!j.eat('{')) return false;
      while (j.ok) {
        std::string k;
        if (!j.str(k) || !j.eat(':')) return false;
        if (k == "dtype") {
          if (!j.str(t.dtype)) return false;
        } else if (k == "shape" || k == "data_offsets") {
          if (!j.eat('[')) return false;
          std::vector<long long> v;
          if (!j.eat(']')) {
            while (true) {
              long long x;
              if (!j.num(x)) return false;
              v.push_back(x);
              if (j.eat(',')) continue;
              if (j.eat(']')) break;
              return false;
            }
          }
          if (k == "shape") t.shape = v;
          else if (v.size() == 2) { t.off0 = v[0]; t.off1 = v[1]; }
        } else if (!j.skip()) {
          return false;
        }
        if (j.eat(',')) continue;
        if (j.eat('}')) break;
        return false;
      }
      tensors[key] = t;
    }
    if (j.eat(',')) continue;
    if (j.eat('}')) return true;
    return false;
  }
  return false;
}

bool read_file(const char* path, std::vector<char>& buf) {
  FILE* f = fopen(path, "rb");
  if (!f) return false;
  fseek(f, 0, SEEK_END);
  long n = ftell(f);
  fseek(f, 0, SEEK_SET);
  if (n < 0) { fclose(f); return false; }
  buf.resize(static_cast<size_t>(n));
  const size_t got = n ? fread(buf.data(), 1, static_cast<size_t>(n), f) : 0;
  fclose(f);
  return got == static_cast<size_t>(n);
}

}  // namespace

int checkpoint_save(const char* path, const float* host_w, int64_t numel, const char* session,
                    int domain, int S, int H, int D, int L) {
  if (!path || !host_w) return fail(GLT_EINVAL, "null argument");
  if (numel != 3LL * L * S * H) return fail(GLT_EINVAL, "weights numel %lld != 3*L*S*H", (long long)numel);
  if (is_dir(path)) return fail(GLT_EIO, "save_safetensors: path is a directory, not a file: %s", path);
  const std::string par = parent_of(path);
  if (!par.empty() && !is_dir(par.c_str()))
    return fail(GLT_EIO, "save_safetensors: parent directory does not exist: %s", par.c_str());
  const std::string hdr = grft_header(session, domain, S, H, D, L);
  const uint64_t pad = (8 - hdr.size() % 8) % 8;
  const uint64_t hsize = hdr.size() + pad;
  std::vector<uint16_t> bf(static_cast<size_t>(numel));
  for (int64_t i = 0; i < numel; ++i) bf[static_cast<size_t>(i)] = f32_to_bf16_bits(host_w[i]);
  FILE* f = fopen(path, "wb");
  if (!f) return fail(GLT_EIO, "cannot open %s for writing", path);
  const uint32_t magic = kGrftMagic;
  const uint8_t ver = kGrftVersion;
  bool ok = fwrite(&magic, 4, 1, f) == 1 && fwrite(&ver, 1, 1, f) == 1 &&
            fwrite(&hsize, 8, 1, f) == 1 && fwrite(hdr.data(), 1, hdr.size(), f) == hdr.size();
  for (uint64_t i = 0; ok && i < pad; ++i) ok = fputc(0, f) != EOF;
  if (ok && numel) ok = fwrite(bf.data(), 2, bf.size(), f) == bf.size();
  ok = (fclose(f) == 0) && ok;
  if (!ok) return fail(GLT_EIO, "short write to %s", path);
  return GLT_OK;
}

int checkpoint_load(const char* path, float* host_w, int64_t numel, int expected_domain,
                    const char* session, int total_proj, int S, int H, int* file_domain) {
  if (!path || !host_w) return fail(GLT_EINVAL, "null argument");
  std::vector<char> buf;
  if (!read_file(path, buf)) return fail(GLT_EIO, "cannot open checkpoint %s", path);
  size_t off = 0;
  uint32_t magic = 0;
  if (buf.size() >= 5) memcpy(&magic, buf.data(), 4);
  if (buf.size() >= 5 && magic == kGrftMagic) off = 5;  // GRFT magic + version byte
  if (buf.size() < off + 8) return fail(GLT_EIO, "safetensors parse failed: file too small");
  uint64_t hlen = 0;
  memcpy(&hlen, buf.data() + off, 8);
  if (hlen > buf.size() - off - 8) return fail(GLT_EIO, "safetensors parse failed: header past end of file");
  StHeader h;
  if (!parse_header(buf.data() + off + 8, static_cast<size_t>(hlen), h))
    return fail(GLT_EIO, "safetensors parse failed: bad JSON header");
  if (!h.has_tensor) return fail(GLT_EIO, "'delta_weights' not found in %s", path);
  if (h.dtype != "BF16") return fail(GLT_EIO, "delta_weights dtype is not BF16");
  if (h.shape.size() != 3 || h.shape[0] != total_proj || h.shape[1] != S || h.shape[2] != H)
    return fail(GLT_EIO, "delta_weights shape mismatch. Expected [%d,%d,%d]", total_proj, S, H);
  if (session && *session && !h.session.empty() && h.session != session)
    return fail(GLT_EIO, "session_id mismatch! Checkpoint has '%s', current training session is '%s'",
                h.session.c_str(), session);
  if (h.domain != -1 && h.domain != expected_domain)
    return fail(GLT_EIO, "checkpoint domain_id mismatch. Checkpoint has %d, current --domain-id is %d",
                h.domain, expected_domain);
  const int64_t n = static_cast<int64_t>(total_proj) * S * H;
  if (numel != n) return fail(GLT_EINVAL, "destination holds %lld elements, need %lld", (long long)numel, (long long)n);
  const uint64_t data0 = off + 8 + hlen;
  if (h.off0 < 0 || h.off1 < h.off0 || data0 + static_cast<uint64_t>(h.off1) > buf.size() ||
      static_cast<uint64_t>(h.off1 - h.off0) < static_cast<uint64_t>(n) * 2)
    return fail(GLT_EIO, "truncated tensor data in %s", path);
  const uint8_t* src = reinterpret_cast<const uint8_t*>(buf.data()) + data0 + h.off0;
  for (int64_t i = 0; i < n; ++i) {
    uint16_t b;
    memcpy(&b, src + 2 * i, 2);
    host_w[i] = bf16_bits_to_f32(b);
  }
  if (file_domain) *file_domain = h.domain;
  return GLT_OK;
}

// Training state.  Each of the three tensors goes through `host_buf`
// (numel floats): `fetch(t, host_buf)` supplies tensor t for a save and
// `store(t, host_buf)` takes it after a load, so a device-resident state
// needs one host staging buffer rather than three.
template <class Fetch>
int train_state_write(const char* path, int64_t numel, const char* session, int domain, int S, int H,
                      int D, int L, int64_t step, float* host_buf, Fetch fetch) {
  if (!path) return fail(GLT_EINVAL, "null argument");
  if (numel != 3LL * L * S * H) return fail(GLT_EINVAL, "state numel %lld != 3*L*S*H", (long long)numel);
  if (step < 0) return fail(GLT_EINVAL, "step must be >= 0");
  if (is_dir(path)) return fail(GLT_EIO, "train state: path is a directory, not a file: %s", path);
  const std::string par = parent_of(path);
  if (!par.empty() && !is_dir(par.c_str()))
    return fail(GLT_EIO, "train state: parent directory does not exist: %s", par.c_str());
  const std::string hdr = state_header(session, domain, S, H, D, L, step);
  const uint64_t pad = (8 - hdr.size() % 8) % 8;
  const uint64_t hsize = hdr.size() + pad;
  FILE* f = fopen(path, "wb");
  if (!f) return fail(GLT_EIO, "cannot open %s for writing", path);
  const uint32_t magic = kStateMagic;
  const uint8_t ver = kStateVersion;
  bool ok = fwrite(&magic, 4, 1, f) == 1 && fwrite(&ver, 1, 1, f) == 1 &&
            fwrite(&hsize, 8, 1, f) == 1 && fwrite(hdr.data(), 1, hdr.size(), f) == hdr.size();
  for (uint64_t i = 0; ok && i < pad; ++i) ok = fputc(0, f) != EOF;
  for (int t = 0; ok && t < 3; ++t) {
    const int st = fetch(t, host_buf);
    if (st != GLT_OK) { fclose(f); return st; }
    ok = numel == 0 || fwrite(host_buf, 4, static_cast<size_t>(numel), f) == static_cast<size_t>(numel);
  }
  ok = (fclose(f) == 0) && ok;
  if (!ok) return fail(GLT_EIO, "short write to %s", path);
  return GLT_OK;
}

template <class Store>
int train_state_read(const char* path, int64_t numel, const char* session, int expected_domain,
                     int total_proj, int S, int H, int64_t* step_out, float* host_buf, Store store) {
  if (!path) return fail(GLT_EINVAL, "null argument");
  FILE* f = fopen(path, "rb");
  if (!f) return fail(GLT_EIO, "cannot open train state %s", path);
  struct Closer { FILE* f; ~Closer() { fclose(f); } } closer{f};
  fseeko(f, 0, SEEK_END);
  const int64_t fsize = static_cast<int64_t>(ftello(f));
  fseeko(f, 0, SEEK_SET);
  uint32_t magic = 0;
  uint8_t ver = 0;
  uint64_t hlen = 0;
  if (fsize < 13 || fread(&magic, 4, 1, f) != 1 || fread(&ver, 1, 1, f) != 1 || fread(&hlen, 8, 1, f) != 1)
    return fail(GLT_EIO, "train state %s: file too small", path);
  if (magic != kStateMagic) return fail(GLT_EIO, "%s is not a training-state file (magic)", path);
  if (ver != kStateVersion) return fail(GLT_EIO, "train state %s: unsupported version %d", path, ver);
  if (hlen > static_cast<uint64_t>(fsize - 13)) return fail(GLT_EIO, "train state: header past end of file");
  std::string hdr(static_cast<size_t>(hlen), '\0');
  if (hlen && fread(&hdr[0], 1, static_cast<size_t>(hlen), f) != hlen)
    return fail(GLT_EIO, "train state: short header read");
  std::map<std::string, std::string> meta;
  std::map<std::string, StTensor> tensors;
  if (!parse_header_all(hdr.data(), hdr.size(), meta, tensors))
    return fail(GLT_EIO, "train state parse failed: bad JSON header");
  if (meta["format"] != "glt-train-state") return fail(GLT_EIO, "train state: wrong format tag");
  if (session && *session && !meta["session_id"].empty() && meta["session_id"] != session)
    return fail(GLT_EIO, "session_id mismatch! State has '%s', current training session is '%s'",
                meta["session_id"].c_str(), session);
  if (meta.count("domain_id") == 0 || atoi(meta["domain_id"].c_str()) != expected_domain)
    return fail(GLT_EIO, "train state domain_id mismatch: state has %s, expected %d",
                meta.count("domain_id") ? meta["domain_id"].c_str() : "none", expected_domain);
  if (meta.count("step") == 0) return fail(GLT_EIO, "train state: no step");
  const long long step = atoll(meta["step"].c_str());
  if (step < 0) return fail(GLT_EIO, "train state: negative step");
  const int64_t n = static_cast<int64_t>(total_proj) * S * H;
  if (numel != n) return fail(GLT_EINVAL, "destination holds %lld elements, need %lld", (long long)numel, (long long)n);
  const int64_t data0 = 13 + static_cast<int64_t>(hlen);
  for (int t = 0; t < 3; ++t) {
    auto it = tensors.find(kStateTensors[t]);
    if (it == tensors.end()) return fail(GLT_EIO, "'%s' not found in %s", kStateTensors[t], path);
    const StTensor& ts = it->second;
    if (ts.dtype != "F32") return fail(GLT_EIO, "%s dtype is not F32", kStateTensors[t]);
    if (ts.shape.size() != 3 || ts.shape[0] != total_proj || ts.shape[1] != S || ts.shape[2] != H)
      return fail(GLT_EIO, "%s shape mismatch. Expected [%d,%d,%d]", kStateTensors[t], total_proj, S, H);
    if (ts.off0 < 0 || ts.off1 - ts.off0 != n * 4 || data0 + ts.off1 > fsize)
      return fail(GLT_EIO, "truncated %s data in %s", kStateTensors[t], path);
    if (fseeko(f, static_cast<off_t>(data0 + ts.off0), SEEK_SET) != 0 ||
        (n && fread(host_buf, 4, static_cast<size_t>(n), f) != static_cast<size_t>(n)))
      return fail(GLT_EIO, "short read of %s from %s", kStateTensors[t], path);
    GLT_TRY(store(t, host_buf));
  }
  if (step_out) *step_out = step;
  return GLT_OK;
}

}  // namespace glt

// ------------------------------- C ABI -------------------------------------
static int copy_weights(void* dst, const void* src, int64_t bytes, int dst_host, int src_host) {
  if (dst_host && src_host) {
    memcpy(dst, src, static_cast<size_t>(bytes));
    return GLT_OK;
  }
  GLT_CUDA_TRY(cudaMemcpy(dst, src, static_cast<size_t>(bytes), cudaMemcpyDefault));
  return GLT_OK;
}

extern "C" int glt_checkpoint_save(const char* path, const float* weights, int64_t numel,
                                   int src_is_host, const char* session_id, int domain_id,
                                   int slice_dim, int h_slice_dim, int hidden_dim, int num_layers) {
  if (!weights) return glt::fail(GLT_EINVAL, "null weights");
  std::vector<float> host;
  const float* hw = weights;
  if (!src_is_host) {
    host.resize(static_cast<size_t>(numel));
    GLT_TRY(copy_weights(host.data(), weights, numel * 4, 1, 0));
    hw = host.data();
  }
  return glt::checkpoint_save(path, hw, numel, session_id, domain_id, slice_dim, h_slice_dim,
                              hidden_dim, num_layers);
}

extern "C" int glt_checkpoint_load(const char* path, float* weights, int64_t numel, int dst_is_host,
                                   int expected_domain_id, const char* session_id,
                                   int total_projections, int slice_dim, int h_slice_dim,
                                   int* file_domain_id) {
  if (!weights) return glt::fail(GLT_EINVAL, "null weights");
  if (dst_is_host)
    return glt::checkpoint_load(path, weights, numel, expected_domain_id, session_id,
                                total_projections, slice_dim, h_slice_dim, file_domain_id);
  std::vector<float> host(static_cast<size_t>(numel > 0 ? numel : 0));
  GLT_TRY(glt::checkpoint_load(path, host.data(), numel, expected_domain_id, session_id,
                               total_projections, slice_dim, h_slice_dim, file_domain_id));
  return copy_weights(weights, host.data(), numel * 4, 0, 1);
}

extern "C" int glt_model_save_checkpoint(GltModel* m, const char* path, const char* session_id,
                                         int domain_id) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  glt::Model* mm = reinterpret_cast<glt::Model*>(m);
  if (!mm->gw) return glt::fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  GLT_CUDA_TRY(cudaDeviceSynchronize());
  return glt_checkpoint_save(path, mm->gw, mm->graft_numel, 0, session_id, domain_id, mm->S,
                             mm->H, mm->D, mm->L);
}

extern "C" int glt_model_load_checkpoint(GltModel* m, const char* path, const char* session_id,
                                         int expected_domain_id) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  glt::Model* mm = reinterpret_cast<glt::Model*>(m);
  if (!mm->gw) return glt::fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  GLT_TRY(glt_checkpoint_load(path, mm->gw, mm->graft_numel, 0, expected_domain_id, session_id,
                              3 * mm->L, mm->S, mm->H, nullptr));
  GLT_TRY(mm->refresh_graft(nullptr));
  GLT_CUDA_TRY(cudaDeviceSynchronize());
  return GLT_OK;
}

extern "C" int glt_train_state_save(const char* path, const float* weights, const float* adam_m,
                                    const float* adam_v, int64_t numel, int src_is_host,
                                    const char* session_id, int domain_id, int slice_dim,
                                    int h_slice_dim, int hidden_dim, int num_layers, int64_t step) {
  if (!weights || !adam_m || !adam_v) return glt::fail(GLT_EINVAL, "null state buffer");
  if (numel < 0) return glt::fail(GLT_EINVAL, "negative numel");
  const float* src[3] = {weights, adam_m, adam_v};
  std::vector<float> host(src_is_host ? 0 : static_cast<size_t>(numel));
  float* hb = host.data();
  return glt::train_state_write(path, numel, session_id, domain_id, slice_dim, h_slice_dim, hidden_dim,
                                num_layers, step, src_is_host ? nullptr : hb,
                                [&](int t, float*& buf) -> int {
                                  if (src_is_host) { buf = const_cast<float*>(src[t]); return GLT_OK; }
                                  return copy_weights(buf, src[t], numel * 4, 1, 0);
                                });
}

extern "C" int glt_train_state_load(const char* path, float* weights, float* adam_m, float* adam_v,
                                    int64_t numel, int dst_is_host, const char* session_id,
                                    int expected_domain_id, int total_projections, int slice_dim,
                                    int h_slice_dim, int64_t* step) {
  if (!weights || !adam_m || !adam_v) return glt::fail(GLT_EINVAL, "null state buffer");
  if (numel < 0) return glt::fail(GLT_EINVAL, "negative numel");
  float* dst[3] = {weights, adam_m, adam_v};
  std::vector<float> host(static_cast<size_t>(numel));
  // read into a scratch buffer first, so a file that fails a check part way
  // leaves the caller's buffers as they were
  std::vector<float> staged(dst_is_host ? 3 * static_cast<size_t>(numel) : 0);
  int64_t st_step = 0;
  GLT_TRY(glt::train_state_read(path, numel, session_id, expected_domain_id, total_projections, slice_dim,
                                h_slice_dim, &st_step, host.data(), [&](int t, float* buf) -> int {
                                  if (dst_is_host) {
                                    memcpy(staged.data() + static_cast<size_t>(t) * numel, buf,
                                           static_cast<size_t>(numel) * 4);
                                    return GLT_OK;
                                  }
                                  return copy_weights(dst[t], buf, numel * 4, 0, 1);
                                }));
  if (dst_is_host)
    for (int t = 0; t < 3; ++t)
      memcpy(dst[t], staged.data() + static_cast<size_t>(t) * numel, static_cast<size_t>(numel) * 4);
  if (step) *step = st_step;
  return GLT_OK;
}

extern "C" int glt_model_save_train_state(GltModel* m, const char* path, const char* session_id,
                                          int domain_id, int64_t step) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  glt::Model* mm = reinterpret_cast<glt::Model*>(m);
  if (!mm->gw) return glt::fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  GLT_CUDA_TRY(cudaDeviceSynchronize());
  return glt_train_state_save(path, mm->gw, mm->adam_m, mm->adam_v, mm->graft_numel, 0, session_id,
                              domain_id, mm->S, mm->H, mm->D, mm->L, step);
}

extern "C" int glt_model_load_train_state(GltModel* m, const char* path, const char* session_id,
                                          int expected_domain_id, int64_t* step) {
  if (!m) return glt::fail(GLT_EINVAL, "null model");
  glt::Model* mm = reinterpret_cast<glt::Model*>(m);
  if (!mm->gw) return glt::fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  if (mm->shadow_baked) return glt::fail(GLT_ESTATE, "the model is shadow-baked");
  GLT_CUDA_TRY(cudaDeviceSynchronize());
  GLT_TRY(glt_train_state_load(path, mm->gw, mm->adam_m, mm->adam_v, mm->graft_numel, 0, session_id,
                               expected_domain_id, 3 * mm->L, mm->S, mm->H, step));
  GLT_TRY(mm->refresh_graft(nullptr));
  GLT_CUDA_TRY(cudaDeviceSynchronize());
  return GLT_OK;
}

// --------------------------- sibling-graft stacks ---------------------------
// The model's graft [3L, S, H] holds N siblings of S / N rows each: concat
// geometry side by side over the full hidden width, the overlay stack
// geometry (max_domains 1) block-diagonal with H / N columns each.
namespace {
struct StackGeom {
  int n, S_sib, H_sib;
  bool diag;
};

int stack_geom(const glt::Model* mm, int n, StackGeom* g) {
  if (n < 1) return glt::fail(GLT_EINVAL, "stack needs at least one sibling");
  if (mm->S % n) return glt::fail(GLT_EINVAL, "slice_dim %d is not a multiple of %d siblings", mm->S, n);
  g->n = n;
  g->S_sib = mm->S / n;
  g->diag = mm->overlay;
  if (mm->overlay) {
    if (mm->cfg.max_domains != 1 || mm->cfg.domain_id != 0)
      return glt::fail(GLT_EINVAL, "an overlay stack uses max_domains = 1, domain_id = 0");
    if (mm->H % n) return glt::fail(GLT_EINVAL, "hidden slice %d is not a multiple of %d siblings", mm->H, n);
    g->H_sib = mm->H / n;
  } else {
    g->H_sib = mm->H;
  }
  return GLT_OK;
}

// Copies sibling d between the stacked graft `all` [3L, S, H] and `sib`
// [3L, S_sib, H_sib] (to_sib: extract; else place).
void stack_copy(const StackGeom& g, int L, int S, int H, int d, float* all, float* sib, bool to_sib) {
  const int c0 = g.diag ? d * g.H_sib : 0;
  for (int64_t p = 0; p < 3LL * L; ++p)
    for (int s = 0; s < g.S_sib; ++s) {
      float* a = all + (p * S + static_cast<int64_t>(d) * g.S_sib + s) * H + c0;
      float* b = sib + (p * g.S_sib + s) * g.H_sib;
      if (to_sib) memcpy(b, a, sizeof(float) * g.H_sib);
      else memcpy(a, b, sizeof(float) * g.H_sib);
    }
}
}  // namespace

extern "C" int glt_model_save_stack(GltModel* m, const char* const* paths, int n, const char* session_id) {
  if (!m || !paths) return glt::fail(GLT_EINVAL, "null argument");
  glt::Model* mm = reinterpret_cast<glt::Model*>(m);
  if (!mm->gw) return glt::fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  StackGeom g;
  GLT_TRY(stack_geom(mm, n, &g));
  for (int d = 0; d < n; ++d)
    if (!paths[d]) return glt::fail(GLT_EINVAL, "null path for sibling %d", d);
  GLT_CUDA_TRY(cudaDeviceSynchronize());
  std::vector<float> all(static_cast<size_t>(mm->graft_numel));
  GLT_TRY(copy_weights(all.data(), mm->gw, mm->graft_numel * 4, 1, 0));
  const int64_t n_sib = 3LL * mm->L * g.S_sib * g.H_sib;
  std::vector<float> sib(static_cast<size_t>(n_sib));
  for (int d = 0; d < n; ++d) {
    stack_copy(g, mm->L, mm->S, mm->H, d, all.data(), sib.data(), true);
    GLT_TRY(glt::checkpoint_save(paths[d], sib.data(), n_sib, session_id, d, g.S_sib, g.H_sib, mm->D, mm->L));
  }
  return GLT_OK;
}

extern "C" int glt_model_load_stack(GltModel* m, const char* const* paths, int n, const char* session_id) {
  if (!m || !paths) return glt::fail(GLT_EINVAL, "null argument");
  glt::Model* mm = reinterpret_cast<glt::Model*>(m);
  if (!mm->gw) return glt::fail(GLT_ESTATE, "graft storage was freed by the shadow bake");
  if (mm->shadow_baked) return glt::fail(GLT_ESTATE, "the model is shadow-baked");
  StackGeom g;
  GLT_TRY(stack_geom(mm, n, &g));
  const int64_t n_sib = 3LL * mm->L * g.S_sib * g.H_sib;
  std::vector<float> all(static_cast<size_t>(mm->graft_numel), 0.f), sib(static_cast<size_t>(n_sib));
  for (int d = 0; d < n; ++d) {
    if (!paths[d]) return glt::fail(GLT_EINVAL, "null path for sibling %d", d);
    // every file is read and checked before the model's graft changes
    GLT_TRY(glt::checkpoint_load(paths[d], sib.data(), n_sib, d, session_id, 3 * mm->L, g.S_sib, g.H_sib,
                                 nullptr));
    stack_copy(g, mm->L, mm->S, mm->H, d, all.data(), sib.data(), false);
  }
  GLT_CUDA_TRY(cudaDeviceSynchronize());
  GLT_TRY(copy_weights(mm->gw, all.data(), mm->graft_numel * 4, 0, 1));
  GLT_TRY(mm->refresh_graft(nullptr));
  GLT_CUDA_TRY(cudaDeviceSynchronize());
  return GLT_OK;
}

// ---------------------------- .bin + batch walk ----------------------------
extern "C" int glt_load_bin(const char* path, int32_t* num_sequences, int32_t* seq_len,
                            int32_t* tokens, int64_t capacity) {
  if (!path || !num_sequences || !seq_len) return glt::fail(GLT_EINVAL, "null argument");
  FILE* f = fopen(path, "rb");
  if (!f) return glt::fail(GLT_EIO, "cannot open %s", path);
  int32_t hdr[2];
  if (fread(hdr, 4, 2, f) != 2) {
    fclose(f);
    return glt::fail(GLT_EIO, "failed reading header from %s", path);
  }
  // trust-boundary checks of load_bin (src/data_impl.inc:22-47)
  if (hdr[0] <= 0 || hdr[1] <= 0) {
    fclose(f);
    return glt::fail(GLT_EIO, "invalid header in %s (num_sequences=%d, seq_len=%d)", path, hdr[0], hdr[1]);
  }
  const int64_t total = static_cast<int64_t>(hdr[0]) * hdr[1];
  if (total > (1LL << 30)) {
    fclose(f);
    return glt::fail(GLT_EIO, "token count %lld in %s exceeds safety limit", (long long)total, path);
  }
  fseek(f, 0, SEEK_END);
  const long end = ftell(f);
  if (end - 8 < total * 4) {
    fclose(f);
    return glt::fail(GLT_EIO, "truncated token data in %s", path);
  }
  *num_sequences = hdr[0];
  *seq_len = hdr[1];
  if (tokens) {
    if (capacity < total) {
      fclose(f);
      return glt::fail(GLT_EINVAL, "token buffer holds %lld, file has %lld", (long long)capacity, (long long)total);
    }
    fseek(f, 8, SEEK_SET);
    if (fread(tokens, 4, static_cast<size_t>(total), f) != static_cast<size_t>(total)) {
      fclose(f);
      return glt::fail(GLT_EIO, "failed reading token data from %s", path);
    }
  }
  fclose(f);
  return GLT_OK;
}

static uint64_t mix_seed(uint64_t x) {  // grafting.hip:928-933
  x += 0x9e3779b97f4a7c15ULL;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ULL;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebULL;
  return x ^ (x >> 31);
}

extern "C" int glt_batch_walk_start(uint64_t seed, int n_domain, int n_ood, int* domain_pos,
                                    int* ood_pos) {
  if (n_domain <= 0 || n_ood <= 0 || !domain_pos || !ood_pos)
    return glt::fail(GLT_EINVAL, "bad arguments");
  *domain_pos = static_cast<int>(mix_seed(seed) % static_cast<uint64_t>(n_domain));
  *ood_pos = static_cast<int>(mix_seed(seed ^ 0x9e3779b97f4a7c15ULL) % static_cast<uint64_t>(n_ood));
  return GLT_OK;
}

extern "C" int glt_batch_step(const int32_t* domain_tokens, int n_domain, const int32_t* ood_tokens,
                              int n_ood, int seq_len, int batch_size, int* domain_pos, int* ood_pos,
                              int32_t* ids_out, int32_t* ood_mask_out) {
  if (!domain_tokens || !ood_tokens || !domain_pos || !ood_pos || !ids_out || !ood_mask_out)
    return glt::fail(GLT_EINVAL, "null argument");
  if (batch_size % 2 != 0) return glt::fail(GLT_EINVAL, "--batch-size must be even");
  if (n_domain <= 0 || n_ood <= 0 || seq_len <= 0) return glt::fail(GLT_EINVAL, "empty corpus");
  const int half = batch_size / 2;
  const size_t T = static_cast<size_t>(seq_len);
  for (int i = 0; i < half; ++i) {  // grafting.hip:965-973
    const int ds = (*domain_pos + i) % n_domain;
    memcpy(ids_out + i * T, domain_tokens + ds * T, T * 4);
    memset(ood_mask_out + i * T, 0, T * 4);
  }
  *domain_pos = (*domain_pos + half) % n_domain;
  for (int i = 0; i < half; ++i) {  // grafting.hip:975-983
    const int os = (*ood_pos + i) % n_ood;
    memcpy(ids_out + (half + i) * T, ood_tokens + os * T, T * 4);
    for (size_t k = 0; k < T; ++k) ood_mask_out[(half + i) * T + k] = 1;
  }
  *ood_pos = (*ood_pos + half) % n_ood;
  return GLT_OK;
}
