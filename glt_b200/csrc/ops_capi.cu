// C ABI of the layer-level kernels (attention, RoPE, RMSNorm) for callers that
// drive their own layer loop, and for unit tests of each kernel.
#include <math.h>

#include <mutex>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "kernels_mem.cuh"

namespace glt {
int flash_fwd_tc(const uint16_t* qkv, uint16_t* o, float* lse, const AttnShape& s, cudaStream_t st);

namespace {
// RoPE cos/sin tables cached per (device, T, hd, theta), at most kRopeCache
// entries per process: the oldest is freed when a new one is needed
// (cudaFree waits for the device, so no kernel still reads it).
constexpr size_t kRopeCache = 8;
struct RopeEntry {
  int dev, T, hd;
  float theta;
  float* c;
  float* s;
};
std::mutex g_rope_mu;
std::vector<RopeEntry> g_rope;   // oldest first

int rope_tables(int T, int hd, float theta, float** c, float** s) {
  int dev = 0;
  GLT_CUDA_TRY(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(g_rope_mu);
  for (const RopeEntry& e : g_rope)
    if (e.dev == dev && e.T == T && e.hd == hd && e.theta == theta) {
      *c = e.c;
      *s = e.s;
      return GLT_OK;
    }
  if (g_rope.size() >= kRopeCache) {
    const RopeEntry& old = g_rope.front();
    int cur = dev;
    GLT_CUDA_TRY(cudaSetDevice(old.dev));
    cudaFree(old.c);
    cudaFree(old.s);
    GLT_CUDA_TRY(cudaSetDevice(cur));
    g_rope.erase(g_rope.begin());
  }
  const int half = hd / 2;
  std::vector<float> hc(static_cast<size_t>(T) * half), hs(hc.size());
  for (int i = 0; i < half; ++i) {
    const float inv = 1.0f / powf(theta, static_cast<float>(2 * i) / static_cast<float>(hd));
    for (int p = 0; p < T; ++p) {
      hc[static_cast<size_t>(p) * half + i] = cosf(static_cast<float>(p) * inv);
      hs[static_cast<size_t>(p) * half + i] = sinf(static_cast<float>(p) * inv);
    }
  }
  float *dc = nullptr, *ds = nullptr;
  GLT_CUDA_TRY(cudaMalloc(&dc, hc.size() * 4));
  if (cudaMalloc(&ds, hs.size() * 4) != cudaSuccess) {
    cudaFree(dc);
    return fail(GLT_ENOMEM, "glt_rope: table allocation failed");
  }
  GLT_CUDA_TRY(cudaMemcpy(dc, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice));
  GLT_CUDA_TRY(cudaMemcpy(ds, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice));
  g_rope.push_back(RopeEntry{dev, T, hd, theta, dc, ds});
  *c = dc;
  *s = ds;
  return GLT_OK;
}
}  // namespace
}  // namespace glt

using glt::AttnShape;

static AttnShape make_shape(int B, int T, int nh, int nkv, int hd, int64_t ld_qkv, int64_t ld_o) {
  return AttnShape{B, T, nh, nkv, hd, ld_qkv, ld_o, 1.0f / sqrtf(static_cast<float>(hd))};
}

extern "C" int glt_attention_fwd(const uint16_t* qkv, int64_t ld_qkv, uint16_t* o, int64_t ld_o,
                                 float* lse, int B, int T, int nh, int nkv, int hd, int impl,
                                 void* stream) {
  if (!qkv || !o || !lse) return glt::fail(GLT_EINVAL, "null argument");
  const AttnShape s = make_shape(B, T, nh, nkv, hd, ld_qkv, ld_o);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (impl == GLT_ATTN_TCGEN05) return glt::flash_fwd_tc(qkv, o, lse, s, st);
  if (impl == GLT_ATTN_MMA_SYNC) return glt::flash_fwd(qkv, o, lse, s, st);
  return glt::fail(GLT_EINVAL, "unknown attention implementation %d", impl);
}

extern "C" int glt_attention_bwd(const uint16_t* qkv, int64_t ld_qkv, const uint16_t* o,
                                 const uint16_t* dout, int64_t ld_o, const float* lse,
                                 uint16_t* dqkv, float* dq_acc, float* dsum, int B, int T, int nh,
                                 int nkv, int hd, int impl, void* stream) {
  if (!qkv || !o || !dout || !lse || !dqkv || !dq_acc || !dsum)
    return glt::fail(GLT_EINVAL, "null argument");
  const AttnShape s = make_shape(B, T, nh, nkv, hd, ld_qkv, ld_o);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (impl == GLT_ATTN_TCGEN05) {
    if (hd == 64) return glt::flash_bwd_tc64(qkv, o, dout, lse, dqkv, dq_acc, dsum, s, st);
    return glt::flash_bwd_tc(qkv, o, dout, lse, dqkv, dq_acc, dsum, s, st);
  }
  if (impl == GLT_ATTN_MMA_SYNC) return glt::flash_bwd(qkv, o, dout, lse, dqkv, dq_acc, dsum, s, st);
  return glt::fail(GLT_EINVAL, "unknown attention implementation %d", impl);
}

extern "C" int glt_rope(uint16_t* qkv, int64_t ld_qkv, int B, int T, int nh, int nkv, int hd,
                        float theta, int inverse, void* stream) {
  if (!qkv) return glt::fail(GLT_EINVAL, "null argument");
  float *c = nullptr, *s = nullptr;
  GLT_TRY(glt::rope_tables(T, hd, theta, &c, &s));
  const AttnShape sh = make_shape(B, T, nh, nkv, hd, ld_qkv, nh * hd);
  return glt::rope_apply(qkv, sh, c, s, inverse, 1, 1, static_cast<cudaStream_t>(stream));
}

extern "C" int glt_rmsnorm_fwd(const uint16_t* x, const uint16_t* w, uint16_t* y, float* var,
                               int M, int D, float eps, void* stream) {
  if (!x || !w || !y || !var) return glt::fail(GLT_EINVAL, "null argument");
  return glt::rmsnorm_fwd(x, w, y, var, M, D, eps, static_cast<cudaStream_t>(stream));
}

extern "C" int glt_rmsnorm_bwd(const float* dy, const uint16_t* x, const uint16_t* w,
                               const float* var, const float* resid, float* dx, int M, int D,
                               float eps, void* stream) {
  if (!dy || !x || !w || !var || !dx) return glt::fail(GLT_EINVAL, "null argument");
  return glt::rmsnorm_bwd(dy, x, w, var, resid, dx, nullptr, M, D, eps,
                          static_cast<cudaStream_t>(stream));
}
