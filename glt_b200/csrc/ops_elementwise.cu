// Stand-alone bandwidth-bound ops of the grafted MLP, for callers that run
// their own layer loop (in the fused training step these live in GEMM
// epilogues and in the model's AdamW):
//   glt_swiglu_fwd  h = bf16(silu(gate_pre) * up), strided rows
//                   (fused_silu_product_strided_kernel,
//                    kernels_elementwise_impl.inc:411-448)
//   glt_swiglu_bwd  grad_gate_pre = gi * up * silu'(gp), grad_up = gi * silu(gp)
//                   (fused_gate_up_bwd_kernel, kernels_elementwise_impl.inc:80-124)
//   glt_stack_grafts  N sibling grafts -> one block-diagonal overlay graft
//                   (the explicit-injection stack of
//                    tests/test6_stack_vs_bake_f32.cpp, as one graft)
//   glt_grad_clip   global-norm clip of a gradient buffer (reduce_l2 /
//                   calc_scale / apply_scale, kernels_elementwise_impl.inc:125-213)
//   glt_adamw_all   AdamW over every projection of the flat [3L, S, H] graft,
//                   skipping disabled projection kinds, optional bf16 image at
//                   the same flat index (adamw_fused_kernel + execute_adamw_all,
//                   kernels_optimizer_impl.inc:11-77)
// Every kernel moves 16 bytes per load/store (8 bf16 or 4 fp32 per vector) in
// a grid-stride loop over a grid sized to the SM count.
#include <math.h>

#include "common.cuh"
#include "gemm.cuh"
#include "kernels_mem.cuh"

namespace glt {
namespace {

__device__ __forceinline__ float silu_ref(float g) { return g * (1.0f / (1.0f + expf(-g))); }

__global__ void swiglu_fwd_kernel(const uint16_t* __restrict__ gate_pre,
                                  const uint16_t* __restrict__ up, uint16_t* __restrict__ out,
                                  int64_t rows, int width, int64_t gate_ld, int64_t up_ld,
                                  int64_t out_ld) {
  // rows in a grid-stride loop over blockIdx.y, 16-byte vectors of a row over x
  const int vpr = width >> 3;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < vpr; v += gridDim.x * blockDim.x) {
      const int c = v << 3;
      float g[8], u[8], h[8];
      unpack8(*reinterpret_cast<const uint4*>(gate_pre + r * gate_ld + c), g);
      unpack8(*reinterpret_cast<const uint4*>(up + r * up_ld + c), u);
#pragma unroll
      for (int k = 0; k < 8; ++k) h[k] = silu_ref(g[k]) * u[k];
      *reinterpret_cast<uint4*>(out + r * out_ld + c) = pack8(h);
    }
  }
}

__global__ void swiglu_bwd_kernel(float* __restrict__ grad_gate_pre, float* __restrict__ grad_up,
                                  const float* __restrict__ grad_h, const uint16_t* __restrict__ up,
                                  const uint16_t* __restrict__ gate_pre, int64_t n) {
  const int64_t nvec = n >> 3;
  for (int64_t v = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; v < nvec;
       v += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = v << 3;
    float g[8], u[8];
    unpack8(*reinterpret_cast<const uint4*>(gate_pre + i), g);
    unpack8(*reinterpret_cast<const uint4*>(up + i), u);
    const float4 a = *reinterpret_cast<const float4*>(grad_h + i);
    const float4 b = *reinterpret_cast<const float4*>(grad_h + i + 4);
    const float gi[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float dg[8], du[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float sg = 1.0f / (1.0f + expf(-g[k]));
      dg[k] = gi[k] * u[k] * (sg * (1.0f + g[k] * (1.0f - sg)));
      du[k] = gi[k] * (g[k] * sg);
    }
    *reinterpret_cast<float4*>(grad_gate_pre + i) = make_float4(dg[0], dg[1], dg[2], dg[3]);
    *reinterpret_cast<float4*>(grad_gate_pre + i + 4) = make_float4(dg[4], dg[5], dg[6], dg[7]);
    *reinterpret_cast<float4*>(grad_up + i) = make_float4(du[0], du[1], du[2], du[3]);
    *reinterpret_cast<float4*>(grad_up + i + 4) = make_float4(du[4], du[5], du[6], du[7]);
  }
}

struct FlatAdam {
  float lr, b1, b2, c1, c2, eps, wd;
  int en[3];
};

// Four consecutive elements per thread; SH % 4 == 0, so a vector never
// straddles two projections.
__global__ void adamw_flat_kernel(float* __restrict__ w, uint16_t* __restrict__ w_bf16,
                                  const float* __restrict__ grad, float* __restrict__ m,
                                  float* __restrict__ v, const float* __restrict__ grad_scale,
                                  int64_t n, int64_t SH, FlatAdam a) {
  const float gs = grad_scale ? *grad_scale : 1.0f;
  const int64_t nvec = n >> 2;
  for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < nvec;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = q << 2;
    if (!a.en[(i / SH) % 3]) continue;
    const float4 g4 = *reinterpret_cast<const float4*>(grad + i);
    const float gp[4] = {g4.x, g4.y, g4.z, g4.w};
    float4 m4 = *reinterpret_cast<const float4*>(m + i);
    float4 v4 = *reinterpret_cast<const float4*>(v + i);
    float4 w4 = *reinterpret_cast<const float4*>(w + i);
    float* mp = reinterpret_cast<float*>(&m4);
    float* vp = reinterpret_cast<float*>(&v4);
    float* wp = reinterpret_cast<float*>(&w4);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float g = gp[k] * gs;
      mp[k] = a.b1 * mp[k] + (1.0f - a.b1) * g;
      vp[k] = a.b2 * vp[k] + (1.0f - a.b2) * g * g;
      const float denom = sqrtf(vp[k] * a.c2) + a.eps;
      wp[k] = wp[k] - a.lr * (mp[k] * a.c1) / denom - a.lr * a.wd * wp[k];
    }
    *reinterpret_cast<float4*>(m + i) = m4;
    *reinterpret_cast<float4*>(v + i) = v4;
    *reinterpret_cast<float4*>(w + i) = w4;
    if (w_bf16) {
      uint2 b;
      b.x = static_cast<uint32_t>(f32_to_bf16_bits(wp[0])) |
            (static_cast<uint32_t>(f32_to_bf16_bits(wp[1])) << 16);
      b.y = static_cast<uint32_t>(f32_to_bf16_bits(wp[2])) |
            (static_cast<uint32_t>(f32_to_bf16_bits(wp[3])) << 16);
      *reinterpret_cast<uint2*>(w_bf16 + i) = b;
    }
  }
}

// Global-norm gradient clip, three passes like the reference
// (reduce_l2_kernel / calc_scale_kernel / apply_scale_kernel): per-CTA
// partial sums of squares (fp64), one CTA turning them into
// norm = sqrt(sum + 1e-8) and scale = clip / norm if norm > clip else 1,
// and an optional in-place rescale of the gradients.
constexpr int CLIP_THREADS = 256;
constexpr int CLIP_MAX_BLOCKS = 1024;
__global__ void __launch_bounds__(CLIP_THREADS) clip_partial_kernel(const float* __restrict__ g,
                                                                    int64_t n, double* __restrict__ partial) {
  __shared__ double red[CLIP_THREADS / 32];
  double acc = 0.0;
  const int64_t nv = n >> 2;
  for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < nv;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(g)[q];
    acc += static_cast<double>(v.x) * v.x + static_cast<double>(v.y) * v.y +
           static_cast<double>(v.z) * v.z + static_cast<double>(v.w) * v.w;
  }
  if (blockIdx.x == 0)   // scalar tail
    for (int64_t i = (nv << 2) + threadIdx.x; i < n; i += blockDim.x) acc += static_cast<double>(g[i]) * g[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < CLIP_THREADS / 32; ++w) t += red[w];
    partial[blockIdx.x] = t;
  }
}

__global__ void __launch_bounds__(CLIP_MAX_BLOCKS) clip_scale_kernel(const double* __restrict__ partial, int np,
                                                                     float clip, float* __restrict__ scale,
                                                                     float* __restrict__ norm_out) {
  __shared__ double red[CLIP_MAX_BLOCKS / 32];
  double acc = threadIdx.x < np ? partial[threadIdx.x] : 0.0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < CLIP_MAX_BLOCKS / 32; ++w) t += red[w];
    const float norm = sqrtf(static_cast<float>(t) + 1e-8f);
    *scale = norm > clip ? clip / norm : 1.0f;
    if (norm_out) *norm_out = norm;
  }
}

__global__ void clip_apply_kernel(float* __restrict__ g, int64_t n, const float* __restrict__ scale) {
  const float sc = *scale;
  const int64_t nv = n >> 2;
  for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < nv;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float4 v = reinterpret_cast<float4*>(g)[q];
    v.x *= sc; v.y *= sc; v.z *= sc; v.w *= sc;
    reinterpret_cast<float4*>(g)[q] = v;
  }
  if (blockIdx.x == 0)
    for (int64_t i = (nv << 2) + threadIdx.x; i < n; i += blockDim.x) g[i] *= sc;
}

constexpr int MAX_STACK = 8;
struct StackSrc {
  const float* g[MAX_STACK];
};

// out[p, r, c] of a [3L, n*S, n*H] graft = g_d[p, r - dS, c - dH] when row r
// and column c fall in the same domain d, else 0 (block-diagonal stack).
__global__ void stack_grafts_kernel(StackSrc src, int n, int64_t projs, int S, int H,
                                    float* __restrict__ out) {
  const int64_t W = static_cast<int64_t>(n) * H;          // output row width
  const int64_t nvec = projs * n * S * (W >> 2);          // 4 floats per vector (H % 4 == 0)
  for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < nvec;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = q << 2;
    const int64_t row = e / W;                             // p * n*S + r
    const int c = static_cast<int>(e - row * W);
    const int64_t p = row / (static_cast<int64_t>(n) * S);
    const int r = static_cast<int>(row - p * n * S);
    const int dr = r / S, dc = c / H;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (dr == dc)
      v = *reinterpret_cast<const float4*>(src.g[dr] + (p * S + (r - dr * S)) * static_cast<int64_t>(H) +
                                           (c - dc * H));
    *reinterpret_cast<float4*>(out + e) = v;
  }
}

// Grid for a grid-stride loop over n units: at most 16 CTAs per SM.
inline int ew_grid(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  if (b > cap) b = cap;
  return static_cast<int>(b < 1 ? 1 : b);
}

}  // namespace
}  // namespace glt

extern "C" int glt_swiglu_fwd(const uint16_t* gate_pre, const uint16_t* up, uint16_t* out,
                              int rows, int width, int64_t gate_ld, int64_t up_ld, int64_t out_ld,
                              void* stream) {
  if (!gate_pre || !up || !out) return glt::fail(GLT_EINVAL, "null argument");
  if (rows < 0 || width < 0) return glt::fail(GLT_EINVAL, "negative size");
  if (rows == 0 || width == 0) return GLT_OK;
  if (width % 8 || gate_ld % 8 || up_ld % 8 || out_ld % 8 || gate_ld < width || up_ld < width ||
      out_ld < width)
    return glt::fail(GLT_EINVAL, "swiglu: width and row strides must be multiples of 8 and >= width");
  if (!glt::aligned16(gate_pre) || !glt::aligned16(up) || !glt::aligned16(out))
    return glt::fail(GLT_EINVAL, "swiglu: pointers must be 16-byte aligned");
  const int vpr = width / 8;
  const int bx = (vpr + 255) / 256;
  const int64_t total = glt::ew_grid(static_cast<int64_t>(rows) * vpr, 256);
  int by = static_cast<int>((total + bx - 1) / bx);
  if (by > rows) by = rows;
  if (by > 65535) by = 65535;
  glt::swiglu_fwd_kernel<<<dim3(bx, by < 1 ? 1 : by), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      gate_pre, up, out, rows, width, gate_ld, up_ld, out_ld);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

extern "C" int glt_swiglu_bwd(float* grad_gate_pre, float* grad_up, const float* grad_h,
                              const uint16_t* up, const uint16_t* gate_pre, int64_t n,
                              void* stream) {
  if (!grad_gate_pre || !grad_up || !grad_h || !up || !gate_pre)
    return glt::fail(GLT_EINVAL, "null argument");
  if (n < 0) return glt::fail(GLT_EINVAL, "negative size");
  if (n == 0) return GLT_OK;
  if (n % 8) return glt::fail(GLT_EINVAL, "swiglu backward: n must be a multiple of 8");
  if (!glt::aligned16(grad_gate_pre) || !glt::aligned16(grad_up) || !glt::aligned16(grad_h) ||
      !glt::aligned16(up) || !glt::aligned16(gate_pre))
    return glt::fail(GLT_EINVAL, "swiglu backward: pointers must be 16-byte aligned");
  glt::swiglu_bwd_kernel<<<glt::ew_grid(n / 8, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      grad_gate_pre, grad_up, grad_h, up, gate_pre, n);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

extern "C" int glt_adamw_all(float* weights, uint16_t* weights_bf16, const float* grads,
                             float* adam_m, float* adam_v, const float* grad_scale,
                             const GltModelConfig* cfg, int step, float lr, void* stream) {
  if (!weights || !grads || !adam_m || !adam_v || !cfg) return glt::fail(GLT_EINVAL, "null argument");
  if (step < 0) return glt::fail(GLT_EINVAL, "negative step");
  const int S = cfg->slice_dim;
  const int H = cfg->layout == GLT_LAYOUT_CONCAT ? cfg->hidden_dim
                                                 : cfg->hidden_dim / (cfg->max_domains > 0 ? cfg->max_domains : 1);
  if (S <= 0 || H <= 0 || cfg->num_layers <= 0) return glt::fail(GLT_EINVAL, "adamw: empty graft");
  const int64_t SH = static_cast<int64_t>(S) * H;
  if (SH % 4) return glt::fail(GLT_EINVAL, "adamw: slice_dim * h_slice_dim must be a multiple of 4");
  if (!glt::aligned16(weights) || !glt::aligned16(grads) || !glt::aligned16(adam_m) ||
      !glt::aligned16(adam_v) || (weights_bf16 && (reinterpret_cast<uintptr_t>(weights_bf16) & 7u)))
    return glt::fail(GLT_EINVAL, "adamw: fp32 buffers must be 16-byte aligned, the bf16 image 8-byte");
  const int64_t n = SH * 3 * cfg->num_layers;
  glt::FlatAdam a;
  a.lr = lr;
  a.b1 = cfg->adam_beta1;
  a.b2 = cfg->adam_beta2;
  a.c1 = 1.0f / (1.0f - powf(cfg->adam_beta1, static_cast<float>(step + 1)));
  a.c2 = 1.0f / (1.0f - powf(cfg->adam_beta2, static_cast<float>(step + 1)));
  a.eps = cfg->adam_eps;
  a.wd = cfg->adam_weight_decay;
  a.en[0] = cfg->graft_proj_gate;
  a.en[1] = cfg->graft_proj_up;
  a.en[2] = cfg->graft_proj_down;
  glt::adamw_flat_kernel<<<glt::ew_grid(n / 4, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      weights, weights_bf16, grads, adam_m, adam_v, grad_scale, n, SH, a);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

extern "C" int glt_stack_grafts(const float* const* grafts, int n, int num_layers, int S, int H,
                                float* out, void* stream) {
  if (!grafts || !out) return glt::fail(GLT_EINVAL, "null argument");
  if (n < 1 || n > glt::MAX_STACK)
    return glt::fail(GLT_EINVAL, "stack of %d grafts: between 1 and %d supported", n, glt::MAX_STACK);
  if (num_layers <= 0 || S <= 0 || H <= 0) return glt::fail(GLT_EINVAL, "empty graft");
  if (H % 4) return glt::fail(GLT_EINVAL, "stack: h_slice_dim must be a multiple of 4");
  glt::StackSrc src{};
  for (int d = 0; d < n; ++d) {
    if (!grafts[d]) return glt::fail(GLT_EINVAL, "stack: graft %d is null", d);
    if (!glt::aligned16(grafts[d])) return glt::fail(GLT_EINVAL, "stack: graft %d not 16-byte aligned", d);
    src.g[d] = grafts[d];
  }
  if (!glt::aligned16(out)) return glt::fail(GLT_EINVAL, "stack: output not 16-byte aligned");
  const int64_t projs = 3 * static_cast<int64_t>(num_layers);
  const int64_t nvec = projs * n * S * (static_cast<int64_t>(n) * H / 4);
  glt::stack_grafts_kernel<<<glt::ew_grid(nvec, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      src, n, projs, S, H, out);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

extern "C" int glt_grad_clip(float* grads, int64_t n, float clip_norm, int apply_in_place,
                             void* workspace, int64_t workspace_bytes, float* scale_out,
                             float* norm_out, void* stream) {
  if (!grads || !workspace || !scale_out) return glt::fail(GLT_EINVAL, "null argument");
  if (n < 0) return glt::fail(GLT_EINVAL, "negative size");
  if (workspace_bytes < static_cast<int64_t>(sizeof(double)) * glt::CLIP_MAX_BLOCKS)
    return glt::fail(GLT_EINVAL, "grad_clip: workspace must hold %d bytes", (int)(sizeof(double) * glt::CLIP_MAX_BLOCKS));
  if (!glt::aligned16(grads) || (reinterpret_cast<uintptr_t>(workspace) & 7u))
    return glt::fail(GLT_EINVAL, "grad_clip: grads must be 16-byte aligned, workspace 8-byte");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int blocks = glt::ew_grid(n / 4 + 1, glt::CLIP_THREADS);
  if (blocks > glt::CLIP_MAX_BLOCKS) blocks = glt::CLIP_MAX_BLOCKS;
  double* partial = static_cast<double*>(workspace);
  glt::clip_partial_kernel<<<blocks, glt::CLIP_THREADS, 0, st>>>(grads, n, partial);
  GLT_LAUNCH_CHECK();
  glt::clip_scale_kernel<<<1, glt::CLIP_MAX_BLOCKS, 0, st>>>(partial, blocks, clip_norm, scale_out, norm_out);
  GLT_LAUNCH_CHECK();
  if (apply_in_place) {
    glt::clip_apply_kernel<<<glt::ew_grid(n / 4 + 1, 256), 256, 0, st>>>(grads, n, scale_out);
    GLT_LAUNCH_CHECK();
  }
  return GLT_OK;
}
