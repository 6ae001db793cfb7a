// Bandwidth-bound kernels of the grafted decoder step: 16-byte vector loads,
// one CTA per row for row reductions (warp shuffles + a shared-memory
// cross-warp stage), grid-stride loops sized to the SM count elsewhere.
#include <math.h>

#include "common.cuh"
#include "gemm.cuh"
#include "kernels_mem.cuh"

namespace glt {

namespace {

constexpr int ROW_THREADS = 128;
constexpr int MAXV = 8;  // 16-byte vectors per thread held in registers (D <= 8192)

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = (l < nw) ? red[l] : 0.f;
  t = warp_sum(t);
  return t;
}

// ------------------------------- RMSNorm -----------------------------------
__global__ void __launch_bounds__(ROW_THREADS) rmsnorm_fwd_kernel(
    const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, uint16_t* __restrict__ y,
    float* __restrict__ var, int D, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nv = D >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * D);
  uint4 xv[MAXV];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = threadIdx.x + k * ROW_THREADS;
    if (i < nv) {
      xv[k] = xr[i];
      float f[8];
      unpack8(xv[k], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
    }
  }
  const float tot = block_sum(ss, red);
  const float v = tot / static_cast<float>(D);
  const float r = rsqrtf(v + eps);
  if (threadIdx.x == 0) var[row] = v;
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  uint4* yr = reinterpret_cast<uint4*>(y + row * D);
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = threadIdx.x + k * ROW_THREADS;
    if (i < nv) {
      float f[8], g[8];
      unpack8(xv[k], f);
      unpack8(wr[i], g);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] = f[j] * r * g[j];
      yr[i] = pack8(f);
    }
  }
}

__global__ void __launch_bounds__(ROW_THREADS) rmsnorm_bwd_kernel(
    const float* __restrict__ dy, const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
    const float* __restrict__ var, const float* resid, float* out, uint16_t* __restrict__ out_bf16,
    int D, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const int nv = D >> 3;
  const float r = rsqrtf(var[row] + eps);
  const float r3 = r * r * r;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * D);
  const uint4* wr = reinterpret_cast<const uint4*>(w);
  const float4* dyr = reinterpret_cast<const float4*>(dy + row * D);
  float acc = 0.f;
  for (int i = threadIdx.x; i < nv; i += ROW_THREADS) {
    float f[8], g[8];
    unpack8(xr[i], f);
    unpack8(wr[i], g);
    const float4 a = dyr[2 * i], b = dyr[2 * i + 1];
    acc += a.x * f[0] * g[0] + a.y * f[1] * g[1] + a.z * f[2] * g[2] + a.w * f[3] * g[3] +
           b.x * f[4] * g[4] + b.y * f[5] * g[5] + b.z * f[6] * g[6] + b.w * f[7] * g[7];
  }
  const float mean = block_sum(acc, red) / static_cast<float>(D);
  for (int i = threadIdx.x; i < nv; i += ROW_THREADS) {
    float f[8], g[8];
    unpack8(xr[i], f);
    unpack8(wr[i], g);
    const float4 a = dyr[2 * i], b = dyr[2 * i + 1];
    const float d[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = d[j] * r * g[j] - f[j] * mean * r3;
    if (resid) {
      const float4 ra = reinterpret_cast<const float4*>(resid + row * D)[2 * i];
      const float4 rb = reinterpret_cast<const float4*>(resid + row * D)[2 * i + 1];
      o[0] += ra.x; o[1] += ra.y; o[2] += ra.z; o[3] += ra.w;
      o[4] += rb.x; o[5] += rb.y; o[6] += rb.z; o[7] += rb.w;
    }
    float4* orow = reinterpret_cast<float4*>(out + row * D);
    orow[2 * i] = make_float4(o[0], o[1], o[2], o[3]);
    orow[2 * i + 1] = make_float4(o[4], o[5], o[6], o[7]);
    if (out_bf16) reinterpret_cast<uint4*>(out_bf16 + row * D)[i] = pack8(o);
  }
}

// ------------------------------- embedding ---------------------------------
__global__ void embedding_kernel(const int32_t* __restrict__ ids, const uint16_t* __restrict__ E,
                                 uint16_t* __restrict__ x, int D, int V, unsigned int* err) {
  const int64_t row = blockIdx.x;
  int id = ids[row];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0 && err) atomicOr(err, GLT_DEVERR_BAD_SHAPE);
    id = 0;
  }
  const uint4* src = reinterpret_cast<const uint4*>(E + static_cast<int64_t>(id) * D);
  uint4* dst = reinterpret_cast<uint4*>(x + row * D);
  for (int i = threadIdx.x; i < (D >> 3); i += blockDim.x) dst[i] = src[i];
}

// ----------------------------- token counts --------------------------------
__global__ void count_tokens_kernel(const int32_t* __restrict__ ood, int B, int T,
                                    DevStats* stats) {
  __shared__ float red[32];
  float dom = 0.f, oc = 0.f;
  const int M = B * T;
  for (int t = threadIdx.x; t < M; t += blockDim.x) {
    const int pos = t % T;
    oc += ood[t] ? 1.f : 0.f;
    if (pos < T - 1) dom += ood[t + 1] ? 0.f : 1.f;
  }
  dom = block_sum(dom, red);
  __syncthreads();
  oc = block_sum(oc, red);
  if (threadIdx.x == 0) {
    stats->in_count = dom < 1.f ? 1.f : dom;
    stats->ood_count = oc;
  }
}

// ----------------------------- cross entropy -------------------------------
constexpr int CE_THREADS = 512;

__global__ void __launch_bounds__(CE_THREADS) cross_entropy_kernel(
    uint16_t* __restrict__ logits, int64_t ld, int row0, int V, const int32_t* __restrict__ ids,
    const int32_t* __restrict__ ood, int T, float scale, DevStats* stats,
    const int* __restrict__ row_map, const int* __restrict__ n_rows) {
  __shared__ float red_m[32], red_s[32];
  __shared__ float s_lab;
  const int r = blockIdx.x;
  // with a row map, logits row r is token row_map[row0 + r] (live by construction)
  if (row_map && row0 + r >= *n_rows) return;
  const int t = row_map ? row_map[row0 + r] : row0 + r;
  const int pos = t % T;
  uint4* row = reinterpret_cast<uint4*>(logits + static_cast<int64_t>(r) * ld);
  const int nv = V >> 3;
  const bool has_label = pos < T - 1;
  const float mask = (has_label && ood[t + 1] == 0) ? 1.f : 0.f;
  if (mask == 0.f) {
    const uint4 z = make_uint4(0, 0, 0, 0);
    for (int i = threadIdx.x; i < nv; i += CE_THREADS) row[i] = z;
    return;
  }
  const int label = ids[t + 1];
  constexpr float LOG2E = 1.4426950408889634f;
  // pass 1: running max / sum of exp
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < nv; i += CE_THREADS) {
    float f[8];
    unpack8(row[i], f);
    float lm = f[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) lm = fmaxf(lm, f[j]);
    if (lm > m) {
      s *= exp2f((m - lm) * LOG2E);
      m = lm;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) s += exp2f((f[j] - m) * LOG2E);
  }
  // combine (m, s) across the block
  {
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = (m == -INFINITY ? 0.f : s * exp2f((m - mm) * LOG2E)) +
          (m2 == -INFINITY ? 0.f : s2 * exp2f((m2 - mm) * LOG2E));
      m = mm;
    }
    if (l == 0) { red_m[w] = m; red_s[w] = s; }
    if (threadIdx.x == 0) s_lab = bf16_bits_to_f32(logits[static_cast<int64_t>(r) * ld + label]);
    __syncthreads();
    const int nw = CE_THREADS / 32;
    m = (l < nw) ? red_m[l] : -INFINITY;
    s = (l < nw) ? red_s[l] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float mm = fmaxf(m, m2);
      s = (m == -INFINITY ? 0.f : s * exp2f((m - mm) * LOG2E)) +
          (m2 == -INFINITY ? 0.f : s2 * exp2f((m2 - mm) * LOG2E));
      m = mm;
    }
  }
  const float lse = m + logf(s);
  if (threadIdx.x == 0) atomicAdd(&stats->ce_sum, static_cast<double>(lse - s_lab));
  const float coef = mask * scale / stats->in_count;
  // pass 2: dlogits in place
  for (int i = threadIdx.x; i < nv; i += CE_THREADS) {
    float f[8];
    unpack8(row[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      float p = exp2f((f[j] - lse) * LOG2E);
      if (i * 8 + j == label) p -= 1.f;
      f[j] = p * coef;
    }
    row[i] = pack8(f);
  }
}

// --------------------------- LM-head rows ---------------------------------
// Token rows whose next-token label counts in the LM loss (position t < T-1
// and ood[t+1] == 0, the mask of cross_entropy_kernel), in order; one CTA,
// chunks of 1024 rows with a ballot + warp-sum scan.
constexpr int LIVE_THREADS = 1024;
__global__ void __launch_bounds__(LIVE_THREADS) live_rows_kernel(const int32_t* __restrict__ ood,
                                                                 int M, int T, int* __restrict__ rows,
                                                                 int* __restrict__ n_rows) {
  __shared__ int warp_off[LIVE_THREADS / 32];
  __shared__ int s_total;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int base = 0;
  for (int c0 = 0; c0 < M; c0 += LIVE_THREADS) {
    const int t = c0 + threadIdx.x;
    const bool live = t < M && (t % T) < T - 1 && ood[t + 1] == 0;
    const unsigned bal = __ballot_sync(0xffffffffu, live);
    if (lane == 0) warp_off[w] = __popc(bal);
    __syncthreads();
    if (w == 0) {
      const int v = warp_off[lane];
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      warp_off[lane] = incl - v;
      if (lane == 31) s_total = incl;
    }
    __syncthreads();
    if (live) rows[base + warp_off[w] + __popc(bal & ((1u << lane) - 1u))] = t;
    base += s_total;
    __syncthreads();
  }
  if (threadIdx.x == 0) *n_rows = base;
}

// dst[i] = src[rows[i]] for i < *n_rows, rows of D bf16 (16-byte vectors).
__global__ void gather_rows_kernel(const uint16_t* __restrict__ src, uint16_t* __restrict__ dst,
                                   const int* __restrict__ rows, const int* __restrict__ n_rows,
                                   int M, int D) {
  const int n = *n_rows;
  const int nv = D >> 3;
  for (int i = blockIdx.x; i < M && i < n; i += gridDim.x) {
    const uint4* s = reinterpret_cast<const uint4*>(src + static_cast<int64_t>(rows[i]) * D);
    uint4* d = reinterpret_cast<uint4*>(dst + static_cast<int64_t>(i) * D);
    for (int v = threadIdx.x; v < nv; v += blockDim.x) d[v] = s[v];
  }
}

// ------------------------------ silence ------------------------------------
__global__ void silence_stats_kernel(const float* __restrict__ esq, const int* __restrict__ en,
                                     int M, int S, int H, const int32_t* __restrict__ ood,
                                     DevStats* stats) {
  __shared__ float red[32];
  const int lp = blockIdx.y;  // layer*3 + proj
  if (!en[lp]) return;
  const int p = lp % 3;
  const float inv = rsqrtf(static_cast<float>(p == 2 ? H : S));
  float d = 0.f, o = 0.f;
  for (int t = blockIdx.x * blockDim.x + threadIdx.x; t < M; t += gridDim.x * blockDim.x) {
    const float e = sqrtf(esq[static_cast<int64_t>(lp) * M + t] + 1e-8f) * inv;
    if (ood[t]) o += e; else d += e;
  }
  d = block_sum(d, red);
  __syncthreads();
  o = block_sum(o, red);
  if (threadIdx.x == 0) {
    atomicAdd(&stats->dom_energy_sum, static_cast<double>(d));
    atomicAdd(&stats->ood_energy_sum, static_cast<double>(o));
  }
}

__global__ void finalize_loss_kernel(DevStats* s, float lambda, int active, float lm_scale) {
  s->lm_loss = static_cast<float>(s->ce_sum / s->in_count);
  s->silence = 0.f;
  s->domain_energy = 0.f;
  s->ood_energy = 0.f;
  s->ratio = 0.f;
  s->lambda_eff = 0.f;
  if (s->ood_count > 0.f && s->in_count > 0.f && active > 0) {
    const float dom = static_cast<float>(s->dom_energy_sum / s->in_count / active);
    const float oe = static_cast<float>(s->ood_energy_sum / s->ood_count / active);
    s->domain_energy = dom;
    s->ood_energy = oe;
    s->ratio = oe > 0.f ? dom / oe : 0.f;
    s->silence = lambda * oe;
    s->lambda_eff = lambda / (s->ood_count * static_cast<float>(active));
  }
  s->total_loss = lm_scale * s->lm_loss + s->silence;
}

__global__ void __launch_bounds__(ROW_THREADS) silence_down_prep_kernel(
    const float* __restrict__ dx, const uint16_t* __restrict__ dd, int64_t ld_dd,
    const float* __restrict__ esq, const int32_t* __restrict__ ood,
    const DevStats* __restrict__ stats, uint16_t* __restrict__ dy, uint16_t* __restrict__ dyg,
    int64_t ld_dyg, int D, int h0, int H) {
  const int64_t row = blockIdx.x;
  float sc = 0.f;
  if (dd && ood[row]) {
    const float norm = sqrtf(esq[row] + 1e-8f);
    sc = stats->lambda_eff / (norm * sqrtf(static_cast<float>(H)));
  }
  const float4* src = reinterpret_cast<const float4*>(dx + row * D);
  for (int i = threadIdx.x; i < (D >> 3); i += ROW_THREADS) {
    const float4 a = src[2 * i], b = src[2 * i + 1];
    float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    reinterpret_cast<uint4*>(dy + row * D)[i] = pack8(f);
    const int j = 8 * i - h0;  // column inside the graft window
    if (j < 0 || j >= H) continue;
    if (dd) {
      float g[8];
      unpack8(*reinterpret_cast<const uint4*>(dd + row * ld_dd + j), g);
#pragma unroll
      for (int k = 0; k < 8; ++k) f[k] += sc * g[k];
    }
    *reinterpret_cast<uint4*>(dyg + row * ld_dyg + j) = pack8(f);
  }
}

// ------------------------------- clip --------------------------------------
__global__ void sumsq_kernel(const float* __restrict__ g, int64_t n, DevStats* stats) {
  __shared__ float red[32];
  float acc = 0.f;
  const int64_t n4 = n >> 2;
  const float4* g4 = reinterpret_cast<const float4*>(g);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float4 v = g4[i];
    acc += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  if (blockIdx.x == 0)
    for (int64_t i = (n4 << 2) + threadIdx.x; i < n; i += blockDim.x) acc += g[i] * g[i];
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) atomicAdd(&stats->grad_sq, static_cast<double>(acc));
}

__global__ void clip_finalize_kernel(DevStats* s, float clip, float gscale) {
  const float norm = sqrtf(static_cast<float>(s->grad_sq) * gscale * gscale + 1e-8f);
  s->grad_norm = norm;
  s->clip_scale = gscale * ((norm > clip) ? clip / norm : 1.f);
}

__global__ void set_scalar_kernel(float* p, float v) { *p = v; }

__global__ void __launch_bounds__(ROW_THREADS) mse_grad_kernel(
    const uint16_t* __restrict__ out, const float* __restrict__ y, float* __restrict__ dx,
    DevStats* stats, int D, float inv_n) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  float acc = 0.f;
  for (int i = threadIdx.x; i < (D >> 3); i += ROW_THREADS) {
    float o[8];
    unpack8(reinterpret_cast<const uint4*>(out + row * D)[i], o);
    const float4 a = reinterpret_cast<const float4*>(y + row * D)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(y + row * D)[2 * i + 1];
    const float t[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    float g[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float d = o[j] - t[j];
      acc += d * d;
      g[j] = 2.f * d * inv_n;
    }
    float4* dr = reinterpret_cast<float4*>(dx + row * D);
    dr[2 * i] = make_float4(g[0], g[1], g[2], g[3]);
    dr[2 * i + 1] = make_float4(g[4], g[5], g[6], g[7]);
  }
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) atomicAdd(&stats->ce_sum, static_cast<double>(acc));
}

// ------------------------------- AdamW -------------------------------------
__device__ __forceinline__ void write_mirror(const MirrorTargets& mt, uint16_t* const* gu,
                                             uint16_t* const* wd, int64_t i, int l, int p, int s,
                                             int h, float w) {
  // Only grafted (layer, kind) pairs carry the delta in the fused weights;
  // the rest stay zero so they contribute nothing (should_graft_proj).
  if (l < mt.layer_begin || l > mt.layer_end || !mt.kinds[p]) return;
  const uint16_t b = f32_to_bf16_bits(w);
  if (mt.plain) {
    mt.plain[i] = b;
    return;
  }
  const int c = mt.f_pad + s;
  if (p < 2) {
    const int64_t row = 256 * (c >> 7) + (c & 127) + (p == 1 ? 128 : 0);
    gu[l][row * mt.D + h] = b;
  } else {
    wd[l][static_cast<int64_t>(h) * mt.ffn + c] = b;
  }
}

struct AdamArgs {
  float lr, b1, b2, c1, c2, eps, wd;
  int en0, en1, en2;
};

__global__ void adamw_kernel(float* __restrict__ w, const float* __restrict__ grad,
                             float* __restrict__ m, float* __restrict__ v, int64_t n, int64_t SH,
                             int H, AdamArgs a, const DevStats* __restrict__ stats,
                             MirrorTargets mt, uint16_t* const* gu, uint16_t* const* wdp) {
  const float cs = stats ? stats->clip_scale : 1.f;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t proj = i / SH;
    const int p = static_cast<int>(proj % 3);
    if ((p == 0 && !a.en0) || (p == 1 && !a.en1) || (p == 2 && !a.en2)) continue;
    const float g = grad[i] * cs;
    float mm = m[i], vv = v[i];
    mm = a.b1 * mm + (1.f - a.b1) * g;
    vv = a.b2 * vv + (1.f - a.b2) * g * g;
    m[i] = mm;
    v[i] = vv;
    const float mh = mm * a.c1, vh = vv * a.c2;
    const float wo = w[i];
    const float nw = wo - a.lr * mh / (sqrtf(vh) + a.eps) - a.lr * a.wd * wo;
    w[i] = nw;
    if (gu || mt.plain) {
      const int64_t r = i - proj * SH;
      write_mirror(mt, gu, wdp, i, static_cast<int>(proj / 3), p, static_cast<int>(r / H),
                   static_cast<int>(r % H), nw);
    }
  }
}

// Vectorized AdamW: four consecutive elements per thread (S*H and H are
// multiples of 4, so a vector stays inside one row of one projection).  The
// bf16 image goes out as one 8-byte store: at the same flat index (overlay),
// or into the interleaved gate/up rows of the concat weights, where h is
// contiguous.  The down projection's image is transposed (h-major rows of
// W_d_cat); with skip_down set it is left to mirror_down_kernel, which stages
// that transpose through shared memory.
__global__ void adamw_vec_kernel(float* __restrict__ w, const float* __restrict__ grad,
                                 float* __restrict__ m, float* __restrict__ v, int64_t n,
                                 int64_t SH, int H, AdamArgs a, const DevStats* __restrict__ stats,
                                 MirrorTargets mt, uint16_t* const* gu, uint16_t* const* wdp,
                                 int skip_down) {
  const float cs = stats ? stats->clip_scale : 1.f;
  const int64_t nvec = n >> 2;
  for (int64_t q = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; q < nvec;
       q += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i = q << 2;
    const int64_t proj = i / SH;
    const int p = static_cast<int>(proj % 3);
    if ((p == 0 && !a.en0) || (p == 1 && !a.en1) || (p == 2 && !a.en2)) continue;
    const float4 g4 = *reinterpret_cast<const float4*>(grad + i);
    const float gv[4] = {g4.x * cs, g4.y * cs, g4.z * cs, g4.w * cs};
    float4 m4 = *reinterpret_cast<const float4*>(m + i);
    float4 v4 = *reinterpret_cast<const float4*>(v + i);
    float4 w4 = *reinterpret_cast<const float4*>(w + i);
    float* mp = reinterpret_cast<float*>(&m4);
    float* vp = reinterpret_cast<float*>(&v4);
    float* wp = reinterpret_cast<float*>(&w4);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      mp[k] = a.b1 * mp[k] + (1.f - a.b1) * gv[k];
      vp[k] = a.b2 * vp[k] + (1.f - a.b2) * gv[k] * gv[k];
      const float mh = mp[k] * a.c1, vh = vp[k] * a.c2;
      wp[k] = wp[k] - a.lr * mh / (sqrtf(vh) + a.eps) - a.lr * a.wd * wp[k];
    }
    *reinterpret_cast<float4*>(m + i) = m4;
    *reinterpret_cast<float4*>(v + i) = v4;
    *reinterpret_cast<float4*>(w + i) = w4;
    if (!gu && !mt.plain) continue;
    const int l = static_cast<int>(proj / 3);
    if (l < mt.layer_begin || l > mt.layer_end || !mt.kinds[p]) continue;
    uint2 b;
    b.x = static_cast<uint32_t>(f32_to_bf16_bits(wp[0])) |
          (static_cast<uint32_t>(f32_to_bf16_bits(wp[1])) << 16);
    b.y = static_cast<uint32_t>(f32_to_bf16_bits(wp[2])) |
          (static_cast<uint32_t>(f32_to_bf16_bits(wp[3])) << 16);
    if (mt.plain) {
      *reinterpret_cast<uint2*>(mt.plain + i) = b;
      continue;
    }
    const int64_t r = i - proj * SH;
    const int s = static_cast<int>(r / H), h = static_cast<int>(r % H);
    if (p < 2) {
      const int c = mt.f_pad + s;
      const int64_t row = 256 * (c >> 7) + (c & 127) + (p == 1 ? 128 : 0);
      *reinterpret_cast<uint2*>(gu[l] + row * mt.D + h) = b;
    } else if (!skip_down) {
#pragma unroll
      for (int k = 0; k < 4; ++k) write_mirror(mt, gu, wdp, i + k, l, 2, s, h + k, wp[k]);
    }
  }
}

// bf16 image of the down projections' graft, [S, H] fp32 -> W_d_cat[h][f_pad + s]
// for every grafted layer.  Tile of 64 s x 32 h per CTA: read 128-byte rows
// along h, transpose in shared memory, write 128-byte rows along s.
constexpr int MD_S = 64, MD_H = 32;
__global__ void __launch_bounds__(256) mirror_down_kernel(const float* __restrict__ w, int S, int H,
                                                          MirrorTargets mt,
                                                          uint16_t* const* __restrict__ wdp) {
  __shared__ float tile[MD_S][MD_H + 1];
  const int l = mt.layer_begin + blockIdx.z;
  const int s0 = blockIdx.y * MD_S, h0 = blockIdx.x * MD_H;
  const int64_t base = (static_cast<int64_t>(l) * 3 + 2) * S * static_cast<int64_t>(H);
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 8 warps
#pragma unroll
  for (int k = 0; k < MD_S / 8; ++k) {
    const int s = s0 + ty + 8 * k, h = h0 + tx;
    tile[ty + 8 * k][tx] = (s < S && h < H) ? w[base + static_cast<int64_t>(s) * H + h] : 0.f;
  }
  __syncthreads();
  uint16_t* dst = wdp[l];
#pragma unroll
  for (int k = 0; k < MD_H / 8; ++k) {
    const int hh = ty + 8 * k, h = h0 + hh;
    const int s = s0 + 2 * tx;
    if (h >= H || s >= S) continue;
    uint16_t* p = dst + static_cast<int64_t>(h) * mt.ffn + mt.f_pad + s;
    const uint16_t lo = f32_to_bf16_bits(tile[2 * tx][hh]);
    if (s + 1 < S) {
      const uint16_t hi = f32_to_bf16_bits(tile[2 * tx + 1][hh]);
      *reinterpret_cast<uint32_t*>(p) = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
    } else {
      *p = lo;
    }
  }
}

__global__ void mirror_kernel(const float* __restrict__ w, int64_t n, int64_t SH, int H,
                              MirrorTargets mt, uint16_t* const* gu, uint16_t* const* wdp,
                              int skip_down) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t proj = i / SH;
    const int64_t r = i - proj * SH;
    if (skip_down && proj % 3 == 2) continue;
    write_mirror(mt, gu, wdp, i, static_cast<int>(proj / 3), static_cast<int>(proj % 3),
                 static_cast<int>(r / H), static_cast<int>(r % H), w[i]);
  }
}

__global__ void shadow_bake_fused_kernel(const float* __restrict__ g, int64_t n, int64_t SH, int H,
                                         int i0, int h0, MirrorTargets mt, uint16_t* const* gu,
                                         uint16_t* const* wdp) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t proj = i / SH;
    const int l = static_cast<int>(proj / 3), p = static_cast<int>(proj % 3);
    if (l < mt.layer_begin || l > mt.layer_end || !mt.kinds[p]) continue;
    const int64_t r = i - proj * SH;
    const int c = i0 + static_cast<int>(r / H);
    const int hh = h0 + static_cast<int>(r % H);
    uint16_t* dst;
    if (p < 2) {
      const int64_t row = 256 * (c >> 7) + (c & 127) + (p == 1 ? 128 : 0);
      dst = gu[l] + row * mt.D + hh;
    } else {
      dst = wdp[l] + static_cast<int64_t>(hh) * mt.ffn + c;
    }
    *dst = f32_to_bf16_bits(bf16_bits_to_f32(*dst) + g[i]);
  }
}

// ------------------------------- bake --------------------------------------
// base += graft, one 64 x 64 (s, h) tile per CTA.  The graft tile is read
// along h and kept in shared memory; the base is then updated along its own
// rows (h for expand, s for contract, where the tile is read transposed) two
// bf16 at a time, so both sides stay coalesced.  Each element is still
// bf16(f32(base) + graft) with round-to-nearest-even, as in the reference.
constexpr int BAKE_T = 64;
__device__ __forceinline__ void bake_pair(uint16_t* base, int64_t idx, bool two, float d0, float d1) {
  if (two && (idx & 1) == 0) {
    uint32_t* p = reinterpret_cast<uint32_t*>(base + idx);
    const uint32_t w = *p;
    const uint16_t lo = f32_to_bf16_bits(bf16_bits_to_f32(static_cast<uint16_t>(w & 0xFFFFu)) + d0);
    const uint16_t hi = f32_to_bf16_bits(bf16_bits_to_f32(static_cast<uint16_t>(w >> 16)) + d1);
    *p = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  } else {
    base[idx] = f32_to_bf16_bits(bf16_bits_to_f32(base[idx]) + d0);
    if (two) base[idx + 1] = f32_to_bf16_bits(bf16_bits_to_f32(base[idx + 1]) + d1);
  }
}

__global__ void __launch_bounds__(256) shadow_bake_kernel(uint16_t* base, int64_t stride,
                                                          const float* __restrict__ g, int S, int H,
                                                          int i0, int h0, int mode) {
  __shared__ float tile[BAKE_T][BAKE_T + 1];   // [s][h]
  const int s0 = blockIdx.y * BAKE_T, hb = blockIdx.x * BAKE_T;
  for (int k = threadIdx.x; k < BAKE_T * BAKE_T; k += blockDim.x) {
    const int ts = k / BAKE_T, th = k % BAKE_T;
    const int s = s0 + ts, h = hb + th;
    tile[ts][th] = (s < S && h < H) ? g[static_cast<int64_t>(s) * H + h] : 0.f;
  }
  __syncthreads();
  for (int k = threadIdx.x; k < BAKE_T * BAKE_T / 2; k += blockDim.x) {
    const int row = k / (BAKE_T / 2), col = 2 * (k % (BAKE_T / 2));
    if (mode == 0) {   // base row i0 + s, columns h0 + h, h0 + h + 1
      const int s = s0 + row, h = hb + col;
      if (s >= S || h >= H) continue;
      bake_pair(base, static_cast<int64_t>(i0 + s) * stride + h0 + h, h + 1 < H, tile[row][col],
                tile[row][col + 1]);
    } else {           // base row h0 + h, columns i0 + s, i0 + s + 1
      const int h = hb + row, s = s0 + col;
      if (h >= H || s >= S) continue;
      bake_pair(base, static_cast<int64_t>(h0 + h) * stride + i0 + s, s + 1 < S, tile[col][row],
                tile[col + 1][row]);
    }
  }
}

// ------------------------------- init --------------------------------------
__device__ __forceinline__ uint64_t splitmix(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
__device__ __forceinline__ float normal_at(uint64_t seed, int64_t i) {
  const uint64_t h = splitmix(seed ^ splitmix(static_cast<uint64_t>(i)));
  const float u1 = (static_cast<float>(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
  const float u2 = static_cast<float>((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
  return sqrtf(-2.f * logf(u1)) * cospif(2.f * u2);
}
__global__ void init_bf16_kernel(uint16_t* p, int64_t n, uint64_t seed, float std) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = f32_to_bf16_bits(std * normal_at(seed, i));
}
__global__ void init_f32_kernel(float* p, int64_t n, uint64_t seed, float std) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = std * normal_at(seed, i);
}
__global__ void fill_bf16_kernel(uint16_t* p, int64_t n, uint16_t v) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    p[i] = v;
}

// ------------------------------- packing -----------------------------------
__global__ void pack_kernel(const void* __restrict__ src, int is_f32, int64_t src_ld, int cols,
                            uint16_t* __restrict__ dst, int64_t ld_dst) {
  const int64_t r = blockIdx.x;
  for (int c = threadIdx.x; c < ld_dst; c += blockDim.x) {
    uint16_t b = 0;
    if (c < cols) {
      b = is_f32 ? f32_to_bf16_bits(static_cast<const float*>(src)[r * src_ld + c])
                 : static_cast<const uint16_t*>(src)[r * src_ld + c];
    }
    dst[r * ld_dst + c] = b;
  }
}
__global__ void cast_kernel(const float* __restrict__ s, uint16_t* __restrict__ d, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    d[i] = f32_to_bf16_bits(s[i]);
}

inline int grid_for(int64_t n, int threads) {
  int64_t b = (n + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  if (b > cap) b = cap;
  return static_cast<int>(b < 1 ? 1 : b);
}

}  // namespace

int rmsnorm_fwd(const uint16_t* x, const uint16_t* w, uint16_t* y, float* var, int M, int D,
                float eps, cudaStream_t st) {
  if (D % 8 || D > ROW_THREADS * 8 * MAXV) return fail(GLT_EINVAL, "rmsnorm: unsupported D=%d", D);
  if (M <= 0) return GLT_OK;
  rmsnorm_fwd_kernel<<<M, ROW_THREADS, 0, st>>>(x, w, y, var, D, eps);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int rmsnorm_bwd(const float* dy, const uint16_t* x, const uint16_t* w, const float* var,
                const float* resid, float* out, uint16_t* out_bf16, int M, int D, float eps,
                cudaStream_t st) {
  if (D % 8) return fail(GLT_EINVAL, "rmsnorm_bwd: D %% 8 != 0");
  if (M <= 0) return GLT_OK;
  rmsnorm_bwd_kernel<<<M, ROW_THREADS, 0, st>>>(dy, x, w, var, resid, out, out_bf16, D, eps);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int embedding_fwd(const int32_t* ids, const uint16_t* E, uint16_t* x, int M, int D, int V,
                  cudaStream_t st) {
  if (D % 8) return fail(GLT_EINVAL, "embedding: D %% 8 != 0");
  if (M <= 0) return GLT_OK;
  embedding_kernel<<<M, 128, 0, st>>>(ids, E, x, D, V, device_error_word());
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int count_tokens(const int32_t* ood, int B, int T, DevStats* stats, cudaStream_t st) {
  count_tokens_kernel<<<1, 1024, 0, st>>>(ood, B, T, stats);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int cross_entropy_chunk(uint16_t* logits, int64_t ld, int rows, int row0, int V,
                        const int32_t* ids, const int32_t* ood, int T, float scale,
                        DevStats* stats, cudaStream_t st, const int* row_map,
                        const int* n_rows) {
  if (V % 8) return fail(GLT_EINVAL, "cross_entropy: V %% 8 != 0");
  if (rows <= 0) return GLT_OK;
  cross_entropy_kernel<<<rows, CE_THREADS, 0, st>>>(logits, ld, row0, V, ids, ood, T, scale,
                                                     stats, row_map, n_rows);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int live_rows(const int32_t* ood, int M, int T, int* rows, int* n_rows, cudaStream_t st) {
  if (M <= 0) return GLT_OK;
  live_rows_kernel<<<1, LIVE_THREADS, 0, st>>>(ood, M, T, rows, n_rows);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int gather_rows(const uint16_t* src, uint16_t* dst, const int* rows, const int* n_rows, int M, int D,
                cudaStream_t st) {
  if (M <= 0) return GLT_OK;
  if (D % 8) return fail(GLT_EINVAL, "gather_rows: D %% 8 != 0");
  gather_rows_kernel<<<grid_for(M, 1), 256, 0, st>>>(src, dst, rows, n_rows, M, D);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int silence_stats(const float* esq, const int* proj_enabled, int L, int M, int S, int H,
                  const int32_t* ood, DevStats* stats, cudaStream_t st) {
  dim3 grid((M + 1023) / 1024 < 64 ? (M + 1023) / 1024 : 64, L * 3);
  silence_stats_kernel<<<grid, 1024, 0, st>>>(esq, proj_enabled, M, S, H, ood, stats);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int finalize_loss(DevStats* stats, float lambda_silence, int active_grafts, float lm_loss_scale,
                  cudaStream_t st) {
  finalize_loss_kernel<<<1, 1, 0, st>>>(stats, lambda_silence, active_grafts, lm_loss_scale);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int silence_down_prep(const float* dx, const uint16_t* delta_down, int64_t ld_dd,
                      const float* esq_down, const int32_t* ood, const DevStats* stats,
                      uint16_t* dy, uint16_t* dyg, int64_t ld_dyg, int M, int D, int h0, int H,
                      cudaStream_t st) {
  if (M <= 0) return GLT_OK;
  if ((h0 | H | ld_dd | ld_dyg) & 7) return fail(GLT_EINVAL, "silence_down_prep: window not 8-aligned");
  silence_down_prep_kernel<<<M, ROW_THREADS, 0, st>>>(dx, delta_down, ld_dd, esq_down, ood, stats,
                                                       dy, dyg, ld_dyg, D, h0, H);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int grad_clip_scale(const float* grad, int64_t n, float clip_norm, float gscale,
                    DevStats* stats, cudaStream_t st) {
  sumsq_kernel<<<grid_for(n / 4 + 1, 512), 512, 0, st>>>(grad, n, stats);
  GLT_LAUNCH_CHECK();
  clip_finalize_kernel<<<1, 1, 0, st>>>(stats, clip_norm, gscale);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

__global__ void collect_error_kernel(unsigned int* word, unsigned int* accum, unsigned int* dst) {
  const unsigned int v = *word | *accum;
  *word = 0u;
  if (dst) {
    *dst = v;
    *accum = 0u;
  } else {
    *accum = v;
  }
}

int collect_device_error(unsigned int* word, unsigned int* accum, unsigned int* dst, cudaStream_t st) {
  if (!word || !accum) return fail(GLT_ECUDA, "device error word unavailable");
  collect_error_kernel<<<1, 1, 0, st>>>(word, accum, dst);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int set_clip_scale(DevStats* stats, float v, cudaStream_t st) {
  set_scalar_kernel<<<1, 1, 0, st>>>(&stats->clip_scale, v);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int set_lambda_eff(DevStats* stats, float v, cudaStream_t st) {
  set_scalar_kernel<<<1, 1, 0, st>>>(&stats->lambda_eff, v);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int mse_grad(const uint16_t* out, const float* y, float* dx, DevStats* stats, int M, int D,
             cudaStream_t st) {
  if (M <= 0) return GLT_OK;
  mse_grad_kernel<<<M, ROW_THREADS, 0, st>>>(out, y, dx, stats, D,
                                             1.0f / (static_cast<float>(M) * D));
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int adamw_step(float* w, const float* grad, float* m, float* v, int L, int S, int H, float lr,
               float beta1, float beta2, float eps, float wd, int step, const int* kinds,
               const DevStats* stats, const MirrorTargets* mirror, cudaStream_t st) {
  AdamArgs a;
  a.lr = lr;
  a.b1 = beta1;
  a.b2 = beta2;
  a.c1 = 1.0f / (1.0f - powf(beta1, static_cast<float>(step + 1)));
  a.c2 = 1.0f / (1.0f - powf(beta2, static_cast<float>(step + 1)));
  a.eps = eps;
  a.wd = wd;
  a.en0 = kinds[0];
  a.en1 = kinds[1];
  a.en2 = kinds[2];
  const int64_t SH = static_cast<int64_t>(S) * H;
  const int64_t n = SH * 3 * L;
  MirrorTargets mt{};
  if (mirror) mt = *mirror;
  uint16_t* const* gu = mirror ? mirror->w_gu : nullptr;
  uint16_t* const* wdp = mirror ? mirror->w_d : nullptr;
  if (SH % 4 != 0 || H % 4 != 0) {   // shapes the vector kernel cannot take
    adamw_kernel<<<grid_for(n, 256), 256, 0, st>>>(w, grad, m, v, n, SH, H, a, stats, mt, gu, wdp);
    GLT_LAUNCH_CHECK();
    return GLT_OK;
  }
  const bool tiled_down = gu != nullptr && !mt.plain && kinds[2] && mt.kinds[2];
  adamw_vec_kernel<<<grid_for(n / 4, 256), 256, 0, st>>>(w, grad, m, v, n, SH, H, a, stats, mt, gu,
                                                          wdp, tiled_down ? 1 : 0);
  GLT_LAUNCH_CHECK();
  if (tiled_down) GLT_TRY(mirror_down(w, L, S, H, mt, st));
  return GLT_OK;
}

int mirror_down(const float* w, int L, int S, int H, const MirrorTargets& mirror, cudaStream_t st) {
  MirrorTargets mt = mirror;   // grafted layers, clamped to the model's
  if (mt.layer_begin < 0) mt.layer_begin = 0;
  if (mt.layer_end > L - 1) mt.layer_end = L - 1;
  const int layers = mt.layer_end - mt.layer_begin + 1;
  if (layers <= 0 || S <= 0 || H <= 0 || !mt.w_d || !mt.kinds[2]) return GLT_OK;
  dim3 grid((H + MD_H - 1) / MD_H, (S + MD_S - 1) / MD_S, layers);
  mirror_down_kernel<<<grid, 256, 0, st>>>(w, S, H, mt, mt.w_d);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int refresh_mirror(const float* w, int L, int S, int H, const MirrorTargets& mirror,
                   cudaStream_t st) {
  const int64_t SH = static_cast<int64_t>(S) * H;
  const int64_t n = SH * 3 * L;
  const bool tiled_down = mirror.w_d != nullptr && !mirror.plain && mirror.kinds[2];
  mirror_kernel<<<grid_for(n, 256), 256, 0, st>>>(w, n, SH, H, mirror, mirror.w_gu, mirror.w_d,
                                                   tiled_down ? 1 : 0);
  GLT_LAUNCH_CHECK();
  if (tiled_down) GLT_TRY(mirror_down(w, L, S, H, mirror, st));
  return GLT_OK;
}

int shadow_bake_fused(const float* g, int L, int S, int H, int i0, int h0,
                      const MirrorTargets& mt, cudaStream_t st) {
  const int64_t SH = static_cast<int64_t>(S) * H;
  const int64_t n = SH * 3 * L;
  if (n <= 0) return GLT_OK;
  shadow_bake_fused_kernel<<<grid_for(n, 256), 256, 0, st>>>(g, n, SH, H, i0, h0, mt, mt.w_gu, mt.w_d);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int shadow_bake(uint16_t* base, int64_t base_stride, const float* g, int S, int H, int i0, int h0,
                int mode, cudaStream_t st) {
  if (S <= 0 || H <= 0) return GLT_OK;
  dim3 grid((H + BAKE_T - 1) / BAKE_T, (S + BAKE_T - 1) / BAKE_T);
  shadow_bake_kernel<<<grid, 256, 0, st>>>(base, base_stride, g, S, H, i0, h0, mode);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int init_normal_bf16(uint16_t* p, int64_t n, uint64_t seed, float std, cudaStream_t st) {
  if (n <= 0) return GLT_OK;
  init_bf16_kernel<<<grid_for(n, 256), 256, 0, st>>>(p, n, seed, std);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}
int init_normal_f32(float* p, int64_t n, uint64_t seed, float std, cudaStream_t st) {
  if (n <= 0) return GLT_OK;
  init_f32_kernel<<<grid_for(n, 256), 256, 0, st>>>(p, n, seed, std);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}
int fill_bf16(uint16_t* p, int64_t n, float v, cudaStream_t st) {
  if (n <= 0) return GLT_OK;
  fill_bf16_kernel<<<grid_for(n, 256), 256, 0, st>>>(p, n, f32_to_bf16_bits(v));
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int pack_bf16(const void* src, int src_is_f32, int64_t src_ld, int rows, int cols, uint16_t* dst,
              int64_t ld_dst, cudaStream_t st) {
  if (rows <= 0) return GLT_OK;
  pack_kernel<<<rows, 128, 0, st>>>(src, src_is_f32, src_ld, cols, dst, ld_dst);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}
int cast_f32_to_bf16(const float* src, uint16_t* dst, int64_t n, cudaStream_t st) {
  if (n <= 0) return GLT_OK;
  cast_kernel<<<grid_for(n, 256), 256, 0, st>>>(src, dst, n);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

}  // namespace glt
