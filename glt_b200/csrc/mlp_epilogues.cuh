// Epilogues that fuse the grafted SwiGLU MLP's elementwise work into the
// tcgen05 GEMMs over the concatenated [base | graft] intermediate dimension.
//
// Intermediate layout.  F' = F_pad + S_pad intermediate columns: base columns
// [0, F), zero padding to F_pad (a multiple of 256), graft columns
// [F_pad, F_pad + S), zero padding to F'.  The fused gate/up weight W_gu is
// [2F', D] with 128-row blocks interleaved: rows [256b, 256b+128) are gate
// rows of intermediate columns [128b, 128b+128) and rows [256b+128, 256b+256)
// the matching up rows.  One 256-wide N tile of x.W_gu^T therefore holds
// gate and up of the same 128 intermediate columns, so SwiGLU (and its
// backward) complete inside one tile's epilogue.
#pragma once

#include "gemm.cuh"
#include "kernels_mem.cuh"

namespace glt {

__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

// Forward: h[t, c] = bf16(silu(gate) * up) for the 128 columns of the tile;
// for graft columns also accumulate sum(gate^2) and sum(up^2) per token
// (the delta energies of fused_inject_clone_energy_kernel,
// src/kernels_elementwise_impl.inc:287-367, where in concat geometry the
// graft columns of gate_pre/up ARE the expand deltas).
struct EpiSwiGLUFwd {
  uint16_t* h;
  int64_t ldh;
  int M;
  int g0, g1;          // graft intermediate columns [g0, g1)
  float* esq_gate;     // [M] or null
  float* esq_up;       // [M] or null
  __device__ __forceinline__ void operator()(const tc::EpiCtx<256>& c) const {
    const int cb = c.n0 >> 1;
    const bool graft = (cb + 128 > g0) && (cb < g1);
    float eg = 0.f, eu = 0.f;
#pragma unroll 1
    for (int j = 0; j < 128; j += 32) {
      float g[32], u[32];
      c.load(j, g);
      c.load(128 + j, u);
      if (c.row < M) {
        uint16_t* dst = h + static_cast<int64_t>(c.row) * ldh + cb + j;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          float o[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] = g[i + k] * sigmoidf_(g[i + k]) * u[i + k];
          uint4 w;
          w.x = pack_bf16x2(o[0], o[1]); w.y = pack_bf16x2(o[2], o[3]);
          w.z = pack_bf16x2(o[4], o[5]); w.w = pack_bf16x2(o[6], o[7]);
          *reinterpret_cast<uint4*>(dst + i) = w;
        }
        if (graft) {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int col = cb + j + i;
            if (col >= g0 && col < g1) {
              eg += g[i] * g[i];
              eu += u[i] * u[i];
            }
          }
        }
      }
    }
    if (graft && c.row < M) {
      if (esq_gate) atomicAdd(esq_gate + c.row, eg);
      if (esq_up) atomicAdd(esq_up + c.row, eu);
    }
  }
};

// Backward, fused into the recompute of x.W_gu^T (layer_recompute_impl.inc:8-91):
//   dgp = dh * up * s(gp) * (1 + gp * (1 - s(gp)));  dup = dh * gp * s(gp)
// (fused_gate_up_bwd_kernel, src/kernels_elementwise_impl.inc:80-124), written
// bf16 into dgu with W_gu's interleaving.  On graft columns the OOD silence
// gradient is added (fused_silence_blend_energy_kernel, :458-560):
//   scale = lambda_eff / (norm * sqrt(S) + 1e-8),  norm = sqrt(sum(delta^2) + 1e-8)
// and h = silu(gp) * up is written to hg for the down weight gradient.
struct EpiSwiGLUBwd {
  const uint16_t* dh;
  int64_t lddh;
  uint16_t* dgu;
  int64_t ldgu;
  uint16_t* hg;        // [M, ldhg] graft h (bf16) or null
  int64_t ldhg;
  int M;
  int g0, g1;
  int S;
  const float* esq_gate;  // null when gate is not grafted in this layer
  const float* esq_up;
  const int32_t* ood;
  const DevStats* stats;
  __device__ __forceinline__ void operator()(const tc::EpiCtx<256>& c) const {
    const int cb = c.n0 >> 1;
    const bool graft = (cb + 128 > g0) && (cb < g1);
    float sg_s = 0.f, su_s = 0.f;
    if (graft && c.row < M && ood[c.row]) {
      const float lam = stats->lambda_eff;
      const float rs = sqrtf(static_cast<float>(S));
      if (esq_gate) sg_s = lam / (sqrtf(esq_gate[c.row] + 1e-8f) * rs + 1e-8f);
      if (esq_up) su_s = lam / (sqrtf(esq_up[c.row] + 1e-8f) * rs + 1e-8f);
    }
#pragma unroll 1
    for (int j = 0; j < 128; j += 32) {
      float g[32], u[32];
      c.load(j, g);
      c.load(128 + j, u);
      if (c.row >= M) continue;
      const uint16_t* dhr = dh + static_cast<int64_t>(c.row) * lddh + cb + j;
      uint16_t* dgr = dgu + static_cast<int64_t>(c.row) * ldgu + c.n0 + j;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        const uint4 dv = *reinterpret_cast<const uint4*>(dhr + i);
        const float d[8] = {bf16_lo(dv.x), bf16_hi(dv.x), bf16_lo(dv.y), bf16_hi(dv.y),
                            bf16_lo(dv.z), bf16_hi(dv.z), bf16_lo(dv.w), bf16_hi(dv.w)};
        float og[8], ou[8], hh[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float gp = g[i + k], up = u[i + k];
          const float sg = sigmoidf_(gp);
          og[k] = d[k] * up * sg * (1.f + gp * (1.f - sg));
          ou[k] = d[k] * gp * sg;
          hh[k] = gp * sg * up;
        }
        if (graft) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int col = cb + j + i + k;
            if (col >= g0 && col < g1) {
              og[k] += sg_s * g[i + k];
              ou[k] += su_s * u[i + k];
              if (hg) hg[static_cast<int64_t>(c.row) * ldhg + (col - g0)] = f32_to_bf16_bits(hh[k]);
            }
          }
        }
        uint4 a, b;
        a.x = pack_bf16x2(og[0], og[1]); a.y = pack_bf16x2(og[2], og[3]);
        a.z = pack_bf16x2(og[4], og[5]); a.w = pack_bf16x2(og[6], og[7]);
        b.x = pack_bf16x2(ou[0], ou[1]); b.y = pack_bf16x2(ou[2], ou[3]);
        b.z = pack_bf16x2(ou[4], ou[5]); b.w = pack_bf16x2(ou[6], ou[7]);
        *reinterpret_cast<uint4*>(dgr + i) = a;
        *reinterpret_cast<uint4*>(dgr + 128 + i) = b;
      }
    }
  }
};

// delta_down = h_graft . Delta_down: stored bf16 and its per-token sum of
// squares accumulated (ContractForward + energy, layer_forward_impl.inc:185-218).
template <int BN>
struct EpiDeltaDown {
  uint16_t* dd;
  int64_t ld;
  float* esq;
  int M, N;
  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
    float ss = 0.f;
#pragma unroll 1
    for (int j = 0; j < BN; j += 32) {
      float v[32];
      c.load(j, v);
      if (c.row >= M || c.n0 + j >= N) continue;
      uint16_t* dst = dd + static_cast<int64_t>(c.row) * ld + c.n0 + j;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        uint4 w;
        w.x = pack_bf16x2(v[i], v[i + 1]); w.y = pack_bf16x2(v[i + 2], v[i + 3]);
        w.z = pack_bf16x2(v[i + 4], v[i + 5]); w.w = pack_bf16x2(v[i + 6], v[i + 7]);
        *reinterpret_cast<uint4*>(dst + i) = w;
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) ss += v[i] * v[i];
    }
    if (c.row < M) atomicAdd(esq + c.row, ss);
  }
};

// Weight gradient of the fused gate/up graft rows: GEMM row r indexes the
// interleaved graft region of dgu; it is routed to gate or up storage
// [S, D] (ExpandWeightGrad, src/graft_ops_impl.inc:120-156), accumulated
// atomically so split-K partial sums combine.
template <int BN>
struct EpiGradGateUp {
  float* g_gate;  // [S, ld] or null (projection not grafted)
  float* g_up;
  int64_t ld;
  int S, N;
  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
    const int r = c.row;
    const int w = r & 255;
    const int s = (r >> 8) * 128 + (w & 127);
    float* base = (w < 128) ? g_gate : g_up;
    const bool ok = base != nullptr && s < S;
#pragma unroll 1
    for (int j = 0; j < BN; j += 32) {
      float v[32];
      c.load(j, v);
      if (!ok) continue;
      float* dst = base + static_cast<int64_t>(s) * ld + c.n0 + j;
#pragma unroll
      for (int i = 0; i < 32; ++i)
        if (c.n0 + j + i < N) red_add_f32(dst + i, v[i]);
    }
  }
};

}  // namespace glt
