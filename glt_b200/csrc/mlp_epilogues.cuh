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

// Logistic sigmoid for the GEMM epilogues: exp on the special-function unit
// and the fast (reciprocal-based) division; its error (a few ulp of fp32)
// stays far below the bf16 rounding every epilogue output gets.  The
// stand-alone SwiGLU ops (ops_elementwise.cu) keep expf and IEEE division.
__device__ __forceinline__ float sigmoidf_(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// Layout of the stored gate_pre/up (EpiSwiGLUFwd::gu, EpiSwiGLUBwdStored):
// a private buffer, so it is laid out for the epilogues' access pattern, in
// which lane i of a warp owns row 32b + i of a 32-row band: element (r, c) of
// the [M, 2F'] matrix (c in W_gu's interleaved order) sits at
//   ((r / 32) * (2F' / 8) + c / 8) * 256 + (r % 32) * 8 + c % 8.
// A warp's 16-byte accesses to 8 columns of its 32 rows are then one
// contiguous 512-byte run (fully coalesced), where the row-major layout
// touches 32 separate lines.
__device__ __forceinline__ int64_t gu_block_offset(int row, int col8, int64_t groups) {
  return ((static_cast<int64_t>(row >> 5) * groups + col8) << 8) + ((row & 31) << 3);
}

// Row-major stores of a warp's 32 rows x 32 bf16 columns, where lane i holds
// row i's 64 bytes as four uint4 (v[0..3]).  The block goes through `stage`
// (2 KB of shared memory per matrix) and leaves as 8-row x 64-byte runs, so
// each store instruction fills whole 32-byte sectors of 8 lines instead of
// half-sectors of 32 lines.  The stores are evict-first: h and dgu are larger
// than L2 and would otherwise push the GEMM's operand rows out of it.  16-byte slots are XOR-swizzled by row so both
// the row-per-lane writes and the run reads are free of bank conflicts.
// dst(m) = dst_m + r * ld for band rows r < rows (rows past M are skipped).
// stage_put writes this lane's 16-byte piece q of matrix m; stage_flush is
// warp-collective (every lane calls it with the same arguments).
__device__ __forceinline__ void stage_put(uint8_t* stage, int m, int q, uint4 v) {
  const int lane = threadIdx.x & 31;
  *reinterpret_cast<uint4*>(stage + m * 2048 + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4)) = v;
}
template <int NMAT>
__device__ __forceinline__ void stage_flush(const uint8_t* stage, uint16_t* const (&dst)[NMAT], int64_t ld,
                                            int rows) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  const int u = lane & 3;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + (lane >> 2);
#pragma unroll
    for (int m = 0; m < NMAT; ++m) {
      const uint4 w = *reinterpret_cast<const uint4*>(stage + m * 2048 + r * 64 + ((u ^ ((r >> 1) & 3)) << 4));
      if (r < rows) __stcs(reinterpret_cast<uint4*>(dst[m] + r * ld + 8 * u), w);   // streaming
    }
  }
  __syncwarp();
}

// Forward: h[t, c] = bf16(silu(gate) * up) for the 128 columns of the tile;
// for graft columns also accumulate sum(gate^2) and sum(up^2) per token
// (the delta energies of fused_inject_clone_energy_kernel,
// src/kernels_elementwise_impl.inc:287-367, where in concat geometry the
// graft columns of gate_pre/up ARE the expand deltas).  With `gu` set the
// tile's gate_pre and up are also stored bf16, in W_gu's interleaving, for
// the backward (EpiSwiGLUBwdStored) -- the bf16 gate_pre/up tensors that
// the reference's recompute_ffn (src/layer_recompute_impl.inc:8-91) rebuilds.
struct EpiSwiGLUFwd {
  uint16_t* h;
  int64_t ldh;
  int M;
  int g0, g1;          // graft intermediate columns [g0, g1)
  float* esq_gate;     // [M] or null
  float* esq_up;       // [M] or null
  uint16_t* gu = nullptr;  // stored gate_pre/up (gu_block_offset layout) or null
  int64_t gu_groups = 0;   // 2F' / 8
  static constexpr int kParts = 2;   // two epilogue warps per 32 rows, 64 columns each
  static constexpr int kScratchPerWarp = 2048;   // h staging (stage_store_32x32)
  __device__ __forceinline__ void operator()(const tc::EpiCtx<256>& c) const {
    const int cb = c.n0 >> 1;
    const bool graft = (cb + 128 > g0) && (cb < g1);
    float eg = 0.f, eu = 0.f;
    const int j0 = c.part * (128 / kParts);
    const int band0 = c.row & ~31;
#pragma unroll 1
    for (int j = j0; j < j0 + 128 / kParts; j += 32) {
      float g[32], u[32];
      c.load(j, g);
      c.load(128 + j, u);
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        float o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = g[i + k] * sigmoidf_(g[i + k]) * u[i + k];
        stage_put(c.scratch, 0, i / 8, make_uint4(pack_bf16x2_rn(o[0], o[1]), pack_bf16x2_rn(o[2], o[3]),
                                                   pack_bf16x2_rn(o[4], o[5]), pack_bf16x2_rn(o[6], o[7])));
      }
      uint16_t* const hdst[1] = {h + static_cast<int64_t>(band0) * ldh + cb + j};
      stage_flush<1>(c.scratch, hdst, ldh, M - band0);
      if (c.row < M) {
        if (gu) {
          const int g8 = (c.n0 + j) >> 3;   // gate columns; up is 128 columns (16 groups) on
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 a, b;
            a.x = pack_bf16x2_rn(g[i], g[i + 1]); a.y = pack_bf16x2_rn(g[i + 2], g[i + 3]);
            a.z = pack_bf16x2_rn(g[i + 4], g[i + 5]); a.w = pack_bf16x2_rn(g[i + 6], g[i + 7]);
            b.x = pack_bf16x2_rn(u[i], u[i + 1]); b.y = pack_bf16x2_rn(u[i + 2], u[i + 3]);
            b.z = pack_bf16x2_rn(u[i + 4], u[i + 5]); b.w = pack_bf16x2_rn(u[i + 6], u[i + 7]);
            // streaming stores: read once, a whole forward/backward later
            __stcs(reinterpret_cast<uint4*>(gu + gu_block_offset(c.row, g8 + i / 8, gu_groups)), a);
            __stcs(reinterpret_cast<uint4*>(gu + gu_block_offset(c.row, g8 + 16 + i / 8, gu_groups)), b);
          }
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
  static constexpr int kParts = 2;
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
    // dh of 32 columns is fetched one chunk ahead (chunk 0 before the
    // accumulator is read) so its latency overlaps the previous chunk
    const int j0 = c.part * (128 / kParts), j1 = j0 + 128 / kParts;
    const uint4* dhrow = reinterpret_cast<const uint4*>(dh + static_cast<int64_t>(c.row) * lddh + cb);
    uint4 nd[4];
    if (c.row < M) {
#pragma unroll
      for (int q = 0; q < 4; ++q) nd[q] = __ldg(dhrow + j0 / 8 + q);
    }
#pragma unroll 1
    for (int j = j0; j < j1; j += 32) {
      float g[32], u[32];
      c.load(j, g);
      c.load(128 + j, u);
      if (c.row >= M) continue;
      uint4 dcur[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) dcur[q] = nd[q];
      if (j + 32 < j1) {
#pragma unroll
        for (int q = 0; q < 4; ++q) nd[q] = __ldg(dhrow + (j + 32) / 8 + q);
      }
      uint16_t* dgr = dgu + static_cast<int64_t>(c.row) * ldgu + c.n0 + j;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        const uint4 dv = dcur[i / 8];
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
        a.x = pack_bf16x2_rn(og[0], og[1]); a.y = pack_bf16x2_rn(og[2], og[3]);
        a.z = pack_bf16x2_rn(og[4], og[5]); a.w = pack_bf16x2_rn(og[6], og[7]);
        b.x = pack_bf16x2_rn(ou[0], ou[1]); b.y = pack_bf16x2_rn(ou[2], ou[3]);
        b.z = pack_bf16x2_rn(ou[4], ou[5]); b.w = pack_bf16x2_rn(ou[6], ou[7]);
        *reinterpret_cast<uint4*>(dgr + i) = a;
        *reinterpret_cast<uint4*>(dgr + 128 + i) = b;
      }
    }
  }
};

// Backward without the recompute: fused into dh = [dy | dyg] . W_d itself
// (N = intermediate columns).  The accumulator is dh (fp32); gate_pre and up
// come from the bf16 copies the training forward stored (EpiSwiGLUFwd::gu,
// gu_block_offset layout), as in the reference, whose
// fused_gate_up_bwd_kernel reads the bf16 gate_pre/up of recompute_ffn.
// Same formulas, silence terms and hg output as EpiSwiGLUBwd; dgu is written
// row-major in W_gu's interleaving, where intermediate column c sits at
// 256 (c / 128) + c % 128 (gate) and +128 (up).
template <int BN>
struct EpiSwiGLUBwdStored {
  const uint16_t* gu;
  int64_t gu_groups;   // 2F' / 8
  uint16_t* dgu;
  int64_t ldgu_out;
  uint16_t* hg;        // [M, ldhg] graft h (bf16) or null
  int64_t ldhg;
  int M, N;
  int g0, g1;
  int S;
  const float* esq_gate;
  const float* esq_up;
  const int32_t* ood;
  const DevStats* stats;
  static constexpr int kParts = 2;   // two epilogue warps per 32 rows, BN/2 columns each
  static constexpr int kScratchPerWarp = 4096;   // dgu gate + up staging (stage_store_32x32)

  // offset of intermediate column col0 (a multiple of 32) in a gu/dgu row
  __device__ __forceinline__ static int64_t pos(int col0) {
    return 2 * static_cast<int64_t>(col0 & ~127) + (col0 & 127);
  }
  __device__ __forceinline__ void fetch(int row, int col0, uint4 (&g)[4], uint4 (&u)[4]) const {
    const int g8 = static_cast<int>(pos(col0) >> 3);
#pragma unroll
    for (int q = 0; q < 4; ++q) {   // last use: evict first
      g[q] = __ldcs(reinterpret_cast<const uint4*>(gu + gu_block_offset(row, g8 + q, gu_groups)));
      u[q] = __ldcs(reinterpret_cast<const uint4*>(gu + gu_block_offset(row, g8 + 16 + q, gu_groups)));
    }
  }

  // The stored operands of 32 columns are fetched one chunk ahead (chunk 0
  // before the accumulator is read), so the HBM latency overlaps the TMEM
  // loads and the math of the previous chunk instead of serialising with
  // every store.
  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
    const bool graft = (c.n0 + BN > g0) && (c.n0 < g1);
    const bool row_ok = c.row < M;
    float sg_s = 0.f, su_s = 0.f;
    if (graft && row_ok && ood[c.row]) {
      const float lam = stats->lambda_eff;
      const float rs = sqrtf(static_cast<float>(S));
      if (esq_gate) sg_s = lam / (sqrtf(esq_gate[c.row] + 1e-8f) * rs + 1e-8f);
      if (esq_up) su_s = lam / (sqrtf(esq_up[c.row] + 1e-8f) * rs + 1e-8f);
    }
    const int j0 = c.part * (BN / kParts), j1 = j0 + BN / kParts;
    const int band0 = c.row & ~31;
    uint4 ng[4] = {}, nu[4] = {};
    if (row_ok && c.n0 + j0 < N) fetch(c.row, c.n0 + j0, ng, nu);
#pragma unroll 1
    for (int j = j0; j < j1; j += 32) {
      float d[32];
      c.load(j, d);   // warp-collective: every lane loads
      const int col0 = c.n0 + j;
      if (col0 >= N) continue;   // the same for the whole warp
      uint4 gv[4], uv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) { gv[q] = ng[q]; uv[q] = nu[q]; }
      if (row_ok && j + 32 < j1 && col0 + 32 < N) fetch(c.row, col0 + 32, ng, nu);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = 8 * q;
        const float g[8] = {bf16_lo(gv[q].x), bf16_hi(gv[q].x), bf16_lo(gv[q].y), bf16_hi(gv[q].y),
                            bf16_lo(gv[q].z), bf16_hi(gv[q].z), bf16_lo(gv[q].w), bf16_hi(gv[q].w)};
        const float u[8] = {bf16_lo(uv[q].x), bf16_hi(uv[q].x), bf16_lo(uv[q].y), bf16_hi(uv[q].y),
                            bf16_lo(uv[q].z), bf16_hi(uv[q].z), bf16_lo(uv[q].w), bf16_hi(uv[q].w)};
        float og[8], ou[8], hh[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float sg = sigmoidf_(g[k]);
          og[k] = d[i + k] * u[k] * sg * (1.f + g[k] * (1.f - sg));
          ou[k] = d[i + k] * g[k] * sg;
          hh[k] = g[k] * sg * u[k];
        }
        if (graft && row_ok) {
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int col = col0 + i + k;
            if (col >= g0 && col < g1) {
              og[k] += sg_s * g[k];
              ou[k] += su_s * u[k];
              if (hg) hg[static_cast<int64_t>(c.row) * ldhg + (col - g0)] = f32_to_bf16_bits(hh[k]);
            }
          }
        }
        stage_put(c.scratch, 0, q, make_uint4(pack_bf16x2_rn(og[0], og[1]), pack_bf16x2_rn(og[2], og[3]),
                                              pack_bf16x2_rn(og[4], og[5]), pack_bf16x2_rn(og[6], og[7])));
        stage_put(c.scratch, 1, q, make_uint4(pack_bf16x2_rn(ou[0], ou[1]), pack_bf16x2_rn(ou[2], ou[3]),
                                              pack_bf16x2_rn(ou[4], ou[5]), pack_bf16x2_rn(ou[6], ou[7])));
      }
      uint16_t* const g_dst = dgu + static_cast<int64_t>(band0) * ldgu_out + pos(col0);
      uint16_t* const dsts[2] = {g_dst, g_dst + 128};
      stage_flush<2>(c.scratch, dsts, ldgu_out, M - band0);
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
        w.x = pack_bf16x2_rn(v[i], v[i + 1]); w.y = pack_bf16x2_rn(v[i + 2], v[i + 3]);
        w.z = pack_bf16x2_rn(v[i + 4], v[i + 5]); w.w = pack_bf16x2_rn(v[i + 6], v[i + 7]);
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

// ---------------------------------------------------------------------------
// Overlay geometry (the reference's own: the graft overlays intermediate
// columns [i0, i0+S) and hidden columns [h0, h0+H) of the base MLP,
// layer_forward_impl.inc:21-22).  The expand deltas delta = x_h . Delta^T come
// from their own GEMM (fp32) and are injected into the accumulators of the
// slice columns before SwiGLU, in place of fused_inject_clone_energy_kernel's
// bf16 read-modify-write.  i0 and S are multiples of 8, so an 8-column chunk
// is either wholly inside the slice or wholly outside it.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void load8f(const float* p, float* v) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Expand / contract delta GEMM: C (fp32) = acc; optional bf16 copy; per-row
// sums of squares of columns [0, split) into esq_lo and [split, N) into
// esq_hi (the delta energies, kernels_elementwise_impl.inc:287-367).
template <int BN>
struct EpiDeltaF32 {
  float* C;
  int64_t ldc;
  uint16_t* Cb;  // bf16 copy or null
  int64_t ldcb;
  int M, N, split;
  float* esq_lo;
  float* esq_hi;
  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
    float lo = 0.f, hi = 0.f;
#pragma unroll 1
    for (int j = 0; j < BN; j += 32) {
      float v[32];
      c.load(j, v);
      if (c.row >= M) continue;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        const int col = c.n0 + j + i;
        if (col >= N) continue;  // N is a multiple of 8
        float* dst = C + static_cast<int64_t>(c.row) * ldc + col;
        *reinterpret_cast<float4*>(dst) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        *reinterpret_cast<float4*>(dst + 4) = make_float4(v[i + 4], v[i + 5], v[i + 6], v[i + 7]);
        if (Cb) {
          uint4 w;
          w.x = pack_bf16x2_rn(v[i], v[i + 1]); w.y = pack_bf16x2_rn(v[i + 2], v[i + 3]);
          w.z = pack_bf16x2_rn(v[i + 4], v[i + 5]); w.w = pack_bf16x2_rn(v[i + 6], v[i + 7]);
          *reinterpret_cast<uint4*>(Cb + static_cast<int64_t>(c.row) * ldcb + col) = w;
        }
        float ss = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += v[i + k] * v[i + k];
        if (col < split) lo += ss; else hi += ss;
      }
    }
    if (c.row < M) {
      if (esq_lo && lo != 0.f) atomicAdd(esq_lo + c.row, lo);
      if (esq_hi && hi != 0.f) atomicAdd(esq_hi + c.row, hi);
    }
  }
};

// C (bf16) = bf16(acc + inj[:, col - c0] on columns [c0, c1) [+ R]).
// Used by the down GEMM (contract delta into hidden columns [h0, h0+H)) and
// by dh (contract input grad into intermediate columns [i0, i0+S)).
template <int BN>
struct EpiBF16Inj {
  uint16_t* C;
  int64_t ldc;
  const uint16_t* R;  // residual (may alias C) or null
  int64_t ldr;
  int M, N;
  const float* inj;   // or null
  int64_t ld_inj;
  int c0, c1;
  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
#pragma unroll 1
    for (int j = 0; j < BN; j += 32) {
      float v[32];
      c.load(j, v);
      if (c.row >= M) continue;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        const int col = c.n0 + j + i;
        if (col >= N) continue;
        float o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = v[i + k];
        if (inj && col >= c0 && col < c1) {
          float d[8];
          load8f(inj + static_cast<int64_t>(c.row) * ld_inj + (col - c0), d);
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] += d[k];
        }
        if (R) {
          float r[8];
          unpack8(*reinterpret_cast<const uint4*>(R + static_cast<int64_t>(c.row) * ldr + col), r);
#pragma unroll
          for (int k = 0; k < 8; ++k) o[k] += r[k];
        }
        *reinterpret_cast<uint4*>(C + static_cast<int64_t>(c.row) * ldc + col) = pack8(o);
      }
    }
  }
};

// Forward gate/up + SwiGLU with the expand deltas injected on [i0, i1).
struct EpiSwiGLUFwdOv {
  uint16_t* h;
  int64_t ldh;
  int M;
  const float* dg;  // [M, ld_inj] gate delta (column s = intermediate i0+s) or null
  const float* du;  // up delta or null
  int64_t ld_inj;
  int i0, i1;
  uint16_t* gu = nullptr;  // stored gate_pre/up after the injection (gu_block_offset layout) or null
  int64_t gu_groups = 0;   // 2F' / 8
  __device__ __forceinline__ void operator()(const tc::EpiCtx<256>& c) const {
    const int cb = c.n0 >> 1;
#pragma unroll 1
    for (int j = 0; j < 128; j += 32) {
      float g[32], u[32];
      c.load(j, g);
      c.load(128 + j, u);
      if (c.row >= M) continue;
      uint16_t* dst = h + static_cast<int64_t>(c.row) * ldh + cb + j;
#pragma unroll
      for (int i = 0; i < 32; i += 8) {
        const int col = cb + j + i;
        if (col >= i0 && col < i1) {
          const int64_t off = static_cast<int64_t>(c.row) * ld_inj + (col - i0);
          float d[8];
          if (dg) {
            load8f(dg + off, d);
#pragma unroll
            for (int k = 0; k < 8; ++k) g[i + k] += d[k];
          }
          if (du) {
            load8f(du + off, d);
#pragma unroll
            for (int k = 0; k < 8; ++k) u[i + k] += d[k];
          }
        }
        if (gu) {
          const int g8 = ((c.n0 + j) >> 3) + i / 8;
          float gg[8], uu[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) { gg[k] = g[i + k]; uu[k] = u[i + k]; }
          __stcs(reinterpret_cast<uint4*>(gu + gu_block_offset(c.row, g8, gu_groups)), pack8(gg));
          __stcs(reinterpret_cast<uint4*>(gu + gu_block_offset(c.row, g8 + 16, gu_groups)), pack8(uu));
        }
        float o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = g[i + k] * sigmoidf_(g[i + k]) * u[i + k];
        *reinterpret_cast<uint4*>(dst + i) = pack8(o);
      }
    }
  }
};

// Backward of the overlay MLP fused into the gate/up recompute
// (layer_recompute_impl.inc:8-91 + layer_backward_impl.inc:36-361):
//   recompute gp/up (+ injected deltas on the slice), SwiGLU backward into
//   dgu for every column (the base input grad uses the plain dgp/dup);
//   on the slice also the silence-blended expand grads
//     dys_gate = dgp + ood * lambda_eff / (norm_g sqrt(S) + 1e-8) * delta_gate
//   (fused_silence_blend_energy_kernel, :458-560) into dys [M, 2S] (gate
//   columns [0, S), up [S, 2S)), and h = silu(gp) up into hg for the contract
//   weight grad.
struct EpiSwiGLUBwdOv {
  const uint16_t* dh;
  int64_t lddh;
  uint16_t* dgu;
  int64_t ldgu;
  const float* dg;  // gate delta or null (gate not grafted)
  const float* du;
  int64_t ld_inj;
  uint16_t* dys;    // [M, lddys] or null
  int64_t lddys;
  uint16_t* hg;     // [M, ldhg] or null (down not grafted)
  int64_t ldhg;
  int M, i0, i1, S;
  const float* esq_gate;
  const float* esq_up;
  const int32_t* ood;
  const DevStats* stats;
  __device__ __forceinline__ void operator()(const tc::EpiCtx<256>& c) const {
    const int cb = c.n0 >> 1;
    const bool slice = (cb + 128 > i0) && (cb < i1);
    float sg_s = 0.f, su_s = 0.f;
    if (slice && c.row < M && ood[c.row]) {
      const float lam = stats->lambda_eff;
      const float rs = sqrtf(static_cast<float>(S));
      if (dg) sg_s = lam / (sqrtf(esq_gate[c.row] + 1e-8f) * rs + 1e-8f);
      if (du) su_s = lam / (sqrtf(esq_up[c.row] + 1e-8f) * rs + 1e-8f);
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
        const int col = cb + j + i;
        const bool in = col >= i0 && col < i1;
        float deg[8] = {}, deu[8] = {};
        const int64_t off = static_cast<int64_t>(c.row) * ld_inj + (col - i0);
        if (in && dg) {
          load8f(dg + off, deg);
#pragma unroll
          for (int k = 0; k < 8; ++k) g[i + k] += deg[k];
        }
        if (in && du) {
          load8f(du + off, deu);
#pragma unroll
          for (int k = 0; k < 8; ++k) u[i + k] += deu[k];
        }
        float d[8];
        unpack8(*reinterpret_cast<const uint4*>(dhr + i), d);
        float og[8], ou[8], hh[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float gp = g[i + k], up = u[i + k];
          const float sg = sigmoidf_(gp);
          og[k] = d[k] * up * sg * (1.f + gp * (1.f - sg));
          ou[k] = d[k] * gp * sg;
          hh[k] = gp * sg * up;
        }
        *reinterpret_cast<uint4*>(dgr + i) = pack8(og);
        *reinterpret_cast<uint4*>(dgr + 128 + i) = pack8(ou);
        if (in) {
          const int s = col - i0;
          if (dys) {
            float bg[8], bu[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              bg[k] = og[k] + sg_s * deg[k];
              bu[k] = ou[k] + su_s * deu[k];
            }
            uint16_t* dr = dys + static_cast<int64_t>(c.row) * lddys + s;
            if (dg) *reinterpret_cast<uint4*>(dr) = pack8(bg);
            if (du) *reinterpret_cast<uint4*>(dr + S) = pack8(bu);
          }
          if (hg) *reinterpret_cast<uint4*>(hg + static_cast<int64_t>(c.row) * ldhg + s) = pack8(hh);
        }
      }
    }
  }
};

// Overlay geometry without the recompute: dh = dy . W_d with, in the
// epilogue, the ContractInputGrad slice gi (fp32 [M, S], intermediate columns
// [i0, i1)) added, SwiGLU's backward from the stored bf16 gate_pre/up (base +
// delta on the slice, EpiSwiGLUFwdOv::gu), dgu staged through shared memory,
// and on the slice the silence-blended expand grads dys and h for the down
// weight grad -- the outputs of EpiSwiGLUBwdOv, whose recompute GEMM this
// replaces.  The expand deltas (dg, du) feed only the silence term.
template <int BN>
struct EpiSwiGLUBwdStoredOv {
  const uint16_t* gu;
  int64_t gu_groups;   // 2F' / 8
  uint16_t* dgu;
  int64_t ldgu_out;
  const float* gi;     // [M, ld_gi] or null (down not grafted)
  int64_t ld_gi;
  const float* dg;     // [M, ld_inj] expand deltas or null
  const float* du;
  int64_t ld_inj;
  uint16_t* dys;       // [M, lddys] or null
  int64_t lddys;
  uint16_t* hg;        // [M, ldhg] or null
  int64_t ldhg;
  int M, N, i0, i1, S;
  const float* esq_gate;
  const float* esq_up;
  const int32_t* ood;
  const DevStats* stats;
  static constexpr int kParts = 2;
  static constexpr int kScratchPerWarp = 4096;

  __device__ __forceinline__ static int64_t pos(int col0) {
    return 2 * static_cast<int64_t>(col0 & ~127) + (col0 & 127);
  }
  __device__ __forceinline__ void fetch(int row, int col0, uint4 (&g)[4], uint4 (&u)[4]) const {
    const int g8 = static_cast<int>(pos(col0) >> 3);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      g[q] = __ldcs(reinterpret_cast<const uint4*>(gu + gu_block_offset(row, g8 + q, gu_groups)));
      u[q] = __ldcs(reinterpret_cast<const uint4*>(gu + gu_block_offset(row, g8 + 16 + q, gu_groups)));
    }
  }

  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
    const bool slice = (c.n0 + BN > i0) && (c.n0 < i1);
    const bool row_ok = c.row < M;
    float sg_s = 0.f, su_s = 0.f;
    if (slice && row_ok && ood[c.row]) {
      const float lam = stats->lambda_eff;
      const float rs = sqrtf(static_cast<float>(S));
      if (dg) sg_s = lam / (sqrtf(esq_gate[c.row] + 1e-8f) * rs + 1e-8f);
      if (du) su_s = lam / (sqrtf(esq_up[c.row] + 1e-8f) * rs + 1e-8f);
    }
    const int j0 = c.part * (BN / kParts), j1 = j0 + BN / kParts;
    const int band0 = c.row & ~31;
    uint4 ng[4] = {}, nu[4] = {};
    if (row_ok && c.n0 + j0 < N) fetch(c.row, c.n0 + j0, ng, nu);
#pragma unroll 1
    for (int j = j0; j < j1; j += 32) {
      float d[32];
      c.load(j, d);   // warp-collective: every lane loads
      const int col0 = c.n0 + j;
      if (col0 >= N) continue;   // the same for the whole warp
      uint4 gv[4], uv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) { gv[q] = ng[q]; uv[q] = nu[q]; }
      if (row_ok && j + 32 < j1 && col0 + 32 < N) fetch(c.row, col0 + 32, ng, nu);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int i = 8 * q;
        const int col = col0 + i;
        const bool in = row_ok && col >= i0 && col < i1;   // i0, S multiples of 8
        float g[8], u[8], dd[8];
        unpack8(gv[q], g);
        unpack8(uv[q], u);
#pragma unroll
        for (int k = 0; k < 8; ++k) dd[k] = d[i + k];
        const int64_t off_s = col - i0;
        if (in && gi) {
          float t[8];
          load8f(gi + static_cast<int64_t>(c.row) * ld_gi + off_s, t);
#pragma unroll
          for (int k = 0; k < 8; ++k) dd[k] += t[k];
        }
        float og[8], ou[8], hh[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float sg = sigmoidf_(g[k]);
          og[k] = dd[k] * u[k] * sg * (1.f + g[k] * (1.f - sg));
          ou[k] = dd[k] * g[k] * sg;
          hh[k] = g[k] * sg * u[k];
        }
        stage_put(c.scratch, 0, q, pack8(og));
        stage_put(c.scratch, 1, q, pack8(ou));
        if (in) {
          if (dys) {
            const int64_t off = static_cast<int64_t>(c.row) * ld_inj + off_s;
            float de[8], b[8];
            uint16_t* dr = dys + static_cast<int64_t>(c.row) * lddys + off_s;
            if (dg) {
              load8f(dg + off, de);
#pragma unroll
              for (int k = 0; k < 8; ++k) b[k] = og[k] + sg_s * de[k];
              *reinterpret_cast<uint4*>(dr) = pack8(b);
            }
            if (du) {
              load8f(du + off, de);
#pragma unroll
              for (int k = 0; k < 8; ++k) b[k] = ou[k] + su_s * de[k];
              *reinterpret_cast<uint4*>(dr + S) = pack8(b);
            }
          }
          if (hg) *reinterpret_cast<uint4*>(hg + static_cast<int64_t>(c.row) * ldhg + off_s) = pack8(hh);
        }
      }
      uint16_t* const g_dst = dgu + static_cast<int64_t>(band0) * ldgu_out + pos(col0);
      uint16_t* const dsts[2] = {g_dst, g_dst + 128};
      stage_flush<2>(c.scratch, dsts, ldgu_out, M - band0);
    }
  }
};

}  // namespace glt
