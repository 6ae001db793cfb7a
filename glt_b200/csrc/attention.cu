// Flash-style causal GQA attention, forward and backward, plus RoPE.
//
// Tiles of 64 queries x 64 keys; 4 warps per CTA, each warp owns 16 rows.
// Q/K/V/dO tiles are staged in shared memory with cp.async (double
// buffered) in an XOR-swizzled layout (16-byte chunk c of row r stored at
// chunk c ^ (r & 7)) so that ldmatrix reads are bank-conflict free.  The
// products run on the bf16 tensor cores with fp32 accumulation; softmax is
// kept online in the exp2 domain.  The backward pass follows the usual
// flash decomposition: one CTA per (64-key tile, kv head, batch) loops over
// the GQA query heads and the causal query tiles, accumulates dK/dV in
// registers and reduces dQ through fp32 atomics.
#include <math.h>

#include "attention.cuh"
#include "common.cuh"
#include "gemm.cuh"

namespace glt {
namespace {

constexpr float LOG2E = 1.4426950408889634f;

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pk(float a, float b) { return pack_bf16x2(a, b); }

// byte offset of element (row, col) in a swizzled tile with ROWB bytes per row
template <int ROWB>
__device__ __forceinline__ uint32_t swz(int row, int col) {
  return static_cast<uint32_t>(row * ROWB + ((((col >> 3) ^ (row & 7))) << 4) + ((col & 7) << 1));
}

// Copies a [64 x HD] bf16 tile (row stride ld elements) into swizzled smem.
template <int HD>
__device__ __forceinline__ void load_tile(uint32_t s_base, const uint16_t* g, int64_t ld) {
  constexpr int CH = HD / 8;  // 16-byte chunks per row
#pragma unroll
  for (int i = threadIdx.x; i < 64 * CH; i += 128) {
    const int r = i / CH, c = i % CH;
    cp_async16(s_base + swz<HD * 2>(r, c * 8), g + r * ld + c * 8);
  }
}

// ------------------------------- forward -----------------------------------
template <int HD>
__global__ void __launch_bounds__(128) flash_fwd_kernel(const uint16_t* __restrict__ qkv,
                                                        uint16_t* __restrict__ o,
                                                        float* __restrict__ lse, AttnShape s) {
  extern __shared__ __align__(128) uint8_t sm[];
  constexpr int TILE = 64 * HD * 2;
  const uint32_t sQ = saddr(sm), sK = sQ + TILE, sV = sK + 2 * TILE;
  const int qt = gridDim.x - 1 - blockIdx.x;  // heaviest tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (s.nh / s.nkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row0 = static_cast<int64_t>(b) * s.T;
  const uint16_t* qg = qkv + (row0 + qt * 64) * s.ld_qkv + h * HD;
  const uint16_t* kg = qkv + row0 * s.ld_qkv + (s.nh + kvh) * HD;
  const uint16_t* vg = qkv + row0 * s.ld_qkv + (s.nh + s.nkv + kvh) * HD;
  const float sl2 = s.scale * LOG2E;

  load_tile<HD>(sQ, qg, s.ld_qkv);
  load_tile<HD>(sK, kg, s.ld_qkv);
  load_tile<HD>(sV, vg, s.ld_qkv);
  cp_commit();

  uint32_t qf[HD / 16][4];
  float oacc[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  const int n_kv = qt + 1;
  for (int j = 0; j < n_kv; ++j) {
    const int st = j & 1;
    if (j + 1 < n_kv) {
      load_tile<HD>(sK + ((j + 1) & 1) * TILE, kg + static_cast<int64_t>(j + 1) * 64 * s.ld_qkv,
                    s.ld_qkv);
      load_tile<HD>(sV + ((j + 1) & 1) * TILE, vg + static_cast<int64_t>(j + 1) * 64 * s.ld_qkv,
                    s.ld_qkv);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk)
        ldsm_x4(sQ + swz<HD * 2>(warp * 16 + (lane & 15), kk * 16 + (lane >> 4) * 8), qf[kk][0],
                qf[kk][1], qf[kk][2], qf[kk][3]);
    }
    const uint32_t kb = sK + st * TILE, vb = sV + st * TILE;
    float sacc[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) sacc[i][0] = sacc[i][1] = sacc[i][2] = sacc[i][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4(kb + swz<HD * 2>(np * 16 + (lane & 7) + (lane >> 4) * 8,
                                 kk * 16 + ((lane >> 3) & 1) * 8),
                r0, r1, r2, r3);
        mma16816(sacc[2 * np], qf[kk], r0, r1);
        mma16816(sacc[2 * np + 1], qf[kk], r2, r3);
      }
    }
    // scale, causal mask, online softmax
    const int qr0 = qt * 64 + warp * 16 + (lane >> 2);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = j * 64 + nt * 8 + (lane & 3) * 2 + (e & 1);
        const int qr = qr0 + (e >> 1) * 8;
        float v = sacc[nt][e] * sl2;
        if (j == qt && key > qr) v = -INFINITY;
        sacc[nt][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mn = fmaxf(mrow[r], mx[r]);
      alpha[r] = (mrow[r] == -INFINITY) ? 0.f : exp2f(mrow[r] - mn);
      mrow[r] = mn;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(sacc[nt][e] - mrow[e >> 1]);
        sacc[nt][e] = p;
        rs[e >> 1] += p;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      lrow[r] = lrow[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
      oacc[i][0] *= alpha[0];
      oacc[i][1] *= alpha[0];
      oacc[i][2] *= alpha[1];
      oacc[i][3] *= alpha[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t pa[4] = {pk(sacc[2 * kk][0], sacc[2 * kk][1]), pk(sacc[2 * kk][2], sacc[2 * kk][3]),
                              pk(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]),
                              pk(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3])};
#pragma unroll
      for (int dp = 0; dp < HD / 16; ++dp) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(vb + swz<HD * 2>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                                   dp * 16 + (lane >> 4) * 8),
                  r0, r1, r2, r3);
        mma16816(oacc[2 * dp], pa, r0, r1);
        mma16816(oacc[2 * dp + 1], pa, r2, r3);
      }
    }
    __syncthreads();
  }
  // epilogue
  const float inv[2] = {1.f / lrow[0], 1.f / lrow[1]};
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t t = row0 + qt * 64 + warp * 16 + (lane >> 2) + r * 8;
    uint16_t* orow = o + t * s.ld_o + h * HD;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt) {
      const int c = nt * 8 + (lane & 3) * 2;
      *reinterpret_cast<uint32_t*>(orow + c) =
          pk(oacc[nt][2 * r] * inv[r], oacc[nt][2 * r + 1] * inv[r]);
    }
    if ((lane & 3) == 0)
      lse[(static_cast<int64_t>(b) * s.nh + h) * s.T + qt * 64 + warp * 16 + (lane >> 2) + r * 8] =
          (mrow[r] + log2f(lrow[r])) / LOG2E;
  }
}

// --------------------------- backward helpers ------------------------------
template <int HD>
__global__ void bwd_dsum_kernel(const uint16_t* __restrict__ o, const uint16_t* __restrict__ dout,
                                float* __restrict__ dsum, AttnShape s) {
  // one warp per (token, head)
  const int64_t gw = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t M = static_cast<int64_t>(s.B) * s.T;
  if (gw >= M * s.nh) return;
  const int64_t t = gw / s.nh;
  const int h = static_cast<int>(gw % s.nh);
  const uint16_t* orow = o + t * s.ld_o + h * HD;
  const uint16_t* drow = dout + t * s.ld_o + h * HD;
  float acc = 0.f;
  for (int d = lane * 2; d < HD; d += 64) {
    const uint32_t a = *reinterpret_cast<const uint32_t*>(orow + d);
    const uint32_t c = *reinterpret_cast<const uint32_t*>(drow + d);
    acc += bf16_lo(a) * bf16_lo(c) + bf16_hi(a) * bf16_hi(c);
  }
  acc = warp_sum(acc);
  if (lane == 0) {
    const int b = static_cast<int>(t / s.T), tt = static_cast<int>(t % s.T);
    dsum[(static_cast<int64_t>(b) * s.nh + h) * s.T + tt] = acc;
  }
}

template <int HD>
__global__ void __launch_bounds__(128) flash_bwd_kernel(
    const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ dout,
    const float* __restrict__ lse, const float* __restrict__ dsum, uint16_t* __restrict__ dqkv,
    float* __restrict__ dq_acc, AttnShape s) {
  extern __shared__ __align__(128) uint8_t sm[];
  constexpr int TILE = 64 * HD * 2;
  const uint32_t sK = saddr(sm), sV = sK + TILE, sQ = sV + TILE, sdO = sQ + 2 * TILE,
                 sdS = sdO + 2 * TILE;
  float* sL = reinterpret_cast<float*>(sm + 6 * TILE + 64 * 64 * 2);  // [2][64]
  float* sD = sL + 128;                                                // [2][64]
  const int kt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rep = s.nh / s.nkv;
  const int nqt = s.T / 64;
  const int64_t row0 = static_cast<int64_t>(b) * s.T;
  const float sl2 = s.scale * LOG2E;
  const uint16_t* kg = qkv + (row0 + kt * 64) * s.ld_qkv + (s.nh + kvh) * HD;
  const uint16_t* vg = qkv + (row0 + kt * 64) * s.ld_qkv + (s.nh + s.nkv + kvh) * HD;
  const int64_t ldq = static_cast<int64_t>(s.nh) * HD;  // dq_acc row stride

  load_tile<HD>(sK, kg, s.ld_qkv);
  load_tile<HD>(sV, vg, s.ld_qkv);
  const int items_per_head = nqt - kt;
  const int n_items = rep * items_per_head;
  auto issue = [&](int item, int stage) {
    const int h = kvh * rep + item / items_per_head;
    const int qt = kt + item % items_per_head;
    load_tile<HD>(sQ + stage * TILE, qkv + (row0 + qt * 64) * s.ld_qkv + h * HD, s.ld_qkv);
    load_tile<HD>(sdO + stage * TILE, dout + (row0 + qt * 64) * s.ld_o + h * HD, s.ld_o);
    if (threadIdx.x < 64) {
      const int64_t li = (static_cast<int64_t>(b) * s.nh + h) * s.T + qt * 64 + threadIdx.x;
      sL[stage * 64 + threadIdx.x] = lse[li] * LOG2E;
      sD[stage * 64 + threadIdx.x] = dsum[li];
    }
  };
  issue(0, 0);
  cp_commit();

  float dk[HD / 8][4], dv[HD / 8][4];
#pragma unroll
  for (int i = 0; i < HD / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  for (int it = 0; it < n_items; ++it) {
    const int stg = it & 1;
    if (it + 1 < n_items) {
      issue(it + 1, (it + 1) & 1);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const int h = kvh * rep + it / items_per_head;
    const int qt = kt + it % items_per_head;
    const uint32_t qb = sQ + stg * TILE, db = sdO + stg * TILE;
    const float* Ls = sL + stg * 64;
    const float* Ds = sD + stg * 64;

    // S^T = K_w Q^T and dP^T = V_w dO^T   (16 keys x 64 queries per warp)
    float st[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[i][e] = dp[i][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t ka[4], va[4];
      ldsm_x4(sK + swz<HD * 2>(warp * 16 + (lane & 15), kk * 16 + (lane >> 4) * 8), ka[0], ka[1],
              ka[2], ka[3]);
      ldsm_x4(sV + swz<HD * 2>(warp * 16 + (lane & 15), kk * 16 + (lane >> 4) * 8), va[0], va[1],
              va[2], va[3]);
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4(qb + swz<HD * 2>(np * 16 + (lane & 7) + (lane >> 4) * 8,
                                 kk * 16 + ((lane >> 3) & 1) * 8),
                r0, r1, r2, r3);
        mma16816(st[2 * np], ka, r0, r1);
        mma16816(st[2 * np + 1], ka, r2, r3);
        ldsm_x4(db + swz<HD * 2>(np * 16 + (lane & 7) + (lane >> 4) * 8,
                                 kk * 16 + ((lane >> 3) & 1) * 8),
                r0, r1, r2, r3);
        mma16816(dp[2 * np], va, r0, r1);
        mma16816(dp[2 * np + 1], va, r2, r3);
      }
    }
    // P^T and dS^T
    const int key0 = kt * 64 + warp * 16 + (lane >> 2);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = nt * 8 + (lane & 3) * 2 + (e & 1);
        const int key = key0 + (e >> 1) * 8;
        float p = exp2f(st[nt][e] * sl2 - Ls[ql]);
        if (qt == kt && key > qt * 64 + ql) p = 0.f;
        st[nt][e] = p;
        dp[nt][e] = p * (dp[nt][e] - Ds[ql]);
      }
    }
    // dV += P^T dO ; dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t pa[4] = {pk(st[2 * kk][0], st[2 * kk][1]), pk(st[2 * kk][2], st[2 * kk][3]),
                              pk(st[2 * kk + 1][0], st[2 * kk + 1][1]),
                              pk(st[2 * kk + 1][2], st[2 * kk + 1][3])};
      const uint32_t sa[4] = {pk(dp[2 * kk][0], dp[2 * kk][1]), pk(dp[2 * kk][2], dp[2 * kk][3]),
                              pk(dp[2 * kk + 1][0], dp[2 * kk + 1][1]),
                              pk(dp[2 * kk + 1][2], dp[2 * kk + 1][3])};
#pragma unroll
      for (int d2 = 0; d2 < HD / 16; ++d2) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(db + swz<HD * 2>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                                   d2 * 16 + (lane >> 4) * 8),
                  r0, r1, r2, r3);
        mma16816(dv[2 * d2], pa, r0, r1);
        mma16816(dv[2 * d2 + 1], pa, r2, r3);
        ldsm_x4_t(qb + swz<HD * 2>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                                   d2 * 16 + (lane >> 4) * 8),
                  r0, r1, r2, r3);
        mma16816(dk[2 * d2], sa, r0, r1);
        mma16816(dk[2 * d2 + 1], sa, r2, r3);
      }
    }
    // dS^T -> smem [key][q] (bf16, swizzled 128-byte rows)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int kr = warp * 16 + (lane >> 2) + r * 8;
        const int qc = nt * 8 + (lane & 3) * 2;
        asm volatile("st.shared.b32 [%0], %1;" ::"r"(sdS + swz<128>(kr, qc)),
                     "r"(pk(dp[nt][2 * r], dp[nt][2 * r + 1])));
      }
    }
    __syncthreads();
    // dQ rows [16w, 16w+16) of this q tile: dS (q x key) * K (key x d)
    {
      float dq[HD / 8][4];
#pragma unroll
      for (int i = 0; i < HD / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        ldsm_x4_t(sdS + swz<128>(kk * 16 + (lane & 7) + (lane >> 4) * 8,
                                 warp * 16 + ((lane >> 3) & 1) * 8),
                  a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int d2 = 0; d2 < HD / 16; ++d2) {
          uint32_t r0, r1, r2, r3;
          ldsm_x4_t(sK + swz<HD * 2>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8,
                                     d2 * 16 + (lane >> 4) * 8),
                    r0, r1, r2, r3);
          mma16816(dq[2 * d2], a, r0, r1);
          mma16816(dq[2 * d2 + 1], a, r2, r3);
        }
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        float* dst = dq_acc + (row0 + qt * 64 + warp * 16 + (lane >> 2) + r * 8) * ldq + h * HD;
#pragma unroll
        for (int nt = 0; nt < HD / 8; ++nt) {
          const int c = nt * 8 + (lane & 3) * 2;
          red_add_f32(dst + c, dq[nt][2 * r] * s.scale);
          red_add_f32(dst + c + 1, dq[nt][2 * r + 1] * s.scale);
        }
      }
    }
    __syncthreads();
  }
  // write dK (scaled) and dV for this warp's 16 keys
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int64_t t = row0 + kt * 64 + warp * 16 + (lane >> 2) + r * 8;
    uint16_t* krow = dqkv + t * s.ld_qkv + (s.nh + kvh) * HD;
    uint16_t* vrow = dqkv + t * s.ld_qkv + (s.nh + s.nkv + kvh) * HD;
#pragma unroll
    for (int nt = 0; nt < HD / 8; ++nt) {
      const int c = nt * 8 + (lane & 3) * 2;
      *reinterpret_cast<uint32_t*>(krow + c) =
          pk(dk[nt][2 * r] * s.scale, dk[nt][2 * r + 1] * s.scale);
      *reinterpret_cast<uint32_t*>(vrow + c) = pk(dv[nt][2 * r], dv[nt][2 * r + 1]);
    }
  }
}

// dq_acc (fp32) -> bf16 q columns of dqkv
__global__ void dq_convert_kernel(const float* __restrict__ acc, uint16_t* __restrict__ dqkv,
                                  int64_t M, int qcols, int64_t ld) {
  const int64_t n = M * qcols / 4;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t e = i * 4;
    const int64_t t = e / qcols;
    const int c = static_cast<int>(e % qcols);
    const float4 v = reinterpret_cast<const float4*>(acc)[i];
    uint2 o;
    o.x = pk(v.x, v.y);
    o.y = pk(v.z, v.w);
    *reinterpret_cast<uint2*>(dqkv + t * ld + c) = o;
  }
}

// dq (fp32 accumulator) -> bf16 q columns of dqkv with the inverse RoPE
// (the transpose of rope_kernel's rotation) applied before the rounding:
// one thread per (token, head, 4 dims of the first half) and their partners.
__global__ void dq_convert_rope_kernel(const float* __restrict__ acc, uint16_t* __restrict__ dqkv, int64_t M,
                                       int nh, int hd, int64_t ld, int T, const float* __restrict__ cs,
                                       const float* __restrict__ sn) {
  const int half = hd / 2;
  const int groups = half / 4;
  const int64_t total = M * nh * groups;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % groups);
    const int64_t r = i / groups;
    const int h = static_cast<int>(r % nh);
    const int64_t t = r / nh;
    const int pos = static_cast<int>(t % T);
    const float* a = acc + t * (static_cast<int64_t>(nh) * hd) + static_cast<int64_t>(h) * hd + g * 4;
    const float4 x1 = *reinterpret_cast<const float4*>(a);
    const float4 x2 = *reinterpret_cast<const float4*>(a + half);
    const float4 co = *reinterpret_cast<const float4*>(cs + static_cast<int64_t>(pos) * half + g * 4);
    const float4 si = *reinterpret_cast<const float4*>(sn + static_cast<int64_t>(pos) * half + g * 4);
    uint2 o1, o2;
    o1.x = pk(x1.x * co.x + x2.x * si.x, x1.y * co.y + x2.y * si.y);
    o1.y = pk(x1.z * co.z + x2.z * si.z, x1.w * co.w + x2.w * si.w);
    o2.x = pk(x2.x * co.x - x1.x * si.x, x2.y * co.y - x1.y * si.y);
    o2.y = pk(x2.z * co.z - x1.z * si.z, x2.w * co.w - x1.w * si.w);
    uint16_t* d = dqkv + t * ld + static_cast<int64_t>(h) * hd + g * 4;
    *reinterpret_cast<uint2*>(d) = o1;
    *reinterpret_cast<uint2*>(d + half) = o2;
  }
}

// RoPE: one thread per (token, head, 8 consecutive dims of the first half)
__global__ void rope_kernel(uint16_t* __restrict__ qkv, AttnShape s, const float* __restrict__ cs,
                            const float* __restrict__ sn, int inverse, int head_begin,
                            int head_end) {
  const int half = s.hd / 2;
  const int vec_per_head = half / 8;
  const int heads = head_end - head_begin;
  const int64_t total = static_cast<int64_t>(s.B) * s.T * heads * vec_per_head;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int v = static_cast<int>(i % vec_per_head);
    const int64_t r = i / vec_per_head;
    const int hh = head_begin + static_cast<int>(r % heads);
    const int64_t t = r / heads;
    const int pos = static_cast<int>(t % s.T);
    uint16_t* p = qkv + t * s.ld_qkv + static_cast<int64_t>(hh) * s.hd + v * 8;
    uint4 a = *reinterpret_cast<uint4*>(p);
    uint4 c = *reinterpret_cast<uint4*>(p + half);
    const float* cp = cs + static_cast<int64_t>(pos) * half + v * 8;
    const float* sp = sn + static_cast<int64_t>(pos) * half + v * 8;
    uint32_t* aw = reinterpret_cast<uint32_t*>(&a);
    uint32_t* cw = reinterpret_cast<uint32_t*>(&c);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x1[2] = {bf16_lo(aw[j]), bf16_hi(aw[j])};
      float x2[2] = {bf16_lo(cw[j]), bf16_hi(cw[j])};
      float r1[2], r2[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const float co = cp[2 * j + k], si = sp[2 * j + k];
        if (!inverse) {
          r1[k] = x1[k] * co - x2[k] * si;
          r2[k] = x2[k] * co + x1[k] * si;
        } else {
          r1[k] = x1[k] * co + x2[k] * si;
          r2[k] = x2[k] * co - x1[k] * si;
        }
      }
      aw[j] = pk(r1[0], r1[1]);
      cw[j] = pk(r2[0], r2[1]);
    }
    *reinterpret_cast<uint4*>(p) = a;
    *reinterpret_cast<uint4*>(p + half) = c;
  }
}

template <int HD>
int fwd_impl(const uint16_t* qkv, uint16_t* o, float* lse, const AttnShape& s, cudaStream_t st) {
  const int smem = 5 * 64 * HD * 2;
  auto k = flash_fwd_kernel<HD>;
  GLT_TRY(ensure_smem_attr(reinterpret_cast<const void*>(k), smem));
  dim3 grid(s.T / 64, s.nh, s.B);
  k<<<grid, 128, smem, st>>>(qkv, o, lse, s);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

template <int HD>
int bwd_prep_impl(const uint16_t* o, const uint16_t* dout, float* dq_acc, float* dsum,
                  const AttnShape& s, cudaStream_t st, bool dsum_ready = false) {
  const int64_t M = static_cast<int64_t>(s.B) * s.T;
  GLT_CUDA_TRY(cudaMemsetAsync(dq_acc, 0, M * s.nh * HD * sizeof(float), st));
  if (dsum_ready) return GLT_OK;
  const int64_t warps = M * s.nh;
  const int blocks = static_cast<int>((warps * 32 + 255) / 256);
  bwd_dsum_kernel<HD><<<blocks, 256, 0, st>>>(o, dout, dsum, s);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int bwd_finish_impl(const float* dq_acc, uint16_t* dqkv, const AttnShape& s, cudaStream_t st,
                    const float* rope_cos = nullptr, const float* rope_sin = nullptr) {
  const int64_t M = static_cast<int64_t>(s.B) * s.T;
  if (rope_cos) {
    const int64_t n = M * s.nh * (s.hd / 8);
    int blocks = static_cast<int>((n + 255) / 256);
    if (blocks > num_sms() * 16) blocks = num_sms() * 16;
    dq_convert_rope_kernel<<<blocks, 256, 0, st>>>(dq_acc, dqkv, M, s.nh, s.hd, s.ld_qkv, s.T, rope_cos, rope_sin);
    GLT_LAUNCH_CHECK();
    return GLT_OK;
  }
  const int64_t n = M * s.nh * s.hd / 4;
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > num_sms() * 16) blocks = num_sms() * 16;
  dq_convert_kernel<<<blocks, 256, 0, st>>>(dq_acc, dqkv, M, s.nh * s.hd, s.ld_qkv);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

template <int HD>
int bwd_impl(const uint16_t* qkv, const uint16_t* o, const uint16_t* dout, const float* lse,
             uint16_t* dqkv, float* dq_acc, float* dsum, const AttnShape& s, cudaStream_t st) {
  GLT_TRY(bwd_prep_impl<HD>(o, dout, dq_acc, dsum, s, st));
  const int smem = 6 * 64 * HD * 2 + 64 * 64 * 2 + 4 * 64 * 4;
  auto k = flash_bwd_kernel<HD>;
  GLT_TRY(ensure_smem_attr(reinterpret_cast<const void*>(k), smem));
  dim3 grid(s.T / 64, s.nkv, s.B);
  k<<<grid, 128, smem, st>>>(qkv, dout, lse, dsum, dqkv, dq_acc, s);
  GLT_LAUNCH_CHECK();
  return bwd_finish_impl(dq_acc, dqkv, s, st);
}

int check_shape(const AttnShape& s) {
  if (s.hd != 64 && s.hd != 128) return fail(GLT_EINVAL, "attention: head_dim %d unsupported", s.hd);
  if (s.T % 64) return fail(GLT_EINVAL, "attention: seq_len %d not a multiple of 64", s.T);
  if (s.nkv <= 0 || s.nh % s.nkv) return fail(GLT_EINVAL, "attention: nh %% nkv != 0");
  if (s.ld_qkv % 8 || s.ld_o % 8) return fail(GLT_EINVAL, "attention: strides not 16-byte");
  return GLT_OK;
}

}  // namespace

int rope_apply(uint16_t* qkv, const AttnShape& s, const float* cos_t, const float* sin_t,
               int inverse, int apply_q, int apply_k, cudaStream_t st) {
  if (s.hd % 16) return fail(GLT_EINVAL, "rope: head_dim %% 16 != 0");
  const int hb = apply_q ? 0 : s.nh;
  const int he = apply_k ? s.nh + s.nkv : s.nh;
  if (he <= hb) return GLT_OK;
  const int64_t total = static_cast<int64_t>(s.B) * s.T * (he - hb) * (s.hd / 16);
  int blocks = static_cast<int>((total + 255) / 256);
  if (blocks > num_sms() * 16) blocks = num_sms() * 16;
  rope_kernel<<<blocks, 256, 0, st>>>(qkv, s, cos_t, sin_t, inverse, hb, he);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

int flash_fwd(const uint16_t* qkv, uint16_t* o, float* lse, const AttnShape& s, cudaStream_t st) {
  GLT_TRY(check_shape(s));
  return s.hd == 128 ? fwd_impl<128>(qkv, o, lse, s, st) : fwd_impl<64>(qkv, o, lse, s, st);
}

int attn_bwd_prep(const uint16_t* o, const uint16_t* dout, float* dq_acc, float* dsum,
                  const AttnShape& s, cudaStream_t st, bool dsum_ready) {
  GLT_TRY(check_shape(s));
  return s.hd == 128 ? bwd_prep_impl<128>(o, dout, dq_acc, dsum, s, st, dsum_ready)
                     : bwd_prep_impl<64>(o, dout, dq_acc, dsum, s, st, dsum_ready);
}

int attn_bwd_finish(const float* dq_acc, uint16_t* dqkv, const AttnShape& s, cudaStream_t st,
                    const float* rope_cos, const float* rope_sin) {
  if (rope_cos && (s.hd % 8 || !rope_sin)) return fail(GLT_EINVAL, "attn_bwd_finish: rope tables");
  return bwd_finish_impl(dq_acc, dqkv, s, st, rope_cos, rope_sin);
}

int flash_bwd(const uint16_t* qkv, const uint16_t* o, const uint16_t* dout, const float* lse,
              uint16_t* dqkv, float* dq_acc, float* dsum, const AttnShape& s, cudaStream_t st) {
  GLT_TRY(check_shape(s));
  return s.hd == 128 ? bwd_impl<128>(qkv, o, dout, lse, dqkv, dq_acc, dsum, s, st)
                     : bwd_impl<64>(qkv, o, dout, lse, dqkv, dq_acc, dsum, s, st);
}

}  // namespace glt
