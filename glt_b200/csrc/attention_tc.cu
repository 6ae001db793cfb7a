// Causal GQA flash-attention forward on the 5th-generation tensor cores.
//
// One CTA per (128-query tile, head, batch); 6 warps:
//   warp 0      TMA producer: the Q tile once, then 64-key K/V tiles into a
//               3-stage ring (128B swizzle, plain per-CTA loads)
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer:
//                 S_j = Q.K_j^T   (M=128, N=64,  K=hd; both operands K-major)
//                 O  += P_j.V_j   (M=128, N=hd,  K=64; P K-major, V MN-major)
//               S_{j+1} is issued before O += P_j.V_j so the softmax of tile j
//               overlaps the next QK^T.
//   warps 2..5  softmax: thread i owns query row i (= TMEM lane i); reads its
//               S row with tcgen05.ld, keeps the running max / sum, writes the
//               bf16 probabilities into a 128B-swizzled smem tile that is the
//               K-major A operand of the PV product, and writes the output.
// TMEM: two S buffers (64 columns each) + O (hd columns).
// The O rescale of online softmax is conditional: the running max used for
// the exponentials only moves when a row's max grows by more than 2^8, so the
// O read-modify-write in TMEM (which must wait for the previous PV product)
// is rare; p = exp2(s - m) stays <= 256, well inside fp32/bf16 range, and the
// final normalisation uses the same m for O and the row sum.
// All mbarrier waits are bounded (tc::mbar_wait); a timeout sets the device
// error word and the CTA drains instead of hanging.
#include <math.h>

#include "attention.cuh"
#include "common.cuh"
#include "gemm.cuh"
#include "tc_gemm.cuh"

namespace glt {
namespace {

using namespace tc;

constexpr int AQ = 128;      // query rows per CTA
constexpr int AK = 64;       // keys per tile
constexpr int KV_STAGES = 3;
constexpr float LOG2E_F = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

template <int HD>
struct FwdSmem {
  static constexpr uint32_t Q_BYTES = AQ * HD * 2;          // HD/64 blocks of [128 x 128B]
  static constexpr uint32_t K_BYTES = AK * HD * 2;          // HD/64 blocks of [64 x 128B]
  static constexpr uint32_t V_BYTES = AK * HD * 2;          // HD/64 chunks of [64 x 128B]
  static constexpr uint32_t P_BYTES = AQ * AK * 2;          // [128 x 128B]
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + KV_STAGES * K_BYTES;
  static constexpr uint32_t OFF_P = OFF_V + KV_STAGES * V_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_P + 2 * P_BYTES;
  static constexpr uint32_t NUM_BARS = 1 + 2 * KV_STAGES + 2 + 2 + 2 + 2 + 1;
  static constexpr uint32_t TOTAL = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
};

template <int HD>
__global__ void __launch_bounds__(192, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_kv, uint16_t* __restrict__ o,
                       float* __restrict__ lse, AttnShape s, unsigned int* err) {
  using L = FwdSmem<HD>;
  constexpr uint32_t TMEM_COLS = 256;   // S0 | S1 | O (HD <= 128)
  constexpr uint32_t ID_S = make_idesc(AK, false, false);
  constexpr uint32_t ID_PV = make_idesc(HD, false, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + KV_STAGES;
  uint64_t* s_full = kv_empty + KV_STAGES;  // [2]
  uint64_t* s_free = s_full + 2;            // [2]
  uint64_t* p_full = s_free + 2;            // [2]
  uint64_t* p_free = p_full + 2;            // [2]  (= PV product done)
  uint64_t* drain = p_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ int abort_flag;
  volatile int& s_abort = abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = gridDim.x - 1 - blockIdx.x;   // heaviest tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (s.nh / s.nkv);
  const int n_kv = (qt * AQ + AQ) / AK;        // causal: keys < (qt+1)*128
  const int row_base = b * s.T;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KV_STAGES; ++i) { mbar_init(&kv_full[i], 1); mbar_init(&kv_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(drain, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_kv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = smem_u32(sm + L::OFF_Q);
  const uint32_t sK = smem_u32(sm + L::OFF_K);
  const uint32_t sV = smem_u32(sm + L::OFF_V);
  const uint32_t sP = smem_u32(sm + L::OFF_P);

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      const int qcol = h * HD, kcol = (s.nh + kvh) * HD, vcol = (s.nh + s.nkv + kvh) * HD;
      mbar_arrive_expect_tx(q_full, L::Q_BYTES);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c)
        tma_load_2d(sm + L::OFF_Q + c * (AQ * 128), &tm_q, q_full, qcol + 64 * c, row_base + qt * AQ);
      for (int j = 0; j < n_kv && !s_abort; ++j) {
        const int st = j % KV_STAGES;
        if (!mbar_wait(&kv_empty[st], ((j / KV_STAGES) & 1) ^ 1, err)) { s_abort = 1; break; }
        mbar_arrive_expect_tx(&kv_full[st], L::K_BYTES + L::V_BYTES);
        uint8_t* kb = sm + L::OFF_K + st * L::K_BYTES;
        uint8_t* vb = sm + L::OFF_V + st * L::V_BYTES;
#pragma unroll
        for (int c = 0; c < HD / 64; ++c) {
          tma_load_2d(kb + c * (AK * 128), &tm_kv, &kv_full[st], kcol + 64 * c, row_base + j * AK);
          tma_load_2d(vb + c * (AK * 128), &tm_kv, &kv_full[st], vcol + 64 * c, row_base + j * AK);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      auto issue_s = [&](int j) -> bool {
        const int st = j % KV_STAGES, sb = j & 1;
        if (!mbar_wait(&kv_full[st], (j / KV_STAGES) & 1, err)) return false;
        if (!mbar_wait(&s_free[sb], ((j >> 1) & 1) ^ 1, err)) return false;
        tc_fence_after();
        const uint32_t kb = sK + st * L::K_BYTES;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t ad = desc_kmajor(sQ + (k >> 2) * (AQ * 128), k & 3);
          const uint64_t bd = desc_kmajor(kb + (k >> 2) * (AK * 128), k & 3);
          umma_bf16(tmem + sb * AK, ad, bd, ID_S, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, err);
      if (ok) { tc_fence_after(); ok = issue_s(0); }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) { ok = false; break; }
        const int sb = j & 1, st = j % KV_STAGES;
        if (!mbar_wait(&p_full[sb], (j >> 1) & 1, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t vb = sV + st * L::V_BYTES;
        const uint32_t pb = sP + sb * L::P_BYTES;
#pragma unroll
        for (int k = 0; k < AK / 16; ++k) {
          const uint64_t ad = desc_kmajor(pb, k);
          const uint64_t bd = desc_mnmajor(vb, k);
          umma_bf16(tmem + 2 * AK, ad, bd, ID_PV, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(&p_free[sb]);
        umma_commit(&kv_empty[st]);
      }
      if (!ok) s_abort = 1;
    }
  } else {
    // ------------------------------- softmax ------------------------------
    const int sub = warp & 3;
    const int r = sub * 32 + lane;             // row in the tile / TMEM lane
    const int qrow = qt * AQ + r;              // position in the sequence
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const float sl2 = s.scale * LOG2E_F;
    float m_run = -INFINITY, l_run = 0.f;
    for (int j = 0; j < n_kv; ++j) {
      const int sb = j & 1;
      if (!mbar_wait(&s_full[sb], (j >> 1) & 1, err)) { s_abort = 1; break; }
      tc_fence_after();
      float sv[AK];
      {
        float t[32];
        tmem_ld32(tmem + lane_off + sb * AK, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[i] = t[i];
        tmem_ld32(tmem + lane_off + sb * AK + 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[32 + i] = t[i];
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[sb]);
      // causal mask (diagonal tiles only) + tile max of the raw scores; the
      // scale is positive, so it is applied to the max and folded into the
      // exponent's FFMA below
      float mr = -INFINITY;
      if ((j + 1) * AK > qt * AQ) {
        const int lim = qrow - j * AK;  // keys i <= lim are visible
#pragma unroll
        for (int i = 0; i < AK; ++i) {
          if (i > lim) sv[i] = -INFINITY;
          mr = fmaxf(mr, sv[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < AK; ++i) mr = fmaxf(mr, sv[i]);
      }
      const float mt = mr * sl2;
      const bool need = mt > m_run + RESCALE_THRESHOLD;   // includes the first tile
      const float m_new = need ? fmaxf(m_run, mt) : m_run;
      const float alpha = (m_run == -INFINITY) ? 0.f : ex2_approx(m_run - m_new);
      // P buffer sb is free once the PV product of tile j-2 is done
      if (j >= 2 && !mbar_wait(&p_free[sb], ((j - 2) >> 1) & 1, err)) { s_abort = 1; break; }
      if (__any_sync(0xffffffffu, need) && j > 0) {
        // O (TMEM) must be quiescent: wait for the PV product of tile j-1
        if (!mbar_wait(&p_free[(j - 1) & 1], ((j - 1) >> 1) & 1, err)) { s_abort = 1; break; }
        tc_fence_after();
        const float f = need ? alpha : 1.f;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          float ov[32];
          tmem_ld32(tmem + lane_off + 2 * AK + c, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= f;
          tmem_st32(tmem + lane_off + 2 * AK + c, ov);
        }
        tmem_wait_st();
      }
      if (need) {
        l_run *= alpha;
        m_run = m_new;
      }
      // probabilities -> bf16 P row (128 bytes, swizzled 16-byte chunks)
      float ls = 0.f;
      const uint32_t prow = sP + sb * L::P_BYTES + r * 128;
      const float neg_m = -m_run;
#pragma unroll
      for (int c = 0; c < AK / 8; ++c) {
        float p[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          p[i] = ex2_approx(fmaf(sv[c * 8 + i], sl2, neg_m));
          ls += p[i];
        }
        const uint32_t w0 = pack_bf16x2_rn(p[0], p[1]), w1 = pack_bf16x2_rn(p[2], p[3]);
        const uint32_t w2 = pack_bf16x2_rn(p[4], p[5]), w3 = pack_bf16x2_rn(p[6], p[7]);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(prow + ((c ^ (r & 7)) << 4)),
                     "r"(w0), "r"(w1), "r"(w2), "r"(w3)
                     : "memory");
      }
      l_run += ls;
      fence_proxy_async_smem();   // generic-proxy smem writes -> visible to the tensor core
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    // epilogue: O / l -> bf16, lse
    if (!s_abort && mbar_wait(&p_free[(n_kv - 1) & 1], ((n_kv - 1) >> 1) & 1, err)) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      uint16_t* orow = o + static_cast<int64_t>(row_base + qrow) * s.ld_o + h * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float ov[32];
        tmem_ld32(tmem + lane_off + 2 * AK + c, ov);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_bf16x2_rn(ov[i] * inv, ov[i + 1] * inv);
          w.y = pack_bf16x2_rn(ov[i + 2] * inv, ov[i + 3] * inv);
          w.z = pack_bf16x2_rn(ov[i + 4] * inv, ov[i + 5] * inv);
          w.w = pack_bf16x2_rn(ov[i + 6] * inv, ov[i + 7] * inv);
          *reinterpret_cast<uint4*>(orow + c + i) = w;
        }
      }
      lse[(static_cast<int64_t>(b) * s.nh + h) * s.T + qrow] = (m_run + log2f(l_run)) / LOG2E_F;
    } else {
      s_abort = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (s_abort) {
      if (lane == 0) {
        umma_commit(drain);
        mbar_wait(drain, 0, err);
      }
      __syncwarp();
    }
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int HD>
int launch_fwd_tc(const uint16_t* qkv, uint16_t* o, float* lse, const AttnShape& s,
                  cudaStream_t st) {
  const int64_t M = static_cast<int64_t>(s.B) * s.T;
  CUtensorMap tq, tkv;
  GLT_TRY(make_tmap_bf16(&tq, qkv, s.ld_qkv, M, s.ld_qkv, AQ));
  GLT_TRY(make_tmap_bf16(&tkv, qkv, s.ld_qkv, M, s.ld_qkv, AK));
  auto k = attn_fwd_tc_kernel<HD>;
  constexpr int smem = FwdSmem<HD>::TOTAL;
  GLT_TRY(ensure_smem_attr(reinterpret_cast<const void*>(k), smem));
  dim3 grid(s.T / AQ, s.nh, s.B);
  k<<<grid, 192, smem, st>>>(tq, tkv, o, lse, s, device_error_word());
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

// ---------------------------------------------------------------------------
// Backward.  One CTA per (128-key tile, kv head, batch) loops over the GQA
// query heads and the causal 64-query tiles ("items").  Per item, with the
// key tile's K and V resident in smem and Q/dO double-buffered:
//   S^T  = K . Q^T      dP^T = V . dO^T          (M=128 keys, N=64 q, K=128)
//   compute warps (thread = key row): P^T = exp2(S^T*scale*log2e - lse),
//     dS^T = P^T (dP^T - rowsum(dO*O)); both written bf16 to smem tiles
//   dV  += P^T . dO     dK  += dS^T . Q          (M=128 keys, N=128 d, K=64)
//   dQ^T = K^T . dS^T                            (M=128 d, N=64 q, K=128)
// Pipeline: the MMA thread issues S/dP of item i+1 before dV/dK/dQ of item
// i, so the compute warps' exponentials for item i+1 overlap the tensor
// core's work on item i.  S/dP are double-buffered in TMEM; dQ^T of item i
// lands in the S^T columns of its own buffer (consumed by then), and the
// buffer is released once the compute warps have read dQ^T out.  Each
// compute warp stages its 32 d-columns of dQ as a [64 q][32 d] fp32 tile and
// adds it into the global fp32 dQ accumulator with its own TMA bulk
// reduce-add, so no barrier spans the compute warps.
// TMEM: buffer b (b = 0, 1): S^T / dQ^T [128b, 128b+64), dP^T [128b+64,
// 128b+128); dV [256, 384); dK [384, 512).
// ---------------------------------------------------------------------------
constexpr int BK_KEYS = 128;  // keys per CTA
constexpr int BQ = 64;        // queries per item

struct BwdSmem {
  static constexpr uint32_t KV_BYTES = BK_KEYS * 128 * 2;  // [128 keys][128 d] = 2 blocks x 16 KB
  static constexpr uint32_t QD_BYTES = BQ * 128 * 2;       // [64 q][128 d] = 2 blocks x 8 KB
  static constexpr uint32_t T_BYTES = BK_KEYS * BQ * 2;    // [128 keys][64 q] bf16
  static constexpr uint32_t DQW_BYTES = BQ * 32 * 4;       // per compute warp: [64 q][32 d] fp32
  static constexpr uint32_t OFF_K = 0;
  static constexpr uint32_t OFF_V = OFF_K + KV_BYTES;
  static constexpr uint32_t OFF_Q = OFF_V + KV_BYTES;       // [2]
  static constexpr uint32_t OFF_DO = OFF_Q + 2 * QD_BYTES;  // [2]
  static constexpr uint32_t OFF_P = OFF_DO + 2 * QD_BYTES;
  static constexpr uint32_t OFF_DS = OFF_P + T_BYTES;
  static constexpr uint32_t OFF_DQ = OFF_DS + T_BYTES;      // [4 warps]
  static constexpr uint32_t OFF_LSE = OFF_DQ + 4 * DQW_BYTES;  // [4 warps][lse 64 | dsum 64]
  static constexpr uint32_t OFF_BAR = OFF_LSE + 4 * 2 * BQ * 4;
  static constexpr uint32_t NUM_BARS = 1 + 2 + 2 + 2 + 2 + 1 + 1 + 1;
  static constexpr uint32_t TOTAL = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
};

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* tm, uint32_t src, int c0,
                                                  int c1) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(tm)),
      "r"(src), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(192, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_dq, const float* __restrict__ lse,
                       const float* __restrict__ dsum, uint16_t* __restrict__ dqkv, AttnShape s,
                       unsigned int* err) {
  using L = BwdSmem;
  constexpr int HD = 128;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t COL_DV = 256, COL_DK = 384;
  constexpr uint32_t ID_SDP = make_idesc(BQ, false, false);   // M=128, N=64, K-major x K-major
  constexpr uint32_t ID_DVK = make_idesc(HD, false, true);    // M=128, N=128, A K-major, B MN-major
  constexpr uint32_t ID_DQ = make_idesc(BQ, true, true);      // M=128, N=64,  A MN, B MN
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = kv_full + 1;    // [2]
  uint64_t* qd_empty = qd_full + 2;   // [2]
  uint64_t* sdp_full = qd_empty + 2;  // [2] per TMEM buffer
  uint64_t* sdp_free = sdp_full + 2;  // [2] per TMEM buffer (dQ^T read out)
  uint64_t* p_full = sdp_free + 2;
  uint64_t* mm_done = p_full + 1;
  uint64_t* drain = mm_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ int abort_flag;
  volatile int& s_abort = abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int rep = s.nh / s.nkv;
  const int q_first = kt * (BK_KEYS / BQ);                 // first causal query tile
  const int per_head = s.T / BQ - q_first;
  const int n_items = rep * per_head;
  const int row0 = b * s.T;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
      mbar_init(&sdp_full[i], 1);
      mbar_init(&sdp_free[i], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(mm_done, 1);
    mbar_init(drain, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sK = smem_u32(sm + L::OFF_K), sV = smem_u32(sm + L::OFF_V);
  const uint32_t sQ = smem_u32(sm + L::OFF_Q), sDO = smem_u32(sm + L::OFF_DO);
  const uint32_t sP = smem_u32(sm + L::OFF_P), sDS = smem_u32(sm + L::OFF_DS);

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      const int kcol = (s.nh + kvh) * HD, vcol = (s.nh + s.nkv + kvh) * HD;
      mbar_arrive_expect_tx(kv_full, 2 * L::KV_BYTES);
      for (int c = 0; c < 2; ++c) {
        tma_load_2d(sm + L::OFF_K + c * (BK_KEYS * 128), &tm_k, kv_full, kcol + 64 * c, row0 + kt * BK_KEYS);
        tma_load_2d(sm + L::OFF_V + c * (BK_KEYS * 128), &tm_k, kv_full, vcol + 64 * c, row0 + kt * BK_KEYS);
      }
      for (int i = 0; i < n_items && !s_abort; ++i) {
        const int st = i & 1;
        const int h = kvh * rep + i / per_head, qt = q_first + i % per_head;
        if (!mbar_wait(&qd_empty[st], ((i >> 1) & 1) ^ 1, err)) { s_abort = 1; break; }
        mbar_arrive_expect_tx(&qd_full[st], 2 * L::QD_BYTES);
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(sm + L::OFF_Q + st * L::QD_BYTES + c * (BQ * 128), &tm_q, &qd_full[st],
                      h * HD + 64 * c, row0 + qt * BQ);
          tma_load_2d(sm + L::OFF_DO + st * L::QD_BYTES + c * (BQ * 128), &tm_do, &qd_full[st],
                      h * HD + 64 * c, row0 + qt * BQ);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      // S^T(j), dP^T(j) into TMEM buffer j & 1 (both operands K-major)
      auto issue_sdp = [&](int j) -> bool {
        const int st = j & 1, bf = j & 1;
        if (!mbar_wait(&qd_full[st], (j >> 1) & 1, err)) return false;
        if (!mbar_wait(&sdp_free[bf], ((j >> 1) & 1) ^ 1, err)) return false;
        tc_fence_after();
        const uint32_t qb = sQ + st * L::QD_BYTES, db = sDO + st * L::QD_BYTES;
        const uint32_t col = 128u * bf;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_bf16(tmem + col, desc_kmajor(sK + (k >> 2) * (BK_KEYS * 128), k & 3),
                    desc_kmajor(qb + (k >> 2) * (BQ * 128), k & 3), ID_SDP, k > 0);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_bf16(tmem + col + 64, desc_kmajor(sV + (k >> 2) * (BK_KEYS * 128), k & 3),
                    desc_kmajor(db + (k >> 2) * (BQ * 128), k & 3), ID_SDP, k > 0);
        umma_commit(&sdp_full[bf]);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, err);
      if (ok && n_items > 0) { tc_fence_after(); ok = issue_sdp(0); }
      for (int i = 0; ok && i < n_items; ++i) {
        if (i + 1 < n_items && !issue_sdp(i + 1)) { ok = false; break; }
        const int st = i & 1;
        if (!mbar_wait(p_full, i & 1, err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qb = sQ + st * L::QD_BYTES, db = sDO + st * L::QD_BYTES;
#pragma unroll
        for (int k = 0; k < BQ / 16; ++k) {
          umma_bf16(tmem + COL_DV, desc_kmajor(sP, k), desc_mnmajor(db, k), ID_DVK, (i > 0 || k > 0));
          umma_bf16(tmem + COL_DK, desc_kmajor(sDS, k), desc_mnmajor(qb, k), ID_DVK, (i > 0 || k > 0));
        }
        // dQ^T = K^T . dS^T into the (consumed) S^T columns of buffer i & 1:
        // A = K tile read MN-major (d contiguous, 16 KB between d blocks),
        // B = dS^T tile read MN-major (q contiguous)
#pragma unroll
        for (int k = 0; k < BK_KEYS / 16; ++k)
          umma_bf16(tmem + 128u * (i & 1), make_sdesc(sK + k * (UMMA_K * 128), BK_KEYS * 128, 1024),
                    make_sdesc(sDS + k * (UMMA_K * 128), 8192, 1024), ID_DQ, k > 0);
        umma_commit(mm_done);
        umma_commit(&qd_empty[st]);
      }
      if (!ok) s_abort = 1;
    }
  } else {
    // ------------------------------- compute ------------------------------
    const int sub = warp & 3;
    const int r = sub * 32 + lane;                  // key row (TMEM lane); for dQ^T: d index
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const float sl2 = s.scale * LOG2E_F;
    const int key = kt * BK_KEYS + r;
    float* w_ls = reinterpret_cast<float*>(sm + L::OFF_LSE) + sub * 2 * BQ;  // this warp's lse | dsum
    float* w_dq = reinterpret_cast<float*>(sm + L::OFF_DQ + sub * L::DQW_BYTES);
    const uint32_t sDQW = smem_u32(w_dq);
    // lse / dsum of item i, prefetched one item ahead (lane holds q = lane, 32 + lane)
    auto lse_index = [&](int i, int q) -> int64_t {
      const int h = kvh * rep + i / per_head, qt = q_first + i % per_head;
      return (static_cast<int64_t>(b) * s.nh + h) * s.T + qt * BQ + q;
    };
    float pl0 = 0.f, pl1 = 0.f, pd0 = 0.f, pd1 = 0.f;
    if (n_items > 0) {
      pl0 = lse[lse_index(0, lane)];
      pl1 = lse[lse_index(0, 32 + lane)];
      pd0 = dsum[lse_index(0, lane)];
      pd1 = dsum[lse_index(0, 32 + lane)];
    }
    // dQ of item j: TMEM -> this warp's [64 q][32 d] tile -> TMA reduce-add
    auto flush_dq = [&](int j) -> bool {
      if (!mbar_wait(mm_done, j & 1, err)) return false;
      tc_fence_after();
      float t0[32], t1[32];
      tmem_ld32(tmem + lane_off + 128u * (j & 1), t0);
      tmem_ld32(tmem + lane_off + 128u * (j & 1) + 32, t1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sdp_free[j & 1]);
        bulk_wait_read0();                          // this warp's previous reduce has read its tile
      }
      __syncwarp();
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        w_dq[q * 32 + lane] = t0[q] * s.scale;
        w_dq[(32 + q) * 32 + lane] = t1[q] * s.scale;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int h = kvh * rep + j / per_head, qt = q_first + j % per_head;
        tma_reduce_add_2d(&tm_dq, sDQW, h * HD + sub * 32, row0 + qt * BQ);
        bulk_commit();
      }
      return true;
    };
    bool ok = true;
    for (int i = 0; i < n_items; ++i) {
      const int qt = q_first + i % per_head;
      // this item's lse*log2e and dsum -> warp-private smem; prefetch the next item's
      w_ls[lane] = pl0 * LOG2E_F;
      w_ls[32 + lane] = pl1 * LOG2E_F;
      w_ls[BQ + lane] = pd0;
      w_ls[BQ + 32 + lane] = pd1;
      __syncwarp();
      if (i + 1 < n_items) {
        pl0 = lse[lse_index(i + 1, lane)];
        pl1 = lse[lse_index(i + 1, 32 + lane)];
        pd0 = dsum[lse_index(i + 1, lane)];
        pd1 = dsum[lse_index(i + 1, 32 + lane)];
      }
      if (!mbar_wait(&sdp_full[i & 1], (i >> 1) & 1, err)) { ok = false; break; }
      tc_fence_after();
      uint32_t pw[BQ / 2], dw[BQ / 2];   // P^T and dS^T rows, packed bf16 pairs
      {
        const uint32_t col = 128u * (i & 1);
        float sv[32], dv[32];
        const bool diag = qt * BQ < (kt + 1) * BK_KEYS;
        const int lim = key - qt * BQ;  // causal: query qt*BQ + c sees this key iff c >= lim
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          tmem_ld32(tmem + lane_off + col + 32 * half, sv);
          tmem_ld32(tmem + lane_off + col + 64 + 32 * half, dv);
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const int q = 32 * half + c;
            const float4 l2 = *reinterpret_cast<const float4*>(w_ls + (q & ~3));
            const float4 d2 = *reinterpret_cast<const float4*>(w_ls + BQ + (q & ~3));
            const float la = (q & 3) == 0 ? l2.x : l2.z, lb = (q & 3) == 0 ? l2.y : l2.w;
            const float da = (q & 3) == 0 ? d2.x : d2.z, db = (q & 3) == 0 ? d2.y : d2.w;
            float p0 = ex2_approx(fmaf(sv[c], sl2, -la));
            float p1 = ex2_approx(fmaf(sv[c + 1], sl2, -lb));
            if (diag) {
              if (q < lim) p0 = 0.f;
              if (q + 1 < lim) p1 = 0.f;
            }
            pw[q >> 1] = pack_bf16x2_rn(p0, p1);
            dw[q >> 1] = pack_bf16x2_rn(p0 * (dv[c] - da), p1 * (dv[c + 1] - db));
          }
        }
      }
      // S^T/dP^T are in registers; dQ of the previous item frees its buffer
      if (i > 0 && !flush_dq(i - 1)) { ok = false; break; }
      // P^T and dS^T rows -> 128-byte swizzled smem rows (the previous item's
      // tiles are free: its mm_done was waited in flush_dq)
#pragma unroll
      for (int c = 0; c < BQ / 8; ++c) {
        const uint32_t off = r * 128 + ((c ^ (r & 7)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(sP + off), "r"(pw[4 * c]),
                     "r"(pw[4 * c + 1]), "r"(pw[4 * c + 2]), "r"(pw[4 * c + 3])
                     : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(sDS + off), "r"(dw[4 * c]),
                     "r"(dw[4 * c + 1]), "r"(dw[4 * c + 2]), "r"(dw[4 * c + 3])
                     : "memory");
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && n_items > 0) ok = flush_dq(n_items - 1);
    if (ok && n_items > 0) {
      // dK (scaled) and dV rows of this CTA's keys (mm_done of the last item was waited)
      uint16_t* krow = dqkv + static_cast<int64_t>(row0 + key) * s.ld_qkv + (s.nh + kvh) * HD;
      uint16_t* vrow = dqkv + static_cast<int64_t>(row0 + key) * s.ld_qkv + (s.nh + s.nkv + kvh) * HD;
#pragma unroll 1
      for (int c0 = 0; c0 < HD; c0 += 32) {
        float t[32];
        tmem_ld32(tmem + lane_off + COL_DV + c0, t);
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          uint4 w;
          w.x = pack_bf16x2_rn(t[c], t[c + 1]); w.y = pack_bf16x2_rn(t[c + 2], t[c + 3]);
          w.z = pack_bf16x2_rn(t[c + 4], t[c + 5]); w.w = pack_bf16x2_rn(t[c + 6], t[c + 7]);
          *reinterpret_cast<uint4*>(vrow + c0 + c) = w;
        }
        tmem_ld32(tmem + lane_off + COL_DK + c0, t);
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          uint4 w;
          w.x = pack_bf16x2_rn(t[c] * s.scale, t[c + 1] * s.scale);
          w.y = pack_bf16x2_rn(t[c + 2] * s.scale, t[c + 3] * s.scale);
          w.z = pack_bf16x2_rn(t[c + 4] * s.scale, t[c + 5] * s.scale);
          w.w = pack_bf16x2_rn(t[c + 6] * s.scale, t[c + 7] * s.scale);
          *reinterpret_cast<uint4*>(krow + c0 + c) = w;
        }
      }
    }
    if (!ok) s_abort = 1;
    if (lane == 0) bulk_wait0();   // this warp's reduce-adds complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    if (s_abort) {
      if (lane == 0) {
        umma_commit(drain);
        mbar_wait(drain, 0, err);
      }
      __syncwarp();
    }
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

int flash_bwd_tc(const uint16_t* qkv, const uint16_t* o, const uint16_t* dout, const float* lse,
                 uint16_t* dqkv, float* dq_acc, float* dsum, const AttnShape& s, cudaStream_t st) {
  if (s.hd != 128) return fail(GLT_EINVAL, "attention backward (tcgen05): head_dim must be 128");
  if (s.T % BK_KEYS) return fail(GLT_EINVAL, "attention backward (tcgen05): seq_len %% 128 != 0");
  if (s.nkv <= 0 || s.nh % s.nkv) return fail(GLT_EINVAL, "attention: nh %% nkv != 0");
  if (s.ld_qkv % 8 || s.ld_o % 8) return fail(GLT_EINVAL, "attention: strides not 16-byte");
  GLT_TRY(attn_bwd_prep(o, dout, dq_acc, dsum, s, st));
  const int64_t M = static_cast<int64_t>(s.B) * s.T;
  CUtensorMap tk, tq, tdo, tdq;
  GLT_TRY(make_tmap_bf16(&tk, qkv, s.ld_qkv, M, s.ld_qkv, BK_KEYS));
  GLT_TRY(make_tmap_bf16(&tq, qkv, s.ld_qkv, M, s.ld_qkv, BQ));
  GLT_TRY(make_tmap_bf16(&tdo, dout, s.ld_o, M, s.ld_o, BQ));
  GLT_TRY(make_tmap_f32_plain(&tdq, dq_acc, static_cast<uint64_t>(s.nh) * s.hd, M,
                              static_cast<uint64_t>(s.nh) * s.hd, 32, BQ));
  constexpr int smem = BwdSmem::TOTAL;
  GLT_TRY(ensure_smem_attr(reinterpret_cast<const void*>(attn_bwd_tc_kernel), smem));
  dim3 grid(s.T / BK_KEYS, s.nkv, s.B);
  attn_bwd_tc_kernel<<<grid, 192, smem, st>>>(tk, tq, tdo, tdq, lse, dsum, dqkv, s,
                                              device_error_word());
  GLT_LAUNCH_CHECK();
  return attn_bwd_finish(dq_acc, dqkv, s, st);
}

int flash_fwd_tc(const uint16_t* qkv, uint16_t* o, float* lse, const AttnShape& s,
                 cudaStream_t st) {
  if (s.hd != 64 && s.hd != 128) return fail(GLT_EINVAL, "attention: head_dim %d unsupported", s.hd);
  if (s.T % AQ) return fail(GLT_EINVAL, "attention (tcgen05): seq_len %d not a multiple of 128", s.T);
  if (s.nkv <= 0 || s.nh % s.nkv) return fail(GLT_EINVAL, "attention: nh %% nkv != 0");
  if (s.ld_qkv % 8 || s.ld_o % 8) return fail(GLT_EINVAL, "attention: strides not 16-byte");
  return s.hd == 128 ? launch_fwd_tc<128>(qkv, o, lse, s, st) : launch_fwd_tc<64>(qkv, o, lse, s, st);
}

}  // namespace glt
