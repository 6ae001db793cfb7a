// Causal GQA flash-attention forward on the 5th-generation tensor cores.
//
// One CTA per (128-query tile, head, batch), two CTAs resident per SM so that
// one CTA's barrier round trips, prologue and epilogue overlap the other's
// tensor-core work; 6 warps:
//   warp 0      TMA producer: the Q tile once, then 64-key K and V tiles into
//               two 2-stage rings (128B swizzle, plain per-CTA loads).  A K
//               stage is released as soon as its S product completes, a V
//               stage after its PV product.
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer:
//                 S_j = Q.K_j^T   (M=128, N=64,  K=hd; A, B from smem, K-major)
//                 O  += P_j.V_j   (M=128, N=hd,  K=64; A = P from TMEM,
//                                  B = V from smem, MN-major)
//               S_{j+1} is issued before O += P_j.V_j so the softmax of tile j
//               overlaps the next QK^T.
//   warps 2..5  softmax: thread i owns query row i (= TMEM lane i); reads its
//               S row with tcgen05.ld, keeps the running max / sum, and writes
//               the bf16 probabilities back over the first 32 columns of the
//               same S buffer with tcgen05.st, where the PV product reads them
//               as its A operand (no shared-memory round trip for P).
// TMEM (256 columns): S/P buffers 0 and 1 (64 columns each) + O (hd columns).
// An S/P buffer is reused for S_{j+2} only after the PV product that read P_j
// from it has completed (its commit), so no tensor-core ordering is assumed.
// The O rescale of online softmax is conditional: the running max used for
// the exponentials only moves when a row's max grows by more than 2^8, so the
// O read-modify-write in TMEM (which must wait for the previous PV product)
// is rare; p = exp2(s - m) stays <= 256, well inside fp32/bf16 range, and the
// final normalisation uses the same m for O and the row sum.
// All mbarrier waits are bounded (tc::mbar_wait); a timeout sets the device
// error word and the CTA's abort flag, the other roles give up their waits,
// and the CTA waits (bounded) for its loads in flight and its issued MMAs
// before it frees TMEM and exits, instead of hanging.
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
constexpr int K_STAGES = 2;
constexpr int V_STAGES = 2;
constexpr float LOG2E_F = 1.4426950408889634f;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]),
      "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]),
      "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  uint32_t u[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(v[i]);
  tmem_st32(taddr, u);
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
// D (TMEM) (+)= A (TMEM) . B (smem descriptor), kind::f16, one CTA.  A is
// M=128 lanes x K=16 bf16, two elements per 32-bit column (8 columns).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

template <int HD>
struct FwdSmem {
  static constexpr uint32_t Q_BYTES = AQ * HD * 2;          // HD/64 blocks of [128 x 128B]
  static constexpr uint32_t K_BYTES = AK * HD * 2;          // HD/64 blocks of [64 x 128B]
  static constexpr uint32_t V_BYTES = AK * HD * 2;          // HD/64 chunks of [64 x 128B]
  static constexpr uint32_t OFF_Q = 0;
  static constexpr uint32_t OFF_K = OFF_Q + Q_BYTES;
  static constexpr uint32_t OFF_V = OFF_K + K_STAGES * K_BYTES;
  static constexpr uint32_t OFF_BAR = OFF_V + V_STAGES * V_BYTES;
  static constexpr uint32_t NUM_BARS = 1 + 2 * K_STAGES + 2 * V_STAGES + 2 + 2 + 2 + 1;
  static constexpr uint32_t TOTAL = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
};
// two CTAs per SM (228 KB of shared memory per SM, 1 KB reserved per CTA)
static_assert(2 * (FwdSmem<128>::TOTAL + 1024) <= 233472, "attention forward: two CTAs do not fit");

constexpr int FWD_THREADS = 192;   // producer, MMA, 4 softmax warps

template <int HD>
__global__ void __launch_bounds__(FWD_THREADS, 2)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_kv, uint16_t* __restrict__ o,
                       float* __restrict__ lse, AttnShape s, unsigned int* err) {
  using L = FwdSmem<HD>;
  constexpr uint32_t TMEM_COLS = 256;   // S/P 0 | S/P 1 | O (HD <= 128)
  constexpr uint32_t COL_O = 2 * AK;
  constexpr uint32_t ID_S = make_idesc(AK, false, false);
  constexpr uint32_t ID_PV = make_idesc(HD, false, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;
  uint64_t* k_empty = k_full + K_STAGES;
  uint64_t* v_full = k_empty + K_STAGES;
  uint64_t* v_empty = v_full + V_STAGES;
  uint64_t* s_full = v_empty + V_STAGES;    // [2]  S_j in buffer j & 1
  uint64_t* p_full = s_full + 2;            // [2]  P_j written over it
  uint64_t* p_free = p_full + 2;            // [2]  PV_j done: buffer reusable, O quiescent
  uint64_t* drain = p_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ int abort_flag;
  volatile int& s_abort = abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // x = query tile, heaviest first within each (head, batch): CTAs that run
  // together share one head's K/V in L2
  const int qt = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (s.nh / s.nkv);
  const int n_kv = (qt * AQ + AQ) / AK;        // causal: keys < (qt+1)*128
  const int row_base = b * s.T;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < K_STAGES; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1); }
    for (int i = 0; i < V_STAGES; ++i) { mbar_init(&v_full[i], 1); mbar_init(&v_empty[i], 1); }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
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
  int nk = 0, nv = 0;   // K and V tiles the producer issued (read on the abort path)

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      const int qcol = h * HD, kcol = (s.nh + kvh) * HD, vcol = (s.nh + s.nkv + kvh) * HD;
      mbar_arrive_expect_tx(q_full, L::Q_BYTES);
#pragma unroll
      for (int c = 0; c < HD / 64; ++c)
        tma_load_2d(sm + L::OFF_Q + c * (AQ * 128), &tm_q, q_full, qcol + 64 * c, row_base + qt * AQ);
      for (int j = 0; j < n_kv && !s_abort; ++j) {
        const int ks = j % K_STAGES, vs = j % V_STAGES;
        if (!mbar_wait(&k_empty[ks], ((j / K_STAGES) & 1) ^ 1, err, &s_abort)) { s_abort = 1; break; }
        mbar_arrive_expect_tx(&k_full[ks], L::K_BYTES);
        uint8_t* kb = sm + L::OFF_K + ks * L::K_BYTES;
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(kb + c * (AK * 128), &tm_kv, &k_full[ks], kcol + 64 * c, row_base + j * AK);
        nk = j + 1;
        if (!mbar_wait(&v_empty[vs], ((j / V_STAGES) & 1) ^ 1, err, &s_abort)) { s_abort = 1; break; }
        mbar_arrive_expect_tx(&v_full[vs], L::V_BYTES);
        uint8_t* vb = sm + L::OFF_V + vs * L::V_BYTES;
#pragma unroll
        for (int c = 0; c < HD / 64; ++c)
          tma_load_2d(vb + c * (AK * 128), &tm_kv, &v_full[vs], vcol + 64 * c, row_base + j * AK);
        nv = j + 1;
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      auto issue_s = [&](int j) -> bool {
        const int ks = j % K_STAGES, sb = j & 1;
        if (!mbar_wait(&k_full[ks], (j / K_STAGES) & 1, err, &s_abort)) return false;
        // buffer sb last held P_{j-2}: wait until PV_{j-2} has read it
        if (!mbar_wait(&p_free[sb], ((j >> 1) & 1) ^ 1, err, &s_abort)) return false;
        tc_fence_after();
        const uint32_t kb = sK + ks * L::K_BYTES;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const uint64_t ad = desc_kmajor(sQ + (k >> 2) * (AQ * 128), k & 3);
          const uint64_t bd = desc_kmajor(kb + (k >> 2) * (AK * 128), k & 3);
          umma_bf16(tmem + sb * AK, ad, bd, ID_S, k > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[ks]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, err, &s_abort);
      if (ok) { tc_fence_after(); ok = issue_s(0); }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j + 1 < n_kv && !issue_s(j + 1)) { ok = false; break; }
        const int sb = j & 1, vs = j % V_STAGES;
        if (!mbar_wait(&v_full[vs], (j / V_STAGES) & 1, err, &s_abort)) { ok = false; break; }
        if (!mbar_wait(&p_full[sb], (j >> 1) & 1, err, &s_abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t vb = sV + vs * L::V_BYTES;
#pragma unroll
        for (int k = 0; k < AK / 16; ++k)
          umma_bf16_ts(tmem + COL_O, tmem + sb * AK + 8 * k, desc_mnmajor(vb, k), ID_PV,
                       (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(&p_free[sb]);
        umma_commit(&v_empty[vs]);
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
      if (!mbar_wait(&s_full[sb], (j >> 1) & 1, err, &s_abort)) { s_abort = 1; break; }
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
      // causal mask (diagonal tiles only) + max of the raw scores (four
      // independent chains); the scale is positive, so it is applied to the
      // max and folded into the exponent's FFMA below
      if ((j + 1) * AK > qt * AQ) {
        const int lim = qrow - j * AK;  // keys i <= lim are visible
#pragma unroll
        for (int i = 0; i < AK; ++i)
          if (i > lim) sv[i] = -INFINITY;
      }
      float m4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int i = 4; i < AK; ++i) m4[i & 3] = fmaxf(m4[i & 3], sv[i]);
      const float mt = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * sl2;
      const bool need = mt > m_run + RESCALE_THRESHOLD;   // includes the first tile
      const float m_new = need ? fmaxf(m_run, mt) : m_run;
      const float alpha = (m_run == -INFINITY) ? 0.f : ex2_approx(m_run - m_new);
      if (__any_sync(0xffffffffu, need) && j > 0) {
        // O (TMEM) must be quiescent: wait for the PV product of tile j-1
        if (!mbar_wait(&p_free[(j - 1) & 1], ((j - 1) >> 1) & 1, err, &s_abort)) { s_abort = 1; break; }
        tc_fence_after();
        const float f = need ? alpha : 1.f;
#pragma unroll 1
        for (int c = 0; c < HD; c += 32) {
          float ov[32];
          tmem_ld32(tmem + lane_off + COL_O + c, ov);
#pragma unroll
          for (int i = 0; i < 32; ++i) ov[i] *= f;
          tmem_st32(tmem + lane_off + COL_O + c, ov);
        }
        tmem_wait_st();
      }
      if (need) {
        l_run *= alpha;
        m_run = m_new;
      }
      // probabilities -> 32 packed bf16 pairs over columns [0, 32) of this S buffer
      float ls4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pw[AK / 2];
      const float neg_m = -m_run;
#pragma unroll
      for (int i = 0; i < AK; i += 2) {
        const float p0 = ex2_approx(fmaf(sv[i], sl2, neg_m));
        const float p1 = ex2_approx(fmaf(sv[i + 1], sl2, neg_m));
        ls4[i & 3] += p0;
        ls4[(i + 1) & 3] += p1;
        pw[i >> 1] = pack_bf16x2_rn(p0, p1);
      }
      l_run += (ls4[0] + ls4[1]) + (ls4[2] + ls4[3]);
      tmem_st32(tmem + lane_off + sb * AK, pw);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
    }
    // epilogue: O / l -> bf16, lse
    if (!s_abort && mbar_wait(&p_free[(n_kv - 1) & 1], ((n_kv - 1) >> 1) & 1, err, &s_abort)) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      uint16_t* orow = o + static_cast<int64_t>(row_base + qrow) * s.ld_o + h * HD;
#pragma unroll 1
      for (int c = 0; c < HD; c += 32) {
        float ov[32];
        tmem_ld32(tmem + lane_off + COL_O + c, ov);
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
  if (warp == 0 && lane == 0 && s_abort) {
    // loads still in flight land before the CTA exits (bounded waits on the
    // last arming of every buffer)
    mbar_wait(q_full, 0, err, nullptr);
    for (int d = 0; d < K_STAGES && d < nk; ++d)
      mbar_wait(&k_full[(nk - 1 - d) % K_STAGES], ((nk - 1 - d) / K_STAGES) & 1, err, nullptr);
    for (int d = 0; d < V_STAGES && d < nv; ++d)
      mbar_wait(&v_full[(nv - 1 - d) % V_STAGES], ((nv - 1 - d) / V_STAGES) & 1, err, nullptr);
  }
  if (warp == 1) {
    tc_fence_after();
    if (s_abort) {
      if (lane == 0) {
        umma_commit(drain);
        mbar_wait(drain, 0, err, nullptr);
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
  // two CTAs per SM need the full shared-memory carveout (a per-device setting)
  GLT_TRY(ensure_smem_carveout_max(reinterpret_cast<const void*>(k)));
  dim3 grid(s.T / AQ, s.nh, s.B);
  k<<<grid, FWD_THREADS, smem, st>>>(tq, tkv, o, lse, s, device_error_word());
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
// Pipeline: S/dP live in one TMEM buffer that the compute warps release as
// soon as they have loaded item i into registers, so the MMA thread issues
// S/dP of item i+1 while the warps are still computing item i, and those
// products run ahead of dV/dK/dQ of item i on the tensor core.  dQ^T gets
// two TMEM buffers of its own: item i writes buffer i & 1, which the warps
// drain during item i+1 and which item i+2 reuses, so draining dQ never
// holds up the next item's S/dP.
// Eight compute warps, two per TMEM lane quarter: warp (quarter, half) owns
// key rows [32 quarter, +32) and query columns [32 half, +32) of each item
// (the backward has no reduction over queries, so the halves never talk).
// Each stages its [32 q][32 d] block of dQ and adds it into the global fp32
// dQ accumulator with its own TMA bulk reduce-add.
// TMEM: S^T [0, 64), dP^T [64, 128); dQ^T buffers [128, 192), [192, 256);
// dV [256, 384); dK [384, 512).
// ---------------------------------------------------------------------------
constexpr int BK_KEYS = 128;  // keys per CTA
constexpr int BQ = 64;        // queries per item
// Q/dO ring depth.  A stage is released only when all five products of its
// item are done, so with two stages the load of item i+2 starts when item i
// finishes and its latency lands on every item; three stages hide it.
#ifndef GLT_ATTN_QD_STAGES
#define GLT_ATTN_QD_STAGES 3
#endif
constexpr int QD_STAGES = GLT_ATTN_QD_STAGES;

struct BwdSmem {
  static constexpr uint32_t KV_BYTES = BK_KEYS * 128 * 2;  // [128 keys][128 d] = 2 blocks x 16 KB
  static constexpr uint32_t QD_BYTES = BQ * 128 * 2;       // [64 q][128 d] = 2 blocks x 8 KB
  static constexpr uint32_t T_BYTES = BK_KEYS * BQ * 2;    // [128 keys][64 q] bf16
  static constexpr uint32_t DQW_BYTES = 32 * 32 * 4;       // one [32 q][32 d] fp32 staging block
  static constexpr uint32_t OFF_K = 0;
  static constexpr uint32_t OFF_V = OFF_K + KV_BYTES;
  static constexpr uint32_t OFF_Q = OFF_V + KV_BYTES;                // [QD_STAGES]
  static constexpr uint32_t OFF_DO = OFF_Q + QD_STAGES * QD_BYTES;   // [QD_STAGES]
  static constexpr uint32_t OFF_P = OFF_DO + QD_STAGES * QD_BYTES;
  static constexpr uint32_t OFF_DS = OFF_P + T_BYTES;
  static constexpr uint32_t OFF_DQ = OFF_DS + T_BYTES;      // [4 dQ warps][2 blocks]
  static constexpr uint32_t OFF_BAR = OFF_DQ + 8 * DQW_BYTES;
  static constexpr uint32_t NUM_BARS = 1 + 2 * QD_STAGES + 1 + 1 + 2 + 1 + 1 + 2 + 2;
  static constexpr uint32_t TOTAL = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
};
static_assert(BwdSmem::TOTAL <= 232448, "attention backward: shared memory over 227 KB");

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

// producer, two MMA issuers (S/dP; dV/dK/dQ), 8 compute warps, 4 dQ warps.
// An MMA thread stalls ~200 cycles on every mbarrier wait it depends on, and
// the tensor pipe holds about one instruction ahead, so a single issuer
// waiting between N=64 products leaves the pipe idle for most of each wait;
// with two issuers one keeps the pipe fed while the other waits.  The dQ
// warps drain dQ^T from TMEM into the global accumulator, which keeps that
// work (a third of the compute warps' time per item) off the chain
// S/dP -> P/dS -> dV/dK/dQ^T -> next item's P/dS.
constexpr int BWD_THREADS = 480;
constexpr int BWD_FIRST_DQ_WARP = 11;

__global__ void __launch_bounds__(BWD_THREADS, 1)
    attn_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_q,
                       const __grid_constant__ CUtensorMap tm_do,
                       const __grid_constant__ CUtensorMap tm_dq, const float* __restrict__ lse,
                       const float* __restrict__ dsum, uint16_t* __restrict__ dqkv, AttnShape s,
                       unsigned int* err) {
  using L = BwdSmem;
  constexpr int HD = 128;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t COL_S = 0, COL_DP = 64, COL_DQ = 128, COL_DV = 256, COL_DK = 384;
  constexpr uint32_t ID_SDP = make_idesc(BQ, false, false);   // M=128, N=64, K-major x K-major
  constexpr uint32_t ID_DVK = make_idesc(HD, false, true);    // M=128, N=128, A K-major, B MN-major
  constexpr uint32_t ID_DQ = make_idesc(BQ, true, true);      // M=128, N=64,  A MN, B MN
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = kv_full + 1;            // [QD_STAGES]
  uint64_t* qd_empty = qd_full + QD_STAGES;   // [QD_STAGES]
  uint64_t* sdp_full = qd_empty + QD_STAGES;  // S/dP of the current item in TMEM
  uint64_t* sdp_free = sdp_full + 1;          // ... loaded into the warps' registers
  uint64_t* dq_free = sdp_free + 1;           // [2] dQ^T buffer drained
  uint64_t* p_full = dq_free + 2;
  uint64_t* mm_done = p_full + 1;
  uint64_t* drain = mm_done + 1;              // [2] abort-path drain of each issuer
  uint64_t* dq_full = drain + 2;              // [2] dQ^T of item i in buffer i & 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(dq_full + 2);
  __shared__ int abort_flag;
  volatile int& s_abort = abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // x = key tile, heaviest (kt = 0) first within each (kv head, batch): CTAs
  // that run together share that group's Q and dO in L2
  const int kt = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int rep = s.nh / s.nkv;
  const int q_first = kt * (BK_KEYS / BQ);                 // first causal query tile
  const int per_head = s.T / BQ - q_first;
  const int n_items = rep * per_head;
  const int row0 = b * s.T;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < QD_STAGES; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(sdp_full, 1);
    mbar_init(sdp_free, 8);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dq_free[i], 4);   // the 4 dQ warps
      mbar_init(&dq_full[i], 1);
    }
    mbar_init(p_full, 8);
    mbar_init(mm_done, 1);
    mbar_init(&drain[0], 1);
    mbar_init(&drain[1], 1);
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
  int issued = 0;   // Q/dO items the producer issued (read on the abort path)

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
        const int st = i % QD_STAGES;
        const int h = kvh * rep + i / per_head, qt = q_first + i % per_head;
        if (!mbar_wait(&qd_empty[st], ((i / QD_STAGES) & 1) ^ 1, err, &s_abort)) { s_abort = 1; break; }
        mbar_arrive_expect_tx(&qd_full[st], 2 * L::QD_BYTES);
        for (int c = 0; c < 2; ++c) {
          tma_load_2d(sm + L::OFF_Q + st * L::QD_BYTES + c * (BQ * 128), &tm_q, &qd_full[st],
                      h * HD + 64 * c, row0 + qt * BQ);
          tma_load_2d(sm + L::OFF_DO + st * L::QD_BYTES + c * (BQ * 128), &tm_do, &qd_full[st],
                      h * HD + 64 * c, row0 + qt * BQ);
        }
        issued = i + 1;
      }
    }
  } else if (warp == 1) {
    // ------------------------- MMA issuer: S^T, dP^T -------------------------
    if (lane == 0) {
      // S^T(j), dP^T(j) into TMEM columns [0, 128) (both operands K-major),
      // once the warps have loaded item j-1's S/dP
      auto issue_sdp = [&](int j) -> bool {
        const int st = j % QD_STAGES;
        if (!mbar_wait(&qd_full[st], (j / QD_STAGES) & 1, err, &s_abort)) return false;
        if (j > 0 && !mbar_wait(sdp_free, (j - 1) & 1, err, &s_abort)) return false;
        tc_fence_after();
        const uint32_t qb = sQ + st * L::QD_BYTES, db = sDO + st * L::QD_BYTES;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_bf16(tmem + COL_S, desc_kmajor(sK + (k >> 2) * (BK_KEYS * 128), k & 3),
                    desc_kmajor(qb + (k >> 2) * (BQ * 128), k & 3), ID_SDP, k > 0);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_bf16(tmem + COL_DP, desc_kmajor(sV + (k >> 2) * (BK_KEYS * 128), k & 3),
                    desc_kmajor(db + (k >> 2) * (BQ * 128), k & 3), ID_SDP, k > 0);
        umma_commit(sdp_full);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, err, &s_abort);
      if (ok) tc_fence_after();
      for (int i = 0; ok && i < n_items; ++i) ok = issue_sdp(i);
      if (!ok) s_abort = 1;
    }
  } else if (warp == 2) {
    // ----------------------- MMA issuer: dV, dK, dQ^T -----------------------
    // Item i's S/dP are complete before its P^T/dS^T exist (the compute warps
    // waited on sdp_full), so this issuer's commit after dQ^T(i) also covers
    // every product that read Q/dO stage i.
    if (lane == 0) {
      bool ok = mbar_wait(kv_full, 0, err, &s_abort);
      for (int i = 0; ok && i < n_items; ++i) {
        const int st = i % QD_STAGES;
        if (!mbar_wait(p_full, i & 1, err, &s_abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qb = sQ + st * L::QD_BYTES, db = sDO + st * L::QD_BYTES;
#pragma unroll
        for (int k = 0; k < BQ / 16; ++k) {
          umma_bf16(tmem + COL_DV, desc_kmajor(sP, k), desc_mnmajor(db, k), ID_DVK, (i > 0 || k > 0));
          umma_bf16(tmem + COL_DK, desc_kmajor(sDS, k), desc_mnmajor(qb, k), ID_DVK, (i > 0 || k > 0));
        }
        // dQ^T = K^T . dS^T into dQ buffer i & 1, drained (item i-2) by now:
        // A = K tile read MN-major (d contiguous, 16 KB between d blocks),
        // B = dS^T tile read MN-major (q contiguous)
        if (!mbar_wait(&dq_free[i & 1], ((i >> 1) & 1) ^ 1, err, &s_abort)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < BK_KEYS / 16; ++k)
          umma_bf16(tmem + COL_DQ + 64u * (i & 1), make_sdesc(sK + k * (UMMA_K * 128), BK_KEYS * 128, 1024),
                    make_sdesc(sDS + k * (UMMA_K * 128), 8192, 1024), ID_DQ, k > 0);
        umma_commit(&dq_full[i & 1]);
        umma_commit(mm_done);
        umma_commit(&qd_empty[st]);
      }
      if (!ok) s_abort = 1;
    }
  } else if (warp >= BWD_FIRST_DQ_WARP) {
    // -------------------------------- dQ warps --------------------------------
    // warp (quarter) drains d rows [32 quarter, +32) of dQ^T for all 64 queries
    // of each item: TMEM -> two [32 q][32 d] fp32 blocks -> TMA reduce-adds.
    // dQ^T(i + 2) reuses buffer i & 1 only after these warps released it, so
    // dq_full never runs two phases ahead of them.
    const int sub = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    float* stg = reinterpret_cast<float*>(sm + L::OFF_DQ + (warp - BWD_FIRST_DQ_WARP) * 2 * L::DQW_BYTES);
    const uint32_t s_stg = smem_u32(stg);
    bool ok = true;
    for (int j = 0; j < n_items; ++j) {
      if (!mbar_wait(&dq_full[j & 1], (j >> 1) & 1, err, &s_abort)) { ok = false; break; }
      tc_fence_after();
      float t0[32], t1[32];
      tmem_ld32(tmem + lane_off + COL_DQ + 64u * (j & 1), t0);
      tmem_ld32(tmem + lane_off + COL_DQ + 64u * (j & 1) + 32, t1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&dq_free[j & 1]);
        bulk_wait_read0();                          // the previous item's reduces have read the blocks
      }
      __syncwarp();
#pragma unroll
      for (int q = 0; q < 32; ++q) {
        stg[q * 32 + lane] = t0[q] * s.scale;
        stg[1024 + q * 32 + lane] = t1[q] * s.scale;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int h = kvh * rep + j / per_head, qt = q_first + j % per_head;
        tma_reduce_add_2d(&tm_dq, s_stg, h * HD + sub * 32, row0 + qt * BQ);
        tma_reduce_add_2d(&tm_dq, s_stg + L::DQW_BYTES, h * HD + sub * 32, row0 + qt * BQ + 32);
        bulk_commit();
      }
    }
    if (!ok) s_abort = 1;
    if (lane == 0) bulk_wait0();   // this warp's reduce-adds complete before the CTA exits
  } else {
    // ------------------------------- compute ------------------------------
    const int sub = warp & 3;                       // TMEM lane quarter
    const int half = (warp - 3) >> 2;               // query columns [32 half, 32 half + 32)
    const int r = sub * 32 + lane;                  // key row (TMEM lane); for dQ^T: d index
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const float sl2 = s.scale * LOG2E_F;
    const int key = kt * BK_KEYS + r;
    // lse / dsum of item i for query 32 half + lane (held by that lane and
    // broadcast by shuffle), prefetched one item ahead
    auto lse_index = [&](int i) -> int64_t {
      const int h = kvh * rep + i / per_head, qt = q_first + i % per_head;
      return (static_cast<int64_t>(b) * s.nh + h) * s.T + qt * BQ + 32 * half + lane;
    };
    float pl = 0.f, pd = 0.f;
    if (n_items > 0) {
      pl = lse[lse_index(0)];
      pd = dsum[lse_index(0)];
    }
    bool ok = true;
    for (int i = 0; i < n_items; ++i) {
      const int qt = q_first + i % per_head;
      // this item's lse*log2e and dsum; prefetch the next item's
      const float cl = pl * LOG2E_F, cd = pd;
      if (i + 1 < n_items) {
        pl = lse[lse_index(i + 1)];
        pd = dsum[lse_index(i + 1)];
      }
      if (!mbar_wait(sdp_full, i & 1, err, &s_abort)) { ok = false; break; }
      tc_fence_after();
      uint32_t pw[16], dw[16];   // P^T and dS^T row segments, packed bf16 pairs
      {
        float sv[32], dv[32];
        tmem_ld32(tmem + lane_off + COL_S + 32 * half, sv);
        tmem_ld32(tmem + lane_off + COL_DP + 32 * half, dv);
        // S/dP are in registers: the MMA thread may overwrite them with item i+1
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sdp_free);
        const bool diag = qt * BQ < (kt + 1) * BK_KEYS;
        // causal: query qt*BQ + 32 half + c sees this key iff c >= lim
        const int lim = key - qt * BQ - 32 * half;
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          const float4 l4 = make_float4(__shfl_sync(0xffffffffu, cl, c), __shfl_sync(0xffffffffu, cl, c + 1),
                                        __shfl_sync(0xffffffffu, cl, c + 2), __shfl_sync(0xffffffffu, cl, c + 3));
          const float4 d4 = make_float4(__shfl_sync(0xffffffffu, cd, c), __shfl_sync(0xffffffffu, cd, c + 1),
                                        __shfl_sync(0xffffffffu, cd, c + 2), __shfl_sync(0xffffffffu, cd, c + 3));
          float p0 = ex2_approx(fmaf(sv[c], sl2, -l4.x));
          float p1 = ex2_approx(fmaf(sv[c + 1], sl2, -l4.y));
          float p2 = ex2_approx(fmaf(sv[c + 2], sl2, -l4.z));
          float p3 = ex2_approx(fmaf(sv[c + 3], sl2, -l4.w));
          if (diag) {
            if (c < lim) p0 = 0.f;
            if (c + 1 < lim) p1 = 0.f;
            if (c + 2 < lim) p2 = 0.f;
            if (c + 3 < lim) p3 = 0.f;
          }
          pw[c >> 1] = pack_bf16x2_rn(p0, p1);
          pw[(c >> 1) + 1] = pack_bf16x2_rn(p2, p3);
          dw[c >> 1] = pack_bf16x2_rn(p0 * (dv[c] - d4.x), p1 * (dv[c + 1] - d4.y));
          dw[(c >> 1) + 1] = pack_bf16x2_rn(p2 * (dv[c + 2] - d4.z), p3 * (dv[c + 3] - d4.w));
        }
      }
      // the P^T / dS^T tiles are free once item i-1's products are done
      if (i > 0) {
        if (!mbar_wait(mm_done, (i - 1) & 1, err, &s_abort)) { ok = false; break; }
        tc_fence_after();
      }
      // P^T and dS^T row segments -> 128-byte swizzled smem rows (16-byte
      // chunks 4 half .. 4 half + 3)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint32_t off = r * 128 + (((4 * half + c) ^ (r & 7)) << 4);
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
    if (ok && n_items > 0) {
      ok = mbar_wait(mm_done, (n_items - 1) & 1, err, &s_abort);
      if (ok) tc_fence_after();
    }
    if (ok && n_items > 0) {
      // dK (scaled) and dV of this CTA's keys, d columns [64 half, 64 half + 64)
      // (mm_done of the last item was waited)
      uint16_t* krow = dqkv + static_cast<int64_t>(row0 + key) * s.ld_qkv + (s.nh + kvh) * HD;
      uint16_t* vrow = dqkv + static_cast<int64_t>(row0 + key) * s.ld_qkv + (s.nh + s.nkv + kvh) * HD;
#pragma unroll 1
      for (int c0 = 64 * half; c0 < 64 * half + 64; c0 += 32) {
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
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0 && s_abort) {
    // loads still in flight land before the CTA exits
    mbar_wait(kv_full, 0, err, nullptr);
    for (int d = 0; d < QD_STAGES && d < issued; ++d)
      mbar_wait(&qd_full[(issued - 1 - d) % QD_STAGES], ((issued - 1 - d) / QD_STAGES) & 1, err, nullptr);
  }
  if ((warp == 1 || warp == 2) && s_abort) {
    // each issuer waits (bounded) for its own MMAs before TMEM is freed
    tc_fence_after();
    if (lane == 0) {
      umma_commit(&drain[warp - 1]);
      mbar_wait(&drain[warp - 1], 0, err, nullptr);
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Backward for head_dim 64.  The head_dim-128 plan above would give the dQ^T
// product M = hd = 64, below the 128 rows a single-CTA tcgen05.mma needs;
// here items are 128 queries, so every product has M = 128 and dQ itself
// (not its transpose) comes out of the tensor core:
//   S^T  = K . Q^T      dP^T = V . dO^T        (M=128 keys, N=128 q, K=64 d)
//   compute warps (thread = key row): P^T, dS^T as above, bf16 to smem
//   dV  += P^T . dO     dK  += dS^T . Q        (M=128 keys, N=64 d,  K=128 q)
//   dQ   = dS  . K                             (M=128 q,    N=64 d,  K=128 keys;
//                                               A = the dS^T tile read MN-major)
// One CTA per (query head, batch, 128-key tile), grid z = key tile so the
// CTAs with the most causal items (key tile 0) start first.  Each CTA covers
// one query head only, so the GQA heads of a KV head run in parallel and
// their dK/dV are added into an fp32 accumulator [B*T, 2 * nkv * 64] with
// TMA reduce-adds (as dQ is), then converted to bf16 with the inverse RoPE
// of dq and dk applied before the rounding.
// TMEM: S^T [0, 128), dP^T [128, 256), dQ buffers [256, 320) and [320, 384),
// dV [384, 448), dK [448, 512).  Eight compute warps: warp (quarter, half)
// owns TMEM lanes [32 quarter, +32) and query columns [64 half, +64) of
// S/dP, and d columns [32 half, +32) of dQ/dK/dV.  Staging tiles for the
// reduce-adds are [32 rows][32 fp32] in the 128-byte swizzle (16-byte chunk
// c of row r at chunk c ^ (r & 7): conflict-free row-per-lane stores).
// ---------------------------------------------------------------------------
constexpr int BWD64_THREADS = 320;   // producer, MMA, 8 compute warps
constexpr int B64_ROWS = 128;      // keys per CTA and queries per item
constexpr int B64_STAGES = 3;      // Q/dO ring depth

struct Bwd64Smem {
  static constexpr uint32_t TILE = B64_ROWS * 64 * 2;        // [128 rows][64 bf16] = 16 KB
  static constexpr uint32_t OFF_K = 0;
  static constexpr uint32_t OFF_V = OFF_K + TILE;
  static constexpr uint32_t OFF_Q = OFF_V + TILE;                  // [B64_STAGES]
  static constexpr uint32_t OFF_DO = OFF_Q + B64_STAGES * TILE;    // [B64_STAGES]
  static constexpr uint32_t OFF_P = OFF_DO + B64_STAGES * TILE;    // 2 blocks [128 keys][64 q]
  static constexpr uint32_t OFF_DS = OFF_P + 2 * TILE;
  static constexpr uint32_t STG_BYTES = 32 * 32 * 4;               // per compute warp
  static constexpr uint32_t OFF_STG = OFF_DS + 2 * TILE;
  static constexpr uint32_t OFF_BAR = OFF_STG + 8 * STG_BYTES;
  static constexpr uint32_t NUM_BARS = 1 + 2 * B64_STAGES + 1 + 1 + 1 + 1 + 2 + 1;
  static constexpr uint32_t TOTAL = 1024 + OFF_BAR + NUM_BARS * 8 + 16;
};
static_assert(Bwd64Smem::TOTAL <= 232448, "attention backward (hd 64): shared memory over 227 KB");
static_assert(Bwd64Smem::OFF_STG % 1024 == 0 && Bwd64Smem::OFF_P % 1024 == 0, "swizzle alignment");

// Row-per-lane [32 rows][32 fp32] tile (this lane = row) into a 128-byte
// swizzled staging tile, scaled.
__device__ __forceinline__ void stage_row32(float* stg, int lane, const float (&t)[32], float scale) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<float4*>(stg + lane * 32 + ((c ^ (lane & 7)) << 2)) =
        make_float4(t[4 * c] * scale, t[4 * c + 1] * scale, t[4 * c + 2] * scale, t[4 * c + 3] * scale);
}

__global__ void __launch_bounds__(BWD64_THREADS, 1)
    attn_bwd_tc64_kernel(const __grid_constant__ CUtensorMap tm_qkv,
                         const __grid_constant__ CUtensorMap tm_do,
                         const __grid_constant__ CUtensorMap tm_dq,
                         const __grid_constant__ CUtensorMap tm_dkv, const float* __restrict__ lse,
                         const float* __restrict__ dsum, AttnShape s, unsigned int* err) {
  using L = Bwd64Smem;
  constexpr int HD = 64;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t COL_S = 0, COL_DP = 128, COL_DQ = 256, COL_DV = 384, COL_DK = 448;
  constexpr uint32_t ID_SDP = make_idesc(128, false, false);   // N = 128 q, both K-major
  constexpr uint32_t ID_DVK = make_idesc(HD, false, true);     // N = 64 d, A K-major, B MN-major
  constexpr uint32_t ID_DQ = make_idesc(HD, true, true);       // N = 64 d, A and B MN-major
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t* kv_full = bars;
  uint64_t* qd_full = kv_full + 1;             // [B64_STAGES]
  uint64_t* qd_empty = qd_full + B64_STAGES;   // [B64_STAGES]
  uint64_t* sdp_full = qd_empty + B64_STAGES;
  uint64_t* sdp_free = sdp_full + 1;
  uint64_t* p_full = sdp_free + 1;
  uint64_t* mm_done = p_full + 1;
  uint64_t* dq_free = mm_done + 1;             // [2]
  uint64_t* drain = dq_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  __shared__ int abort_flag;
  volatile int& s_abort = abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, b = blockIdx.y, kt = blockIdx.z;
  const int kvh = h / (s.nh / s.nkv);
  const int n_items = s.T / B64_ROWS - kt;     // causal query tiles kt .. T/128 - 1
  const int row0 = b * s.T;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < B64_STAGES; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(sdp_full, 1);
    mbar_init(sdp_free, 8);
    mbar_init(p_full, 8);
    mbar_init(mm_done, 1);
    for (int i = 0; i < 2; ++i) mbar_init(&dq_free[i], 8);
    mbar_init(drain, 1);
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_qkv);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
    tma_prefetch_desc(&tm_dkv);
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
  int issued = 0;   // Q/dO items the producer issued (read on the abort path)

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      const int kcol = (s.nh + kvh) * HD, vcol = (s.nh + s.nkv + kvh) * HD;
      mbar_arrive_expect_tx(kv_full, 2 * L::TILE);
      tma_load_2d(sm + L::OFF_K, &tm_qkv, kv_full, kcol, row0 + kt * B64_ROWS);
      tma_load_2d(sm + L::OFF_V, &tm_qkv, kv_full, vcol, row0 + kt * B64_ROWS);
      for (int i = 0; i < n_items && !s_abort; ++i) {
        const int st = i % B64_STAGES;
        const int qrow = row0 + (kt + i) * B64_ROWS;
        if (!mbar_wait(&qd_empty[st], ((i / B64_STAGES) & 1) ^ 1, err, &s_abort)) { s_abort = 1; break; }
        mbar_arrive_expect_tx(&qd_full[st], 2 * L::TILE);
        tma_load_2d(sm + L::OFF_Q + st * L::TILE, &tm_qkv, &qd_full[st], h * HD, qrow);
        tma_load_2d(sm + L::OFF_DO + st * L::TILE, &tm_do, &qd_full[st], h * HD, qrow);
        issued = i + 1;
      }
    }
  } else if (warp == 1) {
    // ------------------------------ MMA issuer ----------------------------
    if (lane == 0) {
      auto issue_sdp = [&](int j) -> bool {
        const int st = j % B64_STAGES;
        if (!mbar_wait(&qd_full[st], (j / B64_STAGES) & 1, err, &s_abort)) return false;
        if (j > 0 && !mbar_wait(sdp_free, (j - 1) & 1, err, &s_abort)) return false;
        tc_fence_after();
        const uint32_t qb = sQ + st * L::TILE, db = sDO + st * L::TILE;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_bf16(tmem + COL_S, desc_kmajor(sK, k), desc_kmajor(qb, k), ID_SDP, k > 0);
#pragma unroll
        for (int k = 0; k < HD / 16; ++k)
          umma_bf16(tmem + COL_DP, desc_kmajor(sV, k), desc_kmajor(db, k), ID_SDP, k > 0);
        umma_commit(sdp_full);
        return true;
      };
      bool ok = mbar_wait(kv_full, 0, err, &s_abort);
      if (ok && n_items > 0) { tc_fence_after(); ok = issue_sdp(0); }
      for (int i = 0; ok && i < n_items; ++i) {
        if (i + 1 < n_items && !issue_sdp(i + 1)) { ok = false; break; }
        const int st = i % B64_STAGES;
        if (!mbar_wait(p_full, i & 1, err, &s_abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qb = sQ + st * L::TILE, db = sDO + st * L::TILE;
        // dV += P^T . dO, dK += dS^T . Q: K = 128 queries, the P^T / dS^T
        // tiles in two 64-query K-major blocks; dO / Q read MN-major
#pragma unroll
        for (int k = 0; k < B64_ROWS / 16; ++k) {
          umma_bf16(tmem + COL_DV, desc_kmajor(sP + (k >> 2) * L::TILE, k & 3), desc_mnmajor(db, k), ID_DVK,
                    (i > 0 || k > 0));
          umma_bf16(tmem + COL_DK, desc_kmajor(sDS + (k >> 2) * L::TILE, k & 3), desc_mnmajor(qb, k), ID_DVK,
                    (i > 0 || k > 0));
        }
        // dQ = dS . K into buffer i & 1 (drained for item i-2 by now): A = the
        // dS^T tile read MN-major (its two 64-query blocks are the M chunks,
        // 16 KB apart), B = the K tile read MN-major (d contiguous)
        if (!mbar_wait(&dq_free[i & 1], ((i >> 1) & 1) ^ 1, err, &s_abort)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < B64_ROWS / 16; ++k)
          umma_bf16(tmem + COL_DQ + 64u * (i & 1), make_sdesc(sDS + k * (UMMA_K * 128), L::TILE, 1024),
                    make_sdesc(sK + k * (UMMA_K * 128), 8192, 1024), ID_DQ, k > 0);
        umma_commit(mm_done);
        umma_commit(&qd_empty[st]);
      }
      if (!ok) s_abort = 1;
    }
  } else {
    // ------------------------------- compute ------------------------------
    const int sub = warp & 3;                 // TMEM lane quarter
    const int half = (warp - 2) >> 2;         // S/dP query columns [64 half, +64); d columns [32 half, +32)
    const int r = sub * 32 + lane;            // key row of S/dP/dK/dV, query row of dQ
    const uint32_t lane_off = static_cast<uint32_t>(sub * 32) << 16;
    const float sl2 = s.scale * LOG2E_F;
    float* stg = reinterpret_cast<float*>(sm + L::OFF_STG + (warp - 2) * L::STG_BYTES);
    const uint32_t sSTG = smem_u32(stg);
    // lse / dsum of this warp's 64 query columns of item i: lane holds
    // columns lane and 32 + lane, broadcast by shuffle; prefetched one item ahead
    auto lse_base = [&](int i) -> int64_t {
      return (static_cast<int64_t>(b) * s.nh + h) * s.T + (kt + i) * B64_ROWS + 64 * half;
    };
    float pl0 = lse[lse_base(0) + lane], pl1 = lse[lse_base(0) + 32 + lane];
    float pd0 = dsum[lse_base(0) + lane], pd1 = dsum[lse_base(0) + 32 + lane];
    auto flush_dq = [&](int j) {
      float t[32];
      tmem_ld32(tmem + lane_off + COL_DQ + 64u * (j & 1) + 32 * half, t);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&dq_free[j & 1]);
        bulk_wait_read0();                    // this warp's previous reduce has read its tile
      }
      __syncwarp();
      stage_row32(stg, lane, t, s.scale);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_2d(&tm_dq, sSTG, h * HD + 32 * half, row0 + (kt + j) * B64_ROWS + 32 * sub);
        bulk_commit();
      }
    };
    bool ok = true;
    for (int i = 0; i < n_items; ++i) {
      const float cl0 = pl0 * LOG2E_F, cl1 = pl1 * LOG2E_F, cd0 = pd0, cd1 = pd1;
      if (i + 1 < n_items) {
        const int64_t nb = lse_base(i + 1);
        pl0 = lse[nb + lane];
        pl1 = lse[nb + 32 + lane];
        pd0 = dsum[nb + lane];
        pd1 = dsum[nb + 32 + lane];
      }
      if (!mbar_wait(sdp_full, i & 1, err, &s_abort)) { ok = false; break; }
      tc_fence_after();
      uint32_t pw[32], dw[32];   // P^T and dS^T row segments, packed bf16 pairs
      {
        float sv[64], dv[64];
        tmem_ld32(tmem + lane_off + COL_S + 64 * half, *reinterpret_cast<float(*)[32]>(sv));
        tmem_ld32(tmem + lane_off + COL_S + 64 * half + 32, *reinterpret_cast<float(*)[32]>(sv + 32));
        tmem_ld32(tmem + lane_off + COL_DP + 64 * half, *reinterpret_cast<float(*)[32]>(dv));
        tmem_ld32(tmem + lane_off + COL_DP + 64 * half + 32, *reinterpret_cast<float(*)[32]>(dv + 32));
        // S/dP are in registers: the MMA thread may overwrite them with item i+1
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sdp_free);
        // causal (diagonal item only): query column c sees key r iff 64 half + c >= r
        const bool diag = i == 0;
        const int lim = r - 64 * half;
#pragma unroll
        for (int c = 0; c < 64; c += 2) {
          const float lc = c < 32 ? cl0 : cl1, dc = c < 32 ? cd0 : cd1;
          const float l0 = __shfl_sync(0xffffffffu, lc, c & 31), l1 = __shfl_sync(0xffffffffu, lc, (c + 1) & 31);
          const float d0 = __shfl_sync(0xffffffffu, dc, c & 31), d1 = __shfl_sync(0xffffffffu, dc, (c + 1) & 31);
          float p0 = ex2_approx(fmaf(sv[c], sl2, -l0));
          float p1 = ex2_approx(fmaf(sv[c + 1], sl2, -l1));
          if (diag) {
            if (c < lim) p0 = 0.f;
            if (c + 1 < lim) p1 = 0.f;
          }
          pw[c >> 1] = pack_bf16x2_rn(p0, p1);
          dw[c >> 1] = pack_bf16x2_rn(p0 * (dv[c] - d0), p1 * (dv[c + 1] - d1));
        }
      }
      // the P^T / dS^T tiles are free once item i-1's products are done
      if (i > 0) {
        if (!mbar_wait(mm_done, (i - 1) & 1, err, &s_abort)) { ok = false; break; }
        tc_fence_after();
      }
      // row r of block `half` (query columns [64 half, +64)), 128-byte swizzle
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint32_t off = half * L::TILE + r * 128 + ((c ^ (r & 7)) << 4);
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
      if (i > 0) flush_dq(i - 1);
    }
    if (ok && n_items > 0) {
      ok = mbar_wait(mm_done, (n_items - 1) & 1, err, &s_abort);
      if (ok) {
        tc_fence_after();
        flush_dq(n_items - 1);
        // dV, then dK (scaled), of this CTA's keys and query head into the
        // shared fp32 accumulator (the GQA heads of the KV head add up there)
        const int krow = row0 + kt * B64_ROWS + 32 * sub;
#pragma unroll 1
        for (int which = 0; which < 2; ++which) {
          float t[32];
          tmem_ld32(tmem + lane_off + (which == 0 ? COL_DV : COL_DK) + 32 * half, t);
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
          stage_row32(stg, lane, t, which == 0 ? 1.0f : s.scale);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int col = (which == 0 ? s.nkv * HD : 0) + kvh * HD + 32 * half;
            tma_reduce_add_2d(&tm_dkv, sSTG, col, krow);
            bulk_commit();
          }
        }
      }
    }
    if (!ok) s_abort = 1;
    if (lane == 0) bulk_wait0();   // this warp's reduce-adds complete before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0 && s_abort) {
    // loads still in flight land before the CTA exits
    mbar_wait(kv_full, 0, err, nullptr);
    for (int d = 0; d < B64_STAGES && d < issued; ++d)
      mbar_wait(&qd_full[(issued - 1 - d) % B64_STAGES], ((issued - 1 - d) / B64_STAGES) & 1, err, nullptr);
  }
  if (warp == 1) {
    tc_fence_after();
    if (s_abort) {
      if (lane == 0) {
        umma_commit(drain);
        mbar_wait(drain, 0, err, nullptr);
      }
      __syncwarp();
    }
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// fp32 accumulator [M, acc_ld] (heads x hd columns) -> bf16 columns of dst
// (dst_ld), with the inverse half-split RoPE (the transpose of the forward
// rotation, rope_impl.inc:21-36) applied before the rounding when cs is given:
// one thread per (token, head, 4 dims of the first half) and their partners.
__global__ void acc_to_bf16_kernel(const float* __restrict__ acc, int64_t acc_ld, int heads, int hd,
                                   uint16_t* __restrict__ dst, int64_t dst_ld, int64_t M, int T,
                                   const float* __restrict__ cs, const float* __restrict__ sn) {
  const int half = hd / 2;
  const int groups = half / 4;
  const int64_t total = M * heads * groups;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % groups);
    const int64_t rr = i / groups;
    const int hh = static_cast<int>(rr % heads);
    const int64_t t = rr / heads;
    const float* a = acc + t * acc_ld + static_cast<int64_t>(hh) * hd + g * 4;
    float4 x1 = *reinterpret_cast<const float4*>(a);
    float4 x2 = *reinterpret_cast<const float4*>(a + half);
    if (cs) {
      const int pos = static_cast<int>(t % T);
      const float4 co = *reinterpret_cast<const float4*>(cs + static_cast<int64_t>(pos) * half + g * 4);
      const float4 si = *reinterpret_cast<const float4*>(sn + static_cast<int64_t>(pos) * half + g * 4);
      const float4 y1 = make_float4(x1.x * co.x + x2.x * si.x, x1.y * co.y + x2.y * si.y,
                                    x1.z * co.z + x2.z * si.z, x1.w * co.w + x2.w * si.w);
      const float4 y2 = make_float4(x2.x * co.x - x1.x * si.x, x2.y * co.y - x1.y * si.y,
                                    x2.z * co.z - x1.z * si.z, x2.w * co.w - x1.w * si.w);
      x1 = y1;
      x2 = y2;
    }
    uint16_t* d = dst + t * dst_ld + static_cast<int64_t>(hh) * hd + g * 4;
    *reinterpret_cast<uint2*>(d) = make_uint2(pack_bf16x2(x1.x, x1.y), pack_bf16x2(x1.z, x1.w));
    *reinterpret_cast<uint2*>(d + half) = make_uint2(pack_bf16x2(x2.x, x2.y), pack_bf16x2(x2.z, x2.w));
  }
}

int acc_to_bf16(const float* acc, int64_t acc_ld, int heads, int hd, uint16_t* dst, int64_t dst_ld,
                int64_t M, int T, const float* cs, const float* sn, cudaStream_t st) {
  const int64_t n = M * heads * (hd / 8);
  int blocks = static_cast<int>((n + 255) / 256);
  if (blocks > num_sms() * 16) blocks = num_sms() * 16;
  if (blocks < 1) return GLT_OK;
  acc_to_bf16_kernel<<<blocks, 256, 0, st>>>(acc, acc_ld, heads, hd, dst, dst_ld, M, T, cs, sn);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

}  // namespace

int flash_bwd_tc(const uint16_t* qkv, const uint16_t* o, const uint16_t* dout, const float* lse,
                 uint16_t* dqkv, float* dq_acc, float* dsum, const AttnShape& s, cudaStream_t st,
                 bool dsum_ready, const float* rope_cos, const float* rope_sin) {
  if (s.hd != 128) return fail(GLT_EINVAL, "attention backward (tcgen05): head_dim must be 128");
  if (s.T % BK_KEYS) return fail(GLT_EINVAL, "attention backward (tcgen05): seq_len %% 128 != 0");
  if (s.nkv <= 0 || s.nh % s.nkv) return fail(GLT_EINVAL, "attention: nh %% nkv != 0");
  if (s.ld_qkv % 8 || s.ld_o % 8) return fail(GLT_EINVAL, "attention: strides not 16-byte");
  GLT_TRY(attn_bwd_prep(o, dout, dq_acc, dsum, s, st, dsum_ready));
  const int64_t M = static_cast<int64_t>(s.B) * s.T;
  CUtensorMap tk, tq, tdo, tdq;
  GLT_TRY(make_tmap_bf16(&tk, qkv, s.ld_qkv, M, s.ld_qkv, BK_KEYS));
  GLT_TRY(make_tmap_bf16(&tq, qkv, s.ld_qkv, M, s.ld_qkv, BQ));
  GLT_TRY(make_tmap_bf16(&tdo, dout, s.ld_o, M, s.ld_o, BQ));
  GLT_TRY(make_tmap_f32_plain(&tdq, dq_acc, static_cast<uint64_t>(s.nh) * s.hd, M,
                              static_cast<uint64_t>(s.nh) * s.hd, 32, 32));
  constexpr int smem = BwdSmem::TOTAL;
  GLT_TRY(ensure_smem_attr(reinterpret_cast<const void*>(attn_bwd_tc_kernel), smem));
  dim3 grid(s.T / BK_KEYS, s.nkv, s.B);
  attn_bwd_tc_kernel<<<grid, BWD_THREADS, smem, st>>>(tk, tq, tdo, tdq, lse, dsum, dqkv, s,
                                              device_error_word());
  GLT_LAUNCH_CHECK();
  return attn_bwd_finish(dq_acc, dqkv, s, st, rope_cos, rope_sin);
}

int flash_bwd_tc64(const uint16_t* qkv, const uint16_t* o, const uint16_t* dout, const float* lse,
                   uint16_t* dqkv, float* acc, float* dsum, const AttnShape& s, cudaStream_t st,
                   bool dsum_ready, const float* rope_cos, const float* rope_sin) {
  if (s.hd != 64) return fail(GLT_EINVAL, "attention backward (tcgen05, hd 64): head_dim must be 64");
  if (s.T % B64_ROWS) return fail(GLT_EINVAL, "attention backward (tcgen05): seq_len %% 128 != 0");
  if (s.nkv <= 0 || s.nh % s.nkv) return fail(GLT_EINVAL, "attention: nh %% nkv != 0");
  if (s.ld_qkv % 8 || s.ld_o % 8) return fail(GLT_EINVAL, "attention: strides not 16-byte");
  if (rope_cos && !rope_sin) return fail(GLT_EINVAL, "attention backward: rope tables");
  GLT_TRY(attn_bwd_prep(o, dout, acc, dsum, s, st, dsum_ready));   // zeroes dq, computes dsum
  const int64_t M = static_cast<int64_t>(s.B) * s.T;
  const int64_t qcols = static_cast<int64_t>(s.nh) * s.hd, kvcols = 2 * static_cast<int64_t>(s.nkv) * s.hd;
  float* dkv = acc + M * qcols;
  GLT_CUDA_TRY(cudaMemsetAsync(dkv, 0, static_cast<size_t>(M * kvcols) * sizeof(float), st));
  CUtensorMap tqkv, tdo, tdq, tdkv;
  GLT_TRY(make_tmap_bf16(&tqkv, qkv, s.ld_qkv, M, s.ld_qkv, B64_ROWS));
  GLT_TRY(make_tmap_bf16(&tdo, dout, s.ld_o, M, s.ld_o, B64_ROWS));
  GLT_TRY(make_tmap_f32_swz128(&tdq, acc, qcols, M, qcols, 32));
  GLT_TRY(make_tmap_f32_swz128(&tdkv, dkv, kvcols, M, kvcols, 32));
  constexpr int smem = Bwd64Smem::TOTAL;
  GLT_TRY(ensure_smem_attr(reinterpret_cast<const void*>(attn_bwd_tc64_kernel), smem));
  dim3 grid(s.nh, s.B, s.T / B64_ROWS);
  attn_bwd_tc64_kernel<<<grid, BWD64_THREADS, smem, st>>>(tqkv, tdo, tdq, tdkv, lse, dsum, s,
                                                         device_error_word());
  GLT_LAUNCH_CHECK();
  GLT_TRY(acc_to_bf16(acc, qcols, s.nh, s.hd, dqkv, s.ld_qkv, M, s.T, rope_cos, rope_sin, st));
  GLT_TRY(acc_to_bf16(dkv, kvcols, s.nkv, s.hd, dqkv + qcols, s.ld_qkv, M, s.T, rope_cos, rope_sin, st));
  return acc_to_bf16(dkv + static_cast<int64_t>(s.nkv) * s.hd, kvcols, s.nkv, s.hd,
                     dqkv + qcols + static_cast<int64_t>(s.nkv) * s.hd, s.ld_qkv, M, s.T, nullptr, nullptr, st);
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
