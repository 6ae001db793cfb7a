// Host-side launch machinery for the tcgen05 GEMM plus the epilogue functors
// shared by every contraction of the grafted decoder step.
#pragma once

#include <climits>

#include "tc_gemm.cuh"
#include "tc_gemm_pair.cuh"

namespace glt {

// One operand of a GEMM in the row-major views described in tc_gemm.cuh.
struct Operand {
  const void* ptr;   // bf16, 16-byte aligned
  int64_t ld;        // leading dimension in elements (multiple of 8)
  bool mn_major;     // false: [rows][K];  true: [K][rows]
};

// Encodes a 2-D bf16 tensor map with 128-byte swizzle:
//   dims {inner, outer}, row stride `ld` elements, box {64, box_outer}.
int make_tmap_bf16(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t outer,
                   uint64_t ld, uint32_t box_outer);
// 2-D fp32 tensor map without swizzle (dims {inner, outer}, row stride ld
// elements, box {box_inner, box_outer}); used for TMA reduce-add stores.
int make_tmap_f32_plain(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t outer,
                        uint64_t ld, uint32_t box_inner, uint32_t box_outer);
// 2-D fp32 tensor map with 128-byte swizzle: box {32, box_outer} (one 128-byte
// row of 32 floats per box row; 16-byte chunk c of row r at chunk c ^ (r & 7)
// in shared memory, which must be 1024-byte aligned).
int make_tmap_f32_swz128(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t outer,
                         uint64_t ld, uint32_t box_outer);

int num_sms();

// Dynamic tile claiming (GemmShape::tile_ctr) for the GEMMs this host thread
// launches: a device int[2], zero at rest, used by one stream at a time.
// A model sets its own counter around its steps (ScopedTileCounter); every
// other caller keeps the round-robin schedule.
inline int*& gemm_tile_counter() {
  static thread_local int* ctr = nullptr;
  return ctr;
}
struct ScopedTileCounter {
  int* prev;
  explicit ScopedTileCounter(int* c) : prev(gemm_tile_counter()) { gemm_tile_counter() = c; }
  ~ScopedTileCounter() { gemm_tile_counter() = prev; }
};
// SMs left to a collective that starts beside the next GEMMs this host thread
// launches: the next `launches` GEMMs run `sms` fewer CTAs (CTA pairs: sms / 2
// fewer clusters).  A persistent GEMM otherwise holds every SM, the
// collective's CTAs wait for it, and on the other ranks that collective's
// CTAs spin on SMs their own GEMMs' statically scheduled tiles are waiting
// for; with the SMs left free the collective starts at once and the GEMM's
// round-robin tiles balance over the rest.
struct SmReserve {
  int sms = 0;
  int launches = 0;
};
inline SmReserve& gemm_sm_reserve() {
  static thread_local SmReserve r;
  return r;
}
// SMs the GEMM being launched leaves free (consumes one reserved launch).
inline int take_sm_reserve() {
  SmReserve& r = gemm_sm_reserve();
  if (r.launches <= 0 || r.sms <= 0) return 0;
  --r.launches;
  return r.sms;
}
// Drops any reserve left when a step ends (also on its error paths).
struct ScopedSmReserveReset {
  ~ScopedSmReserveReset() { gemm_sm_reserve() = SmReserve{}; }
};
// Sets the dynamic-smem attribute of `func` to `bytes` once per (device, function).
int ensure_smem_attr(const void* func, int bytes);
// Prefers the largest shared-memory carveout for `func`, once per (device, function).
int ensure_smem_carveout_max(const void* func);
// Number of two-CTA clusters of `func` (threads, dynamic smem) resident at
// once on this device, cached per (device, function).
int max_active_pairs(const void* func, int threads, int smem, int* pairs);

// Whether launch_gemm runs its 256-column GEMMs on CTA pairs
// (tc_gemm_pair.cuh); glt_gemm_pair_mode sets it, GLT_GEMM_PAIR=0 in the
// environment turns the default (on) off.
bool gemm_pair_mode();

// ---------------------------------------------------------------------------
// Launcher
// ---------------------------------------------------------------------------
// err: the launch's error word (default: this device's, device_error_word());
// timeout_ns bounds every mbarrier wait; selftest_skip_first_load is the
// failure-path self-test switch of GemmShape (0 in every product launch).
// group_m: m-tiles per raster group.  32 keeps a 32-tile block of A (32 MB
// at K = 4096) resident in L2 while the 148 persistent CTAs sweep N, so a
// K = 4096 weight such as W_gu (252 MB) streams from HBM once per 32 m-tiles
// rather than once per 8; at the config-3 step this is worth ~1.5% under the
// 1 kW power cap (less DRAM energy, same tensor work).
// Deepest stage ring of 32 KB stages (at most 8) that fits beside the
// barriers and the epilogue's scratch.
template <class Epi>
constexpr int pair_stages() {
  constexpr int scratch = 4 * tc::EpiParts<Epi>::value * tc::EpiScratch<Epi>::value;
  constexpr int avail = 232448 - 64 - 1024 - 512 - scratch;
  constexpr int s = avail / static_cast<int>(tc::PairSmemLayout<1>::STAGE_BYTES);
  return s > 8 ? 8 : s;
}

// The same contraction on CTA pairs: 256 x 256 output tiles, each CTA of a
// pair staging 128 rows of A and 128 rows of B per k-block.  group_m counts
// 256-row tiles.  Static round-robin schedule over clusters.
template <bool A_MN, bool B_MN, class Epi>
int launch_gemm_pair(const Operand& A, const Operand& B, int M, int N, int K, const Epi& epi,
                     cudaStream_t stream, int k_splits, const Operand* A2, int a2_n_tile,
                     int group_m, const int* m_dev, int m_off, unsigned int* err, uint64_t timeout_ns) {
  using namespace tc;
  constexpr int STAGES = pair_stages<Epi>();
  static_assert(STAGES >= 3, "pair GEMM: too little shared memory for the stage ring");
  if (M <= 0 || N <= 0 || K <= 0) return GLT_OK;
  if (A.mn_major != A_MN || B.mn_major != B_MN)
    return fail(GLT_EINVAL, "launch_gemm_pair: operand major-ness mismatch");
  CUtensorMap ta, ta2, tb;
  if (!A_MN) {
    GLT_TRY(make_tmap_bf16(&ta, A.ptr, K, M, A.ld, BM));
  } else {
    GLT_TRY(make_tmap_bf16(&ta, A.ptr, M, K, A.ld, 64));
  }
  if (A2) {
    if (A2->mn_major != A_MN) return fail(GLT_EINVAL, "launch_gemm_pair: A2 major-ness mismatch");
    if (!A_MN) {
      GLT_TRY(make_tmap_bf16(&ta2, A2->ptr, K, M, A2->ld, BM));
    } else {
      GLT_TRY(make_tmap_bf16(&ta2, A2->ptr, M, K, A2->ld, 64));
    }
  } else {
    ta2 = ta;
  }
  if (!B_MN) {
    GLT_TRY(make_tmap_bf16(&tb, B.ptr, K, N, B.ld, PAIR_BN / 2));
  } else {
    GLT_TRY(make_tmap_bf16(&tb, B.ptr, N, K, B.ld, 64));
  }
  GemmShape shape;
  shape.M = M;
  shape.N = N;
  shape.K = K;
  shape.k_splits = k_splits < 1 ? 1 : k_splits;
  shape.a2_n_tile = A2 ? a2_n_tile : INT_MAX;
  shape.group_m = group_m < 1 ? 1 : group_m;
  shape.m_dev = m_dev;
  shape.m_off = m_off;
  shape.tile_ctr = nullptr;
  shape.err = err ? err : device_error_word();
  if (!shape.err) return fail(GLT_ECUDA, "device error word unavailable");
  shape.timeout_ns = timeout_ns;
  shape.selftest_skip_first_load = 0;
  auto kern = tc_gemm_pair_kernel<STAGES, A_MN, B_MN, Epi>;
  constexpr int smem = gemm_pair_smem_bytes<STAGES, Epi>();
  constexpr int threads = gemm_threads<Epi>();
  GLT_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), smem));
  int pairs = 0;
  GLT_TRY(max_active_pairs(reinterpret_cast<const void*>(kern), threads, smem, &pairs));
  const int units = ((M + PAIR_BM - 1) / PAIR_BM) * ((N + PAIR_BN - 1) / PAIR_BN) * shape.k_splits;
  pairs -= take_sm_reserve() / 2;
  if (pairs < 1) pairs = 1;
  const int clusters = units < pairs ? units : pairs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  GLT_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, ta, ta2, tb, shape, epi));
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi>
int launch_gemm(const Operand& A, const Operand& B, int M, int N, int K, const Epi& epi,
                cudaStream_t stream, int k_splits = 1, const Operand* A2 = nullptr,
                int a2_n_tile = INT_MAX, int group_m = 32, const int* m_dev = nullptr,
                int m_off = 0, unsigned int* err = nullptr, uint64_t timeout_ns = tc::GLT_MBAR_TIMEOUT_NS,
                int selftest_skip_first_load = 0) {
  using namespace tc;
  if (M <= 0 || N <= 0 || K <= 0) return GLT_OK;
  if (A.mn_major != A_MN || B.mn_major != B_MN)
    return fail(GLT_EINVAL, "launch_gemm: operand major-ness mismatch");
  if constexpr (BN == 256) {
    if (gemm_pair_mode() && gemm_tile_counter() == nullptr && selftest_skip_first_load == 0)
      return launch_gemm_pair<A_MN, B_MN>(A, B, M, N, K, epi, stream, k_splits, A2, a2_n_tile,
                                          (group_m + 1) / 2, m_dev, m_off, err, timeout_ns);
  }
  CUtensorMap ta, ta2, tb;
  // A: K-major [M][K] -> dims {K, M}, box {64, 128};  MN-major [K][M] -> {M, K}, box {64, 64}
  if (!A_MN) {
    GLT_TRY(make_tmap_bf16(&ta, A.ptr, K, M, A.ld, BM));
  } else {
    GLT_TRY(make_tmap_bf16(&ta, A.ptr, M, K, A.ld, 64));
  }
  if (A2) {
    if (A2->mn_major != A_MN) return fail(GLT_EINVAL, "launch_gemm: A2 major-ness mismatch");
    if (!A_MN) {
      GLT_TRY(make_tmap_bf16(&ta2, A2->ptr, K, M, A2->ld, BM));
    } else {
      GLT_TRY(make_tmap_bf16(&ta2, A2->ptr, M, K, A2->ld, 64));
    }
  } else {
    ta2 = ta;
  }
  if (!B_MN) {
    GLT_TRY(make_tmap_bf16(&tb, B.ptr, K, N, B.ld, BN));
  } else {
    GLT_TRY(make_tmap_bf16(&tb, B.ptr, N, K, B.ld, 64));
  }
  GemmShape shape;
  shape.M = M;
  shape.N = N;
  shape.K = K;
  shape.k_splits = k_splits < 1 ? 1 : k_splits;
  shape.a2_n_tile = A2 ? a2_n_tile : INT_MAX;
  shape.group_m = group_m;
  shape.m_dev = m_dev;
  shape.m_off = m_off;
  shape.tile_ctr = gemm_tile_counter();
  shape.err = err ? err : device_error_word();
  if (!shape.err) return fail(GLT_ECUDA, "device error word unavailable");
  shape.timeout_ns = timeout_ns;
  shape.selftest_skip_first_load = selftest_skip_first_load;
  auto kern = tc_gemm_kernel<BN, STAGES, A_MN, B_MN, Epi>;
  constexpr int smem = gemm_smem_bytes<BN, STAGES, Epi>();
  GLT_TRY(ensure_smem_attr(reinterpret_cast<const void*>(kern), smem));
  const int units = ((M + BM - 1) / BM) * ((N + BN - 1) / BN) * shape.k_splits;
  int sms = num_sms() - take_sm_reserve();
  if (sms < 1) sms = 1;
  const int grid = units < sms ? units : sms;
  kern<<<grid, gemm_threads<Epi>(), smem, stream>>>(ta, ta2, tb, shape, epi);
  GLT_LAUNCH_CHECK();
  return GLT_OK;
}

// Picks a k-split so that the work units fill the SMs (weight-grad GEMMs have
// few output tiles and a long K = token dimension): about `waves2 / 2` waves
// of units (default 2 waves; fewer splits mean fewer fp32 atomics).
inline int pick_k_splits(int M, int N, int K, int bn, int waves2 = 4) {
  const int tiles = ((M + 127) / 128) * ((N + bn - 1) / bn);
  const int sms = num_sms();
  if (tiles >= sms) return 1;
  int s = (waves2 * sms + 2 * tiles - 1) / (2 * tiles);
  const int max_s = K / (tc::BK * 4);    // keep >= 4 k-blocks per split
  if (s > max_s) s = max_s;
  return s < 1 ? 1 : s;
}

// ---------------------------------------------------------------------------
// Epilogues
// ---------------------------------------------------------------------------
__device__ __forceinline__ void red_add_f32(float* p, float v) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}

// C (fp32) = alpha * acc + beta * C;  with `atomic`, C += alpha * acc (split-K).
template <int BN>
struct EpiF32 {
  float* C;
  int64_t ldc;
  int M, N;
  float alpha, beta;
  int atomic;
  int vec_ok;  // C, ldc and N allow 16-byte vector access
  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
#pragma unroll 1
    for (int j = 0; j < BN; j += 32) {
      float v[32];
      c.load(j, v);
      if (c.row >= M) continue;
      const int col0 = c.n0 + j;
      if (col0 >= N) continue;
      float* dst = C + static_cast<int64_t>(c.row) * ldc + col0;
      if (atomic) {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (col0 + i < N) red_add_f32(dst + i, alpha * v[i]);
      } else if (vec_ok && col0 + 32 <= N) {
#pragma unroll
        for (int i = 0; i < 32; i += 4) {
          float4 o;
          if (beta != 0.f) {
            const float4 old = *reinterpret_cast<const float4*>(dst + i);
            o = make_float4(alpha * v[i] + beta * old.x, alpha * v[i + 1] + beta * old.y,
                            alpha * v[i + 2] + beta * old.z, alpha * v[i + 3] + beta * old.w);
          } else {
            o = make_float4(alpha * v[i], alpha * v[i + 1], alpha * v[i + 2], alpha * v[i + 3]);
          }
          *reinterpret_cast<float4*>(dst + i) = o;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (col0 + i < N) dst[i] = alpha * v[i] + (beta != 0.f ? beta * dst[i] : 0.f);
      }
    }
  }
};

// C[rows[row]] (fp32) = acc for the first *n - off rows (row scatter; used
// with a device-side row count, so rows past it in the last tile are skipped).
template <int BN>
struct EpiF32Rows {
  float* C;
  int64_t ldc;
  const int* rows;   // row map of this launch (already offset)
  const int* n;      // device row count
  int off;
  int N;
  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
    // every lane takes part in the (warp-collective) TMEM loads; only live
    // rows store
    const bool live = c.row < *n - off;
    float* base = live ? C + static_cast<int64_t>(rows[c.row]) * ldc : nullptr;
#pragma unroll 1
    for (int j = 0; j < BN; j += 32) {
      const int col0 = c.n0 + j;   // the same for the whole warp
      if (col0 >= N) break;
      float v[32];
      c.load(j, v);
      if (!live) continue;
      float* dst = base + col0;
      if (col0 + 32 <= N) {
#pragma unroll
        for (int i = 0; i < 32; i += 4)
          *reinterpret_cast<float4*>(dst + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
      } else {
        for (int i = 0; i < 32 && col0 + i < N; ++i) dst[i] = v[i];
      }
    }
  }
};

// C (bf16) = bf16(acc [+ R]) where R is an optional bf16 residual (may alias C).
template <int BN>
struct EpiBF16 {
  uint16_t* C;
  int64_t ldc;
  const uint16_t* R;
  int64_t ldr;
  int M, N;
  int vec_ok;
  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
#pragma unroll 1
    for (int j = 0; j < BN; j += 32) {
      float v[32];
      c.load(j, v);
      if (c.row >= M) continue;
      const int col0 = c.n0 + j;
      if (col0 >= N) continue;
      uint16_t* dst = C + static_cast<int64_t>(c.row) * ldc + col0;
      if (vec_ok && col0 + 32 <= N) {
        if (R) {
          const uint16_t* rr = R + static_cast<int64_t>(c.row) * ldr + col0;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            const uint4 r4 = *reinterpret_cast<const uint4*>(rr + i);
            v[i + 0] += bf16_lo(r4.x); v[i + 1] += bf16_hi(r4.x);
            v[i + 2] += bf16_lo(r4.y); v[i + 3] += bf16_hi(r4.y);
            v[i + 4] += bf16_lo(r4.z); v[i + 5] += bf16_hi(r4.z);
            v[i + 6] += bf16_lo(r4.w); v[i + 7] += bf16_hi(r4.w);
          }
        }
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 o;
          o.x = pack_bf16x2_rn(v[i + 0], v[i + 1]);
          o.y = pack_bf16x2_rn(v[i + 2], v[i + 3]);
          o.z = pack_bf16x2_rn(v[i + 4], v[i + 5]);
          o.w = pack_bf16x2_rn(v[i + 6], v[i + 7]);
          *reinterpret_cast<uint4*>(dst + i) = o;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          if (col0 + i < N) {
            float x = v[i];
            if (R) x += bf16_bits_to_f32(R[static_cast<int64_t>(c.row) * ldr + col0 + i]);
            dst[i] = f32_to_bf16_bits(x);
          }
        }
      }
    }
  }
};

// The QKV projection with RoPE in its epilogue: C (bf16) = bf16(rope(acc)).
// Columns [0, rope_cols) hold the q and k heads (hd columns each), rotated
// half-split at their token's position (row % T) -- the rotation of
// rope_impl.inc:21-36 that rope_kernel applies to stored bf16 q/k, here on
// the fp32 accumulator before its one rounding; v columns pass through.  A
// tile holds whole heads (BN % hd == 0, hd in {64, 128}), so each pair of
// 32-column chunks (i, i + hd/2) is in the same tile.
template <int BN>
struct EpiBF16Rope {
  uint16_t* C;
  int64_t ldc;
  int M, N;
  int rope_cols, T, hd;
  const float* cs;   // [T, hd/2]
  const float* sn;
  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
    const bool row_ok = c.row < M;
    const int half = hd >> 1;
    const int pos = c.row % T;
#pragma unroll 1
    for (int hb = 0; hb < BN; hb += hd) {
#pragma unroll 1
      for (int jj = 0; jj < half; jj += 32) {
        const int j1 = hb + jj, j2 = j1 + half;
        float a[32], b[32];
        c.load(j1, a);   // warp-collective: every lane loads
        c.load(j2, b);
        const int col1 = c.n0 + j1;   // the same for the whole warp
        if (col1 >= N || !row_ok) continue;
        if (col1 < rope_cols) {
          const float4* cp = reinterpret_cast<const float4*>(cs + static_cast<int64_t>(pos) * half + jj);
          const float4* sp = reinterpret_cast<const float4*>(sn + static_cast<int64_t>(pos) * half + jj);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 co = __ldg(cp + q), si = __ldg(sp + q);
            const float cv[4] = {co.x, co.y, co.z, co.w}, sv[4] = {si.x, si.y, si.z, si.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float x1 = a[4 * q + k], x2 = b[4 * q + k];
              a[4 * q + k] = x1 * cv[k] - x2 * sv[k];
              b[4 * q + k] = x2 * cv[k] + x1 * sv[k];
            }
          }
        }
        uint16_t* d1 = C + static_cast<int64_t>(c.row) * ldc + col1;
        uint16_t* d2 = d1 + half;
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          *reinterpret_cast<uint4*>(d1 + i) = make_uint4(pack_bf16x2_rn(a[i], a[i + 1]), pack_bf16x2_rn(a[i + 2], a[i + 3]),
                                                         pack_bf16x2_rn(a[i + 4], a[i + 5]), pack_bf16x2_rn(a[i + 6], a[i + 7]));
          *reinterpret_cast<uint4*>(d2 + i) = make_uint4(pack_bf16x2_rn(b[i], b[i + 1]), pack_bf16x2_rn(b[i + 2], b[i + 3]),
                                                         pack_bf16x2_rn(b[i + 4], b[i + 5]), pack_bf16x2_rn(b[i + 6], b[i + 7]));
        }
      }
    }
  }
};

// The dO GEMM with the attention backward's row sums in its epilogue:
// C (bf16) = bf16(acc) and, per row and head (hd columns, whole heads per
// tile), dsum[(b * nh + h) * T + t] = sum over the head of bf16(dO) * O --
// the D_i = rowsum(dO o O) the flash backward needs (bwd_dsum_kernel's
// value, summed in another order), from the rounded dO it stores.
template <int BN>
struct EpiBF16Dsum {
  uint16_t* C;
  int64_t ldc;
  int M, N;
  const uint16_t* O;
  int64_t ldo;
  float* dsum;
  int T, nh, hd;
  __device__ __forceinline__ void operator()(const tc::EpiCtx<BN>& c) const {
    const bool row_ok = c.row < M;
#pragma unroll 1
    for (int hb = 0; hb < BN; hb += hd) {
      float acc = 0.f;
#pragma unroll 1
      for (int jj = 0; jj < hd; jj += 32) {
        float v[32];
        c.load(hb + jj, v);   // warp-collective: every lane loads
        const int col = c.n0 + hb + jj;
        if (col >= N || !row_ok) continue;
        uint16_t* dst = C + static_cast<int64_t>(c.row) * ldc + col;
        const uint4* orow = reinterpret_cast<const uint4*>(O + static_cast<int64_t>(c.row) * ldo + col);
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          uint4 w;
          w.x = pack_bf16x2_rn(v[i], v[i + 1]); w.y = pack_bf16x2_rn(v[i + 2], v[i + 3]);
          w.z = pack_bf16x2_rn(v[i + 4], v[i + 5]); w.w = pack_bf16x2_rn(v[i + 6], v[i + 7]);
          *reinterpret_cast<uint4*>(dst + i) = w;
          const uint4 o = __ldg(orow + i / 8);
          acc += bf16_lo(w.x) * bf16_lo(o.x) + bf16_hi(w.x) * bf16_hi(o.x) + bf16_lo(w.y) * bf16_lo(o.y) +
                 bf16_hi(w.y) * bf16_hi(o.y) + bf16_lo(w.z) * bf16_lo(o.z) + bf16_hi(w.z) * bf16_hi(o.z) +
                 bf16_lo(w.w) * bf16_lo(o.w) + bf16_hi(w.w) * bf16_hi(o.w);
        }
      }
      const int h = (c.n0 + hb) / hd;
      if (row_ok && c.n0 + hb < N) {
        const int b = c.row / T, t = c.row - b * T;
        dsum[(static_cast<int64_t>(b) * nh + h) * T + t] = acc;
      }
    }
  }
};

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace glt
