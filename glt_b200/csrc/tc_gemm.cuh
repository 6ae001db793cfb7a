// tcgen05 / TMEM / TMA GEMM core for sm_100a.
//
//   D[M,N] (+)= A[M,K] * B[N,K]^T          (bf16 operands, fp32 accumulate)
//
// A is "K-major" when stored row-major [M][K] (K contiguous) and "MN-major"
// when stored [K][M] (M contiguous); likewise B is K-major when stored
// [N][K] and MN-major when stored [K][N].  All four combinations run on the
// tensor cores directly (the UMMA smem descriptor carries the major-ness), so
// forward (x.W^T), input-grad (dy.W) and weight-grad (X^T.dY, K = tokens)
// contractions of the grafted MLP need no transposed copies.
//
// Structure (one persistent CTA per SM, 2 + 4 * parts warps):
//   warp 0      TMA producer: 128B-swizzled tiles into a STAGES-deep ring
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//   warps 2..   epilogue: tcgen05.ld of the 128 x BN fp32 accumulator,
//               user epilogue functor (stores / SwiGLU / residual / atomics).
//               An epilogue functor with `static constexpr int kParts = 2`
//               gets 8 epilogue warps: two per TMEM sub-partition (32 rows),
//               which split the tile's columns (EpiCtx::part / parts); the
//               memory-heavy SwiGLU epilogues use it for twice the loads and
//               stores in flight.  `static constexpr int kScratchPerWarp`
//               reserves that many bytes of shared memory per epilogue warp
//               (EpiCtx::scratch), used to turn row-per-lane results into
//               coalesced stores.
// Two TMEM accumulators (2*BN columns) let the epilogue of tile i overlap
// the main loop of tile i+1.  The producer picks each CTA's work units and
// hands them to the MMA and epilogue warps through a small shared-memory
// ring: round-robin (unit = blockIdx.x + t * gridDim.x) by default, or, with
// GemmShape::tile_ctr, claimed from a device counter in raster order, so a
// CTA that starts late (its SM busy with another kernel, such as a
// collective) takes fewer tiles instead of finishing last.  Every TMA load is a plain per-CTA load into
// the CTA's own shared memory, so the kernel is safe in multi-GPU jobs.
//
// Every mbarrier wait is bounded (GemmShape::timeout_ns of %globaltimer,
// GLT_MBAR_TIMEOUT_NS by default); a timed-out wait records
// GLT_DEVERR_MBAR_TIMEOUT in the launch's error word and sets the CTA's abort
// flag, on which every other role of the CTA gives up its own wait; the CTA
// then waits (bounded) for its loads in flight and its issued MMAs, frees its
// TMEM and exits, instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include <type_traits>

#include "common.cuh"

namespace glt {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;             // one 128-byte swizzle span of bf16
constexpr int UMMA_K = 16;
constexpr int NUM_THREADS = 192;   // 6 warps: producer, MMA, 4 epilogue warps (kParts = 1)
constexpr uint64_t GLT_MBAR_TIMEOUT_NS = 4000000000ull;  // 4 s

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait.  Returns false after `timeout_ns` of %globaltimer (and
// records GLT_DEVERR_MBAR_TIMEOUT in *err), or as soon as *abort (a flag in
// the CTA's own shared memory, nullable) is set by another role of the same
// CTA that gave up first.  Nothing outside the CTA is consulted, so a timeout
// in one launch never shortens the waits of a later one.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned int* err,
                                          const volatile int* abort = nullptr,
                                          uint64_t timeout_ns = GLT_MBAR_TIMEOUT_NS) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(addr, parity)) return true;
    if (globaltimer() - t0 > timeout_ns) {
      if (err) atomicOr(err, GLT_DEVERR_MBAR_TIMEOUT);
      return false;
    }
    if (abort && *abort != 0) return false;
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
// Same load with an L2 eviction-priority policy (createpolicy value).
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* tm, uint64_t* bar,
                                                 int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
// L2 policy: keep the lines (evicted after evict_normal/evict_first lines).
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives
// row (lane_base + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------
// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, M = 128.
__host__ __device__ constexpr uint32_t make_idesc(int n, bool a_mn, bool b_mn) {
  return (1u << 4)                                  // D format f32
         | (1u << 7)                                // A bf16
         | (1u << 10)                               // B bf16
         | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((static_cast<uint32_t>(n) >> 3) << 17)    // N / 8
         | ((static_cast<uint32_t>(BM) >> 4) << 24);  // M / 16
}

// Shared-memory matrix descriptor, SWIZZLE_128B, sm100 version bits.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46) |
         (2ull << 61);
}

// Byte sizes of one stage's operand tiles.
template <int ROWS>
struct TileBytes {
  static constexpr uint32_t value = ROWS * BK * 2;
};

// K-major tile: ROWS rows of 128 bytes, 8-row swizzle atoms 1024 B apart.
// k-th UMMA slice starts 32 bytes further inside the atom.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile_saddr, int k) {
  return make_sdesc(tile_saddr + k * (UMMA_K * 2), 16, 1024);
}
// MN-major tile: (ROWS/64) chunks of [64 K-rows x 128 B] (8 KB each); the
// chunks are the leading-dimension step, 8-row K groups the stride step.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile_saddr, int k) {
  return make_sdesc(tile_saddr + k * (UMMA_K * 128), 8192, 1024);
}

// ---------------------------------------------------------------------------
// Problem description passed by value to the kernel
// ---------------------------------------------------------------------------
struct GemmShape {
  int M, N, K;
  int k_splits;        // split-K factor (epilogue must accumulate atomically if > 1)
  int a2_n_tile;       // n-tiles >= this use the second A operand map (INT_MAX: never)
  int group_m;         // m-tiles per raster group (L2 reuse)
  unsigned int* err;   // device error word
  // Optional device-side row count: the kernel runs min(M, *m_dev - m_off)
  // rows (clamped at 0), read once at start by every thread.  M stays the
  // capacity the tensor maps were built for; a row count produced by an
  // earlier kernel on the stream then needs no host round trip.
  const int* m_dev = nullptr;
  int m_off = 0;
  // Optional dynamic tile claiming: two ints, zero before the launch; the
  // last CTA to finish sets them back to zero for the next launch on the
  // stream.  One counter pair per stream (launches on it must not overlap).
  int* tile_ctr = nullptr;
  // Bound of every mbarrier wait of the launch.
  uint64_t timeout_ns = GLT_MBAR_TIMEOUT_NS;
  // Failure-path self-test only (glt_selftest_wait_timeout): CTA 0's
  // producer never arms or loads its first k-block, so that CTA's MMA wait
  // runs out and the CTA takes the abort path.  0 in every product launch.
  int selftest_skip_first_load = 0;
};

constexpr int UNIT_RING = 4;   // work units in flight between the producer and the consumers

// Epilogue warps per TMEM sub-partition: Epi::kParts when the functor
// declares it, else 1.
template <class Epi, class = void>
struct EpiParts {
  static constexpr int value = 1;
};
template <class Epi>
struct EpiParts<Epi, std::void_t<decltype(Epi::kParts)>> {
  static constexpr int value = Epi::kParts;
};
template <class Epi>
constexpr int gemm_threads() {
  return 64 + 128 * EpiParts<Epi>::value;
}
// Shared memory per epilogue warp: Epi::kScratchPerWarp when declared, else 0.
template <class Epi, class = void>
struct EpiScratch {
  static constexpr int value = 0;
};
template <class Epi>
struct EpiScratch<Epi, std::void_t<decltype(Epi::kScratchPerWarp)>> {
  static constexpr int value = Epi::kScratchPerWarp;
};

// Per-thread view handed to epilogue functors.
template <int BN>
struct EpiCtx {
  uint32_t tmem_row;  // TMEM address of (this thread's lane, accumulator column 0)
  int row;            // global row of this thread
  int m0, n0;         // tile origin
  int split;          // split-K index of this work unit
  int part, parts;    // this warp's share of the tile's columns (kParts > 1)
  uint8_t* scratch;   // this warp's kScratchPerWarp bytes of shared memory (128-byte aligned)
  __device__ __forceinline__ void load(int col, float (&v)[32]) const {
    tmem_ld32(tmem_row + static_cast<uint32_t>(col), v);
  }
};

template <int BN, int STAGES>
struct SmemLayout {
  static constexpr uint32_t A_BYTES = TileBytes<BM>::value;
  static constexpr uint32_t B_BYTES = TileBytes<BN>::value;
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TILES_BYTES = STAGES * STAGE_BYTES;
  // barriers (stages, accumulators, drain, unit ring) + unit ids + tmem slot after the tiles
  static constexpr uint32_t BAR_BYTES = (2 * STAGES + 5 + 2 * UNIT_RING) * 8 + UNIT_RING * 4 + 16;
  static constexpr uint32_t TOTAL = 1024 /*align slack*/ + TILES_BYTES + BAR_BYTES;
  // epilogue scratch after the barriers
  static constexpr uint32_t SCRATCH_OFF = (TILES_BYTES + BAR_BYTES + 127) / 128 * 128;
};

// Dynamic shared memory of tc_gemm_kernel<BN, STAGES, *, *, Epi>.
template <int BN, int STAGES, class Epi>
constexpr uint32_t gemm_smem_bytes() {
  using L = SmemLayout<BN, STAGES>;
  return EpiScratch<Epi>::value == 0
             ? L::TOTAL
             : 1024 + L::SCRATCH_OFF + 4 * EpiParts<Epi>::value * EpiScratch<Epi>::value;
}

__device__ __forceinline__ void unit_coords(int unit, const GemmShape& s, int num_m, int num_n,
                                            int& mt, int& nt, int& split) {
  const int tiles = num_m * num_n;
  split = unit / tiles;
  int t = unit - split * tiles;
  const int per_group = s.group_m * num_n;
  const int g = t / per_group;
  const int first_m = g * s.group_m;
  const int gm = min(s.group_m, num_m - first_m);
  const int r = t - g * per_group;
  mt = first_m + r % gm;
  nt = r / gm;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi>
__global__ void __launch_bounds__(gemm_threads<Epi>(), 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmA2,
                   const __grid_constant__ CUtensorMap tmB, const GemmShape shape,
                   const Epi epi) {
  using L = SmemLayout<BN, STAGES>;
  constexpr int PARTS = EpiParts<Epi>::value;
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN");
  static_assert(PARTS == 1 || PARTS == 2, "kParts");
  static_assert(gemm_smem_bytes<BN, STAGES, Epi>() <= 232448 - 64, "shared memory");
  constexpr uint32_t TMEM_COLS = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64
                                 : (2 * BN <= 128) ? 128 : (2 * BN <= 256) ? 256 : 512;
  constexpr uint32_t IDESC = make_idesc(BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128B swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::TILES_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint64_t* drain_bar = tempty_bar + 2;      // [1] final MMA drain
  uint64_t* ufull_bar = drain_bar + 1;       // [UNIT_RING] unit id published
  uint64_t* uempty_bar = ufull_bar + UNIT_RING;  // [UNIT_RING] unit id read by every consumer
  volatile int* unit_ring = reinterpret_cast<volatile int*>(uempty_bar + UNIT_RING);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(const_cast<int*>(unit_ring) + UNIT_RING);
  __shared__ int s_abort_storage;
  volatile int& s_abort = s_abort_storage;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  int m_rows = shape.M;
  if (shape.m_dev) {
    const int v = *shape.m_dev - shape.m_off;
    m_rows = v < 0 ? 0 : (v < m_rows ? v : m_rows);
  }
  const int num_m = (m_rows + BM - 1) / BM;
  const int num_n = (shape.N + BN - 1) / BN;
  const int units = num_m * num_n * shape.k_splits;
  const int k_per_split = (shape.K + shape.k_splits - 1) / shape.k_splits;
  // split ranges are aligned to BK so TMA coordinates stay on 128 B.
  const int k_chunk = ((k_per_split + BK - 1) / BK) * BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 4 * PARTS);
    }
    mbar_init(drain_bar, 1);
    for (int r = 0; r < UNIT_RING; ++r) {
      mbar_init(&ufull_bar[r], 1);
      mbar_init(&uempty_bar[r], 1 + 4 * PARTS);   // MMA thread + epilogue warps
    }
    s_abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmA2);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // producer state read again on the abort path: k-blocks issued, and the one
  // never armed by the failure-path self-test (-1: none)
  int p_issued = 0;
  const int skip_it = (shape.selftest_skip_first_load && blockIdx.x == 0) ? 0 : -1;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      // A rows are reused by every N tile of the raster group (one group
      // sweeps N in ~10 waves of the grid) while epilogues stream far more
      // than L2 through it: A loads carry evict_last, B loads (reused by the
      // group's M tiles within about one wave) the default.
      const uint64_t pol_a = l2_policy_evict_last();
      int* const ctr = shape.tile_ctr;
      int claim = ctr ? atomicAdd(ctr, 1) : static_cast<int>(blockIdx.x);
      int it = 0;
      for (int t = 0; !s_abort; ++t) {
        // publish this CTA's next unit (-1: none left) to the MMA and epilogue warps
        const int slot = t % UNIT_RING;
        if (!mbar_wait(&uempty_bar[slot], ((t / UNIT_RING) & 1) ^ 1, shape.err, &s_abort, shape.timeout_ns)) {
          s_abort = 1;
          break;
        }
        const int unit = claim < units ? claim : -1;
        unit_ring[slot] = unit;
        mbar_arrive(&ufull_bar[slot]);
        if (unit < 0) break;
        // the next claim is in flight while this unit's loads are issued
        claim = ctr ? atomicAdd(ctr, 1) : unit + static_cast<int>(gridDim.x);
        int mt, nt, split;
        unit_coords(unit, shape, num_m, num_n, mt, nt, split);
        const CUtensorMap* tma = (nt >= shape.a2_n_tile) ? &tmA2 : &tmA;
        const int k_begin = split * k_chunk;
        const int k_end = min(shape.K, k_begin + k_chunk);
        const int m0 = mt * BM, n0 = nt * BN;
        for (int k0 = k_begin; k0 < k_end; k0 += BK, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, shape.err, &s_abort, shape.timeout_ns)) { s_abort = 1; break; }
          if (it == skip_it) continue;
          uint8_t* a_tile = tiles + s * L::STAGE_BYTES;
          uint8_t* b_tile = a_tile + L::A_BYTES;
          mbar_arrive_expect_tx(&full_bar[s], L::STAGE_BYTES);
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              tma_load_2d_hint(a_tile + c * 8192, tma, &full_bar[s], m0 + 64 * c, k0, pol_a);
          } else {
            tma_load_2d_hint(a_tile, tma, &full_bar[s], k0, m0, pol_a);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(b_tile + c * 8192, &tmB, &full_bar[s], n0 + 64 * c, k0);
          } else {
            tma_load_2d(b_tile, &tmB, &full_bar[s], k0, n0);
          }
        }
      }
      p_issued = it;
      if (ctr) {
        // every claim of this CTA is done; the last CTA out re-arms the counter
        __threadfence();
        if (atomicAdd(ctr + 1, 1) == static_cast<int>(gridDim.x) - 1) {
          atomicExch(ctr, 0);
          atomicExch(ctr + 1, 0);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------- MMA issuer -------------------------------
    if (lane == 0) {
      int it = 0;
      for (int local = 0; !s_abort; ++local) {
        const int slot = local % UNIT_RING;
        if (!mbar_wait(&ufull_bar[slot], (local / UNIT_RING) & 1, shape.err, &s_abort, shape.timeout_ns)) {
          s_abort = 1;
          break;
        }
        const int unit = unit_ring[slot];
        mbar_arrive(&uempty_bar[slot]);
        if (unit < 0) break;
        int mt, nt, split;
        unit_coords(unit, shape, num_m, num_n, mt, nt, split);
        const int k_begin = split * k_chunk;
        const int k_end = min(shape.K, k_begin + k_chunk);
        const int buf = local & 1;
        if (!mbar_wait(&tempty_bar[buf], ((local >> 1) & 1) ^ 1, shape.err, &s_abort, shape.timeout_ns)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        uint32_t acc = 0;
        bool ok = true;
        for (int k0 = k_begin; k0 < k_end; k0 += BK, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full_bar[s], ph, shape.err, &s_abort, shape.timeout_ns)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + s * L::STAGE_BYTES);
          const uint32_t b_addr = a_addr + L::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint64_t ad = A_MN ? desc_mnmajor(a_addr, k) : desc_kmajor(a_addr, k);
            const uint64_t bd = B_MN ? desc_mnmajor(b_addr, k) : desc_kmajor(b_addr, k);
            umma_bf16(d_tmem, ad, bd, IDESC, acc);
            acc = 1;
          }
          umma_commit(&empty_bar[s]);  // frees the smem slot once these MMAs retire
        }
        if (!ok) { s_abort = 1; break; }
        umma_commit(&tfull_bar[buf]);  // accumulator ready for the epilogue
      }
    }
  } else {
    // -------------------------------- epilogue --------------------------------
    const int sub = warp & 3;  // TMEM sub-partition this warp may access
    const int part = (warp - 2) >> 2;
    // every decision below is warp-uniform: the epilogue's TMEM loads are
    // warp-collective
    for (int local = 0;; ++local) {
      if (__shfl_sync(0xffffffffu, static_cast<int>(s_abort), 0)) break;
      const int slot = local % UNIT_RING;
      if (!__all_sync(0xffffffffu, mbar_wait(&ufull_bar[slot], (local / UNIT_RING) & 1, shape.err, &s_abort,
                                             shape.timeout_ns))) {
        s_abort = 1;
        break;
      }
      const int unit = __shfl_sync(0xffffffffu, unit_ring[slot], 0);
      __syncwarp();
      if (lane == 0) mbar_arrive(&uempty_bar[slot]);
      if (unit < 0) break;
      int mt, nt, split;
      unit_coords(unit, shape, num_m, num_n, mt, nt, split);
      const int buf = local & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull_bar[buf], (local >> 1) & 1, shape.err, &s_abort,
                                             shape.timeout_ns))) {
        s_abort = 1;
        break;
      }
      tc_fence_after();
      EpiCtx<BN> ctx;
      ctx.tmem_row = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) +
                     static_cast<uint32_t>(buf * BN);
      ctx.m0 = mt * BM;
      ctx.n0 = nt * BN;
      ctx.row = ctx.m0 + sub * 32 + lane;
      ctx.split = split;
      ctx.part = part;
      ctx.parts = PARTS;
      ctx.scratch = smem + L::SCRATCH_OFF + (warp - 2) * EpiScratch<Epi>::value;
      epi(ctx);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty_bar[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0 && s_abort) {
    // Abort path: loads this thread issued may still be landing in shared
    // memory.  Wait (bounded) for the last arming of every stage -- k-block
    // p_issued - 1 - d filled stage (p_issued - 1 - d) % STAGES -- before
    // the CTA exits.
    for (int d = 0; d < STAGES && d < p_issued; ++d) {
      const int j = p_issued - 1 - d;
      if (j == skip_it) continue;
      mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1, shape.err, nullptr, shape.timeout_ns);
    }
  }
  if (warp == 1) {
    tc_fence_after();
    if (s_abort) {
      // Abort path: make sure no issued MMA still writes TMEM before freeing it
      // (a bounded wait that ignores the abort flag).
      if (lane == 0) {
        umma_commit(drain_bar);
        mbar_wait(drain_bar, 0, shape.err, nullptr, shape.timeout_ns);
      }
      __syncwarp();
    }
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace tc
}  // namespace glt
