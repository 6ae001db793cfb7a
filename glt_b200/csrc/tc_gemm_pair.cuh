// Two-SM (cta_group::2) variant of the persistent tcgen05 GEMM in tc_gemm.cuh.
//
// A cluster of two CTAs computes one 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256, N = 256): CTA r of the pair holds rows
// [128 r, 128 r + 128) of the A tile and rows [128 r, 128 r + 128) of the
// B tile (the B tile's N is split between the pair), and its TMEM receives
// its own 128 rows x all 256 columns of the accumulator.  Per k-block each
// CTA therefore stages 16 KB of A and 16 KB of B (32 KB, against 48 KB for a
// one-SM 128 x 256 tile), which buys a deeper stage ring in the same shared
// memory and halves the B traffic per FLOP out of L2.
//
// Roles (per CTA, same warp layout as tc_gemm.cuh):
//   warp 0      TMA producer: its own A and B halves into its own shared
//               memory with cp.async.bulk.tensor...cta_group::2 (plain
//               loads, no cluster multicast); both CTAs' loads complete on
//               the leader's (rank 0) full barrier, which the leader's
//               producer arms with the bytes of both.
//   warp 1      both CTAs: TMEM allocation (cta_group::2, 2 x 256 columns).
//               Leader: the single tcgen05.mma issuer; every k-block's
//               commit is multicast to both CTAs' empty barriers, every
//               tile's to both CTAs' accumulator barriers.  Peer: only
//               follows the unit ring.
//   warps 2..   epilogue of the CTA's 128 rows (the same functors as the
//               one-SM kernel, with BN = 256); each epilogue warp of either
//               CTA releases the accumulator buffer on the leader's barrier.
// Cross-CTA arrives and waits use CTA-scope ordering, as the tcgen05 fences
// around them order the tensor-core work; cluster-scope release/acquire on
// the per-k-block path costs ~2.7x in throughput.
// The work-unit sequence is the round-robin one over clusters, computed by
// both CTAs alike (no dynamic claiming).
//
// Every wait is bounded as in tc_gemm.cuh.  On the abort path the leader
// waits (bounded by GLT_PAIR_DRAIN_NS) for the stages its producer armed --
// those barriers count both CTAs' bytes -- and for its issued MMAs; the peer,
// which cannot observe its own loads (they complete on the leader's
// barrier), waits GLT_PAIR_DRAIN_NS after its last issue, far longer than a
// TMA load takes.  A cluster barrier at the end keeps both CTAs resident
// until then and until both epilogues are done with the pair's TMEM.
#pragma once

#include "tc_gemm.cuh"

namespace glt {
namespace tc {

constexpr int PAIR_BM = 256;   // output rows per CTA pair (128 per CTA)
constexpr int PAIR_BN = 256;   // output columns per CTA pair (B: 128 rows per CTA)

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the object at the same offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t cta_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(cta_addr), "r"(rank));
  return r;
}
// Arrive on a barrier of either CTA of the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2-D tiled load into this CTA's shared memory whose completion (bytes) is
// counted on the barrier at `bar_cluster`, which may be the pair leader's.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* tm, uint32_t bar_cluster,
                                                 int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
// Same load without an L2 policy.
__device__ __forceinline__ void tma_load_2d_pair_nohint(void* dst, const CUtensorMap* tm, uint32_t bar_cluster,
                                                        int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}
// Bound of each abort-path drain of the pair kernel.
constexpr uint64_t GLT_PAIR_DRAIN_NS = 2000000ull;   // 2 ms
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// Arrive on the barrier at this offset in both CTAs of the pair once the
// issued MMAs retire.
__device__ __forceinline__ void umma_commit_pair_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}
// Arrive on this CTA's barrier only.
__device__ __forceinline__ void umma_commit_pair_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Instruction descriptor, kind::f16: bf16 x bf16 -> f32, M = 256 (pair), N = 256.
__host__ __device__ constexpr uint32_t make_idesc_pair(bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((static_cast<uint32_t>(PAIR_BN) >> 3) << 17) | ((static_cast<uint32_t>(PAIR_BM) >> 4) << 24);
}

template <int STAGES>
struct PairSmemLayout {
  static constexpr uint32_t A_BYTES = TileBytes<BM>::value;         // 128 rows of A
  static constexpr uint32_t B_BYTES = TileBytes<PAIR_BN / 2>::value;  // 128 rows of B
  static constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TILES_BYTES = STAGES * STAGE_BYTES;
  // full, empty [STAGES]; tfull, tempty [2]; drain; unit ring
  static constexpr uint32_t BAR_BYTES = (2 * STAGES + 5 + 2 * UNIT_RING) * 8 + UNIT_RING * 4 + 16;
  static constexpr uint32_t TOTAL = 1024 + TILES_BYTES + BAR_BYTES;
  static constexpr uint32_t SCRATCH_OFF = (TILES_BYTES + BAR_BYTES + 127) / 128 * 128;
};

template <int STAGES, class Epi>
constexpr uint32_t gemm_pair_smem_bytes() {
  using L = PairSmemLayout<STAGES>;
  return EpiScratch<Epi>::value == 0
             ? L::TOTAL
             : 1024 + L::SCRATCH_OFF + 4 * EpiParts<Epi>::value * EpiScratch<Epi>::value;
}

template <int STAGES, bool A_MN, bool B_MN, class Epi>
__global__ void __launch_bounds__(gemm_threads<Epi>(), 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmA2,
                        const __grid_constant__ CUtensorMap tmB, const GemmShape shape,
                        const Epi epi) {
  using L = PairSmemLayout<STAGES>;
  constexpr int BN = PAIR_BN;
  constexpr int PARTS = EpiParts<Epi>::value;
  static_assert(PARTS == 1 || PARTS == 2, "kParts");
  static_assert(gemm_pair_smem_bytes<STAGES, Epi>() <= 232448 - 64, "shared memory");
  constexpr uint32_t TMEM_COLS = 2 * BN;   // two accumulators of 256 columns
  constexpr uint32_t IDESC = make_idesc_pair(A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* tiles = smem;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::TILES_BYTES);   // leader's: both CTAs' bytes
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2] leader: both CTAs' epilogues done
  uint64_t* drain_bar = tempty_bar + 2;
  uint64_t* ufull_bar = drain_bar + 1;
  uint64_t* uempty_bar = ufull_bar + UNIT_RING;
  volatile int* unit_ring = reinterpret_cast<volatile int*>(uempty_bar + UNIT_RING);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(const_cast<int*>(unit_ring) + UNIT_RING);
  __shared__ int s_abort_storage;
  volatile int& s_abort = s_abort_storage;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = static_cast<int>(blockIdx.x >> 1);
  const int clusters = static_cast<int>(gridDim.x >> 1);

  int m_rows = shape.M;
  if (shape.m_dev) {
    const int v = *shape.m_dev - shape.m_off;
    m_rows = v < 0 ? 0 : (v < m_rows ? v : m_rows);
  }
  const int num_m = (m_rows + PAIR_BM - 1) / PAIR_BM;
  const int num_n = (shape.N + BN - 1) / BN;
  const int units = num_m * num_n * shape.k_splits;
  const int k_per_split = (shape.K + shape.k_splits - 1) / shape.k_splits;
  const int k_chunk = ((k_per_split + BK - 1) / BK) * BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 2 * 4 * PARTS);
    }
    mbar_init(drain_bar, 1);
    for (int r = 0; r < UNIT_RING; ++r) {
      mbar_init(&ufull_bar[r], 1);
      mbar_init(&uempty_bar[r], 1 + 4 * PARTS);
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
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // both CTAs' barriers are initialised and their TMEM allocated before any
  // remote arrive or pair MMA
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  int p_issued = 0;
  uint64_t p_last_issue = 0;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      const uint64_t pol_a = l2_policy_evict_last();
      int it = 0;
      for (int t = 0; !s_abort; ++t) {
        const int slot = t % UNIT_RING;
        if (!mbar_wait(&uempty_bar[slot], ((t / UNIT_RING) & 1) ^ 1, shape.err, &s_abort, shape.timeout_ns)) {
          s_abort = 1;
          break;
        }
        const int claim = cluster + t * clusters;
        const int unit = claim < units ? claim : -1;
        unit_ring[slot] = unit;
        mbar_arrive(&ufull_bar[slot]);
        if (unit < 0) break;
        int mt, nt, split;
        unit_coords(unit, shape, num_m, num_n, mt, nt, split);
        const CUtensorMap* tma = (nt >= shape.a2_n_tile) ? &tmA2 : &tmA;
        const int k_begin = split * k_chunk;
        const int k_end = min(shape.K, k_begin + k_chunk);
        const int m0 = mt * PAIR_BM + static_cast<int>(rank) * BM;
        const int n0 = nt * BN + static_cast<int>(rank) * (BN / 2);
        for (int k0 = k_begin; k0 < k_end; k0 += BK, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty_bar[s], ph ^ 1, shape.err, &s_abort, shape.timeout_ns)) { s_abort = 1; break; }
          uint8_t* a_tile = tiles + s * L::STAGE_BYTES;
          uint8_t* b_tile = a_tile + L::A_BYTES;
          if (leader) mbar_arrive_expect_tx(&full_bar[s], 2 * L::STAGE_BYTES);
          const uint32_t fb = mapa_shared(smem_u32(&full_bar[s]), 0);
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < BM / 64; ++c)
              tma_load_2d_pair(a_tile + c * 8192, tma, fb, m0 + 64 * c, k0, pol_a);
          } else {
            tma_load_2d_pair(a_tile, tma, fb, k0, m0, pol_a);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 2 / 64; ++c)
              tma_load_2d_pair_nohint(b_tile + c * 8192, &tmB, fb, n0 + 64 * c, k0);
          } else {
            tma_load_2d_pair_nohint(b_tile, &tmB, fb, k0, n0);
          }
          p_last_issue = globaltimer();
        }
      }
      p_issued = it;
    }
  } else if (warp == 1) {
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
        if (!leader) continue;   // the peer only follows the ring
        // ------------------------- MMA issuer (leader) -------------------------
        int mt, nt, split;
        unit_coords(unit, shape, num_m, num_n, mt, nt, split);
        const int k_begin = split * k_chunk;
        const int k_end = min(shape.K, k_begin + k_chunk);
        bool ok = true;
        const int buf = local & 1;
        if (!mbar_wait(&tempty_bar[buf], ((local >> 1) & 1) ^ 1, shape.err, &s_abort, shape.timeout_ns)) {
          s_abort = 1;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        uint32_t acc = 0;
        for (int k0 = k_begin; k0 < k_end; k0 += BK, ++it) {
          const int s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1;
          if (!mbar_wait(&full_bar[s], ph, shape.err, &s_abort, shape.timeout_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(tiles + s * L::STAGE_BYTES);
          const uint32_t b_addr = a_addr + L::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            const uint64_t ad = A_MN ? desc_mnmajor(a_addr, k) : desc_kmajor(a_addr, k);
            const uint64_t bd = B_MN ? desc_mnmajor(b_addr, k) : desc_kmajor(b_addr, k);
            umma_bf16_pair(d_tmem, ad, bd, IDESC, acc);
            acc = 1;
          }
          umma_commit_pair_both(&empty_bar[s]);   // frees the stage in both CTAs
        }
        if (!ok) { s_abort = 1; break; }
        umma_commit_pair_both(&tfull_bar[buf]);   // both CTAs' accumulators ready
      }
    }
  } else {
    // -------------------------------- epilogue --------------------------------
    const int sub = warp & 3;
    const int part = (warp - 2) >> 2;
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
      ctx.tmem_row = tmem_base + (static_cast<uint32_t>(sub * 32) << 16) + static_cast<uint32_t>(buf * BN);
      ctx.m0 = mt * PAIR_BM + static_cast<int>(rank) * BM;
      ctx.n0 = nt * BN;
      ctx.row = ctx.m0 + sub * 32 + lane;
      ctx.split = split;
      ctx.part = part;
      ctx.parts = PARTS;
      ctx.scratch = smem + L::SCRATCH_OFF + (warp - 2) * EpiScratch<Epi>::value;
      epi(ctx);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&tempty_bar[buf]), 0));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0 && lane == 0 && s_abort && p_issued > 0) {
    if (leader) {
      // Abort path: wait (bounded) for the stages this producer armed; each
      // completes once both CTAs' loads of it have landed.
      for (int d = 0; d < STAGES && d < p_issued; ++d) {
        const int j = p_issued - 1 - d;
        mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1, nullptr, nullptr, GLT_PAIR_DRAIN_NS);
      }
    } else {
      // Abort path: this CTA's loads complete on the leader's barrier, out of
      // its sight; stay (with the leader, through the cluster barrier below)
      // GLT_PAIR_DRAIN_NS past the last one issued.
      while (globaltimer() - p_last_issue < GLT_PAIR_DRAIN_NS) {
      }
    }
  }
  if (warp == 1 && leader && s_abort) {
    // Abort path: no issued pair MMA may still read either CTA's shared
    // memory or write TMEM once the pair passes the cluster barrier.
    tc_fence_after();
    if (lane == 0) {
      umma_commit_pair_local(drain_bar);
      mbar_wait(drain_bar, 0, shape.err, nullptr, GLT_PAIR_DRAIN_NS);
    }
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace tc
}  // namespace glt
