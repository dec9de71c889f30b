// Two-CTA tcgen05 GEMM (`cta_group::2`): a cluster of two CTAs on two SMs
// computes a 256 x 256 output tile with one MMA stream, C = A * W^T.
//
// Why: with one CTA per 128 x 256 tile, every K step reads a 128-row A slice
// and the whole 256-row W slice from shared memory; the tensor core's
// shared-memory read port was ~85-90 % busy (ncu: sm__mem_tensor_cycles_active).
// With a CTA pair each SM stages only its half of W (128 rows) and the pair's
// MMA reads each half once for both SMs: per FLOP a third less shared-memory
// and L2->SM traffic.
//
// Split (the 2x1-SM MMA layout): CTA r of the pair holds A rows
// [256m + 128r, +128) and W rows [256n + 128r, +128) of every K block, and
// receives accumulator rows [128r, +128) x all 256 columns in its own tensor
// memory.  Roles per CTA (320 threads):
//   warp 0      : TMA producer for this CTA's halves; both CTAs' loads complete
//                 on the leader's (rank 0) full barrier, which the leader arms
//                 with the pair's total bytes
//   warp 1      : TMEM allocation (both CTAs, cta_group::2); in the leader, one
//                 lane issues the pair's MMAs and commits to the empty / full
//                 barriers of both CTAs (tcgen05.commit multicast)
//   warps 2..9  : epilogue of this CTA's 128 rows (as the one-CTA kernel);
//                 they release an accumulator by arriving on the leader's
//                 acc_empty barrier (remote arrive from rank 1)
// No TMA load uses cluster multicast: each CTA loads its own halves.
// Every wait is bounded; both CTAs meet at a cluster barrier before exit, so
// neither leaves while the other may still touch its shared memory.
#pragma once

#include "gemm.cuh"

namespace vd {

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of `local`'s counterpart in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (this CTA's or the peer's).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Bounded wait (as mbar_wait) with cluster-scope acquire, for barriers that
// the other CTA of the pair arrives on.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                                  int code, uint64_t limit_ns = 0) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t limit = limit_ns ? limit_ns : VD_WAIT_TIMEOUT_NS;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit) {
      *abort_flag = 1;
      record_error(err, code);
      return false;
    }
  }
}

// 2-D tile load into this CTA's shared memory whose completion is signalled on
// an mbarrier of either CTA of the pair (cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

// The same load with an L2 eviction-priority hint (a createpolicy value).
__device__ __forceinline__ void tma_load_2d_pair_hint(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                      int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// The pair's MMA (issued by the leader): D (256 x N over both CTAs' TMEM) (+)= A * B^T.
__device__ __forceinline__ void umma_f16kind_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at this shared offset in every CTA of `mask`
// when the pair's MMAs issued so far have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

struct Gemm2Config {
  static constexpr int BM = 128;       // rows per CTA (256 per pair)
  static constexpr int BN = 256;       // output columns per tile
  static constexpr int BK = 64;
  static constexpr int STAGES = 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;  // this CTA's half of W
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int PAIR_STAGE_BYTES = 2 * STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int BAR_BYTES = 1024;
  static constexpr int EPI_WARPS = 8;
  static constexpr int EPI_STAGE_BYTES = 4096;
  static constexpr int SMEM_BYTES =
      1024 /*alignment slack*/ + STAGES * STAGE_BYTES + BAR_BYTES + EPI_WARPS * EPI_STAGE_BYTES;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int GROUP_M = 16;   // pair tiles (256 rows) per raster group
};

// tmB: W with 128-row boxes (a CTA's half of a 256-row tile).
template <int EPI, class T>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Gemm2Config::THREADS, 1)
    gemm2_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                         GemmShape shape, EpiParams ep, int* err) {
  using Cfg = Gemm2Config;
  constexpr int BM = Cfg::BM, BN = Cfg::BN, BK = Cfg::BK, STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = umma_idesc_f16kind(2 * BM, BN, Elem<T>::kUmmaFormat);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* epi_ld = acc_empty + 3;  // [EPI_WARPS] TMA loads of the residual (kEpiResidualNorm)
  uint8_t* epi_stage = smem + STAGES * Cfg::STAGE_BYTES + Cfg::BAR_BYTES;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);   // the leader's arm; both CTAs' bytes complete it
      mbar_init(&empty[s], 1);  // the leader's MMA commit, multicast to both CTAs
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&acc_full[j], 1);
      mbar_init(&acc_empty[j], 2 * Cfg::EPI_WARPS);  // epilogue warps of both CTAs (leader's copy is used)
    }
    for (int w = 0; w < Cfg::EPI_WARPS; ++w) mbar_init(&epi_ld[w], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched with programmatic stream serialization, the set-up above ran
  // under the previous kernel's tail.  Every role waits for that kernel's
  // results before it touches global memory; the producer first loads the
  // weight tiles of its first k-blocks, which do not depend on it.
  pdl_trigger_next();

  const int num_m = (shape.M + 2 * BM - 1) / (2 * BM);
  const int num_n = shape.N / BN;
  const int tiles = num_m * num_n;
  const int kblocks = shape.K / BK;
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      tma_prefetch_desc(&tmC);
      if constexpr (EPI == kEpiResidualNorm) tma_prefetch_desc(&tmD);
      const uint64_t pol_keep = l2_policy_evict_last(), pol_stream = l2_policy_evict_first();
      // The first tile's first `pre` stages (all free: nothing has used them
      // yet) get their W halves now and their A rows after the wait.
      int pre = 0;
      if (pair < tiles) {
        int m, n;
        tile_coords(pair, num_m, num_n, shape.group_m, m, n);
        const int yb = n * BN + static_cast<int>(rank) * (BN / 2);
        pre = kblocks < STAGES ? kblocks : STAGES;
        for (int kb = 0; kb < pre; ++kb) {
          if (leader) mbar_arrive_expect_tx(&full[kb], Cfg::PAIR_STAGE_BYTES);
          const uint32_t bar = mapa_shared(smem_u32(&full[kb]), 0);
          if (shape.l2_hints) tma_load_2d_pair_hint(sB + kb * Cfg::B_BYTES, &tmB, bar, kb * BK, yb, pol_stream);
          else tma_load_2d_pair(sB + kb * Cfg::B_BYTES, &tmB, bar, kb * BK, yb);
        }
      }
      pdl_wait_prior();
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = pair; tile < tiles; tile += pairs) {
        int m, n;
        tile_coords(tile, num_m, num_n, shape.group_m, m, n);
        const int ya = m * 2 * BM + static_cast<int>(rank) * BM;
        const int yb = n * BN + static_cast<int>(rank) * (BN / 2);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_cluster(&empty[stage], phase ^ 1, abort_flag, err, kErrTimeoutEmpty, shape.wait_ns)) goto producer_done;
          const bool w_loaded = tile == pair && kb < pre;
          if (leader && !w_loaded) mbar_arrive_expect_tx(&full[stage], Cfg::PAIR_STAGE_BYTES);
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
          if (shape.l2_hints) {
            // A rows are reused by every N tile of the raster group (long reuse
            // distance): keep them; W tiles are used by the group's M tiles at
            // about the same time and then not again for a while.
            tma_load_2d_pair_hint(sA + stage * Cfg::A_BYTES, &tmA, bar, kb * BK, ya, pol_keep);
            if (!w_loaded) tma_load_2d_pair_hint(sB + stage * Cfg::B_BYTES, &tmB, bar, kb * BK, yb, pol_stream);
          } else {
            tma_load_2d_pair(sA + stage * Cfg::A_BYTES, &tmA, bar, kb * BK, ya);
            if (!w_loaded) tma_load_2d_pair(sB + stage * Cfg::B_BYTES, &tmB, bar, kb * BK, yb);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Drain: every stage this CTA filled has been consumed by the pair's MMAs
      // (the leader's commit arrives here too) before the CTA may exit.
      for (int i = 0; i < STAGES; ++i) {
        if (!mbar_wait_cluster(&empty[stage], phase ^ 1, abort_flag, err, kErrTimeoutEmpty, shape.wait_ns)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = pair; tile < tiles; tile += pairs) {
        if (!mbar_wait_cluster(&acc_empty[acc], acc_phase ^ 1, abort_flag, err, kErrTimeoutAccEmpty, shape.wait_ns)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_cluster(&full[stage], phase, abort_flag, err, kErrTimeoutFull, shape.wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_f16kind_pair(d_tmem, sw128_kmajor_desc(a_addr + k * 32), sw128_kmajor_desc(b_addr + k * 32), IDESC,
                              (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair(&empty[stage], 0x3);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair(&acc_full[acc], 0x3);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else {
    pdl_wait_prior();
    // Epilogue warps 2..9 of this CTA's 128 accumulator rows (TMEM lane
    // quarter warp % 4, column half (warp - 2) / 4).
    const int lane_group = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = lane_group * 32 + lane;
    EpiOut o{epi_stage + (warp - 2) * Cfg::EPI_STAGE_BYTES, &tmC, 0, lane, 0, &tmD, &epi_ld[warp - 2], 0u,
             shape.wait_ns, err};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = pair; tile < tiles; tile += pairs) {
      int m, n;
      tile_coords(tile, num_m, num_n, shape.group_m, m, n);
      if (!mbar_wait_cluster(&acc_full[acc], acc_phase, abort_flag, err, kErrTimeoutAccFull, shape.wait_ns)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + acc * BN + (static_cast<uint32_t>(lane_group * 32) << 16);
      const int row0 = m * 2 * BM + static_cast<int>(rank) * BM;
      const int row = row0 + row_in_tile;
      o.y = row0 + lane_group * 32;
      gemm_epilogue<BN, EPI, T>(o, taddr, row, row < shape.M, n * BN, half, ep);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&acc_empty[acc]), 0));
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still read or signal its shared memory
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace vd
