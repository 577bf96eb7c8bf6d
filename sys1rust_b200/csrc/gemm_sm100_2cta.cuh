// Two-CTA variant of the persistent bf16 GEMM (gemm_sm100.cuh): a cluster of 2 CTAs on 2 SMs
// computes one 256 x 256 tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16 per
// instruction). Each CTA loads only its own 128 rows of A and its own 128 rows of B (plain TMA
// tile loads from local HBM, no multi-destination forms); the MMA issued by the cluster's first
// CTA reads both CTAs' shared memory and leaves each CTA's 128 x 256 accumulator in its own TMEM.
// Per SM that is 32 KB of operands per 64-wide K step instead of 48 KB for the one-CTA 128 x 256
// tile, for the same tensor work, which is what lets the mainloop keep the tensor pipe busy.
//
// Roles per CTA (192 threads), as in the one-CTA kernel:
//   warp 0      TMA producer: 6-stage ring; both CTAs' loads complete on the first CTA's "full"
//               barrier (which expects the bytes of both); each CTA waits on its own "empty".
//   warp 1      TMEM owner (cta_group::2 allocation of 512 columns in both CTAs); in the first
//               CTA it also issues the MMAs and commits to the barriers of both CTAs.
//   warps 2..5  epilogue on this CTA's accumulator rows (shared epilogue code), then arrive on the
//               first CTA's "tmem empty" barrier (256 arrivals: both CTAs' epilogue threads).
#pragma once
#include "gemm_sm100.cuh"

namespace s1c {

constexpr int GEMM2_STAGES = 6;

__host__ __device__ constexpr size_t gemm2_smem_bytes() {
  return (size_t)GEMM2_STAGES * (128 * 64 * 2 + 128 * 64 * 2) + 8 * GEMM_STG_BYTES + 1024 + 256;
}

S1C_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
S1C_DEV uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
S1C_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
S1C_DEV void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
S1C_DEV void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
S1C_DEV void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
S1C_DEV void umma2_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on the barrier at shared::cluster address `cbar` once this thread's prior tcgen05 ops finish.
S1C_DEV void umma2_commit(uint32_t cbar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cbar) : "memory");
}
// TMA tile load into this CTA's shared memory whose completion is counted on the barrier at
// shared::cluster address `cbar` (the first CTA's "full" barrier).
S1C_DEV void tma_load_2d_cg2(void* dst, const void* tmap, uint32_t cbar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(cbar), "r"(x), "r"(y)
      : "memory");
}
S1C_DEV void mbar_arrive_cluster(uint32_t cbar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cbar) : "memory");
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM_THREADS, 1)
    gemm2_bf16_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  constexpr int BK = GEMM_BK, STAGES = GEMM2_STAGES, BN = 256;
  constexpr uint32_t A_BYTES = 128 * BK * 2, B_BYTES = 128 * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 512;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_u + 1023u) & ~1023u) - raw_u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sStg = sB + STAGES * B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sStg + 8 * GEMM_STG_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
  const int num_m = (args.M + 255) / 256, num_n = (args.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int nk = (args.K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 256);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc2(tmem_slot, TMEM_COLS);
    tmem_relinquish2();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised and TMEM allocated before any use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      int s = 0, issued = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int tile = cluster; ok && tile < num_tiles; tile += n_clusters) {
        const int m0 = (tile / num_n) * 256 + (int)rank * 128, n0 = (tile % num_n) * BN + (int)rank * 128;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, args.status, DEV_TIMEOUT_PRODUCER, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t cfull = map_to_rank(smem_u32(&full[s]), 0);
          if (leader) mbar_arrive_expect_tx(&full[s], 2 * STAGE_BYTES);
          tma_load_2d_cg2(sA + s * A_BYTES, &tmA, cfull, kb * BK, m0);
          tma_load_2d_cg2(sB + s * B_BYTES, &tmB, cfull, kb * BK, n0);
          ++issued;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // Drain: every stage this CTA loaded is consumed (hence landed) before the CTA exits.
      int back = issued < STAGES ? issued : STAGES;
      int ss = s;
      uint32_t pp = ph;
      for (int i = 0; i < back; ++i) {
        if (--ss < 0) {
          ss = STAGES - 1;
          pp ^= 1u;
        }
        mbar_wait(&empty[ss], pp, args.status, DEV_TIMEOUT_DRAIN, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_bf16_f32(256, BN);
      // Stage 0's descriptors built once; a stage's are these plus its byte offset >> 4 (see the
      // one-CTA kernel); the empty / tfull barriers' cluster addresses are mapped once too.
      const uint64_t adesc0 = sdesc_kmajor_sw128(smem_u32(sA)), bdesc0 = sdesc_kmajor_sw128(smem_u32(sB));
      const uint32_t e0r0 = map_to_rank(smem_u32(&empty[0]), 0), e0r1 = map_to_rank(smem_u32(&empty[0]), 1);
      int s = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      for (int tile = cluster; ok && tile < num_tiles; tile += n_clusters) {
        if (!mbar_wait(&tempty[acc], aph ^ 1u, args.status, DEV_TIMEOUT_MMA_TEMPTY, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[s], ph, args.status, DEV_TIMEOUT_MMA_FULL, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = adesc0 + (uint64_t)(s * (A_BYTES >> 4)), bd = bdesc0 + (uint64_t)(s * (B_BYTES >> 4));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) umma2_bf16(d, ad + 2u * k, bd + 2u * k, idesc, (kb | k) != 0 ? 1u : 0u);
          umma2_commit(e0r0 + 8u * (uint32_t)s);
          umma2_commit(e0r1 + 8u * (uint32_t)s);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t tf = smem_u32(&tfull[acc]);
        umma2_commit(map_to_rank(tf, 0));
        umma2_commit(map_to_rank(tf, 1));
        acc ^= 1;
        if (acc == 0) aph ^= 1u;
      }
      umma2_commit(map_to_rank(smem_u32(drain), 0));
      mbar_wait(drain, 0, args.status, DEV_TIMEOUT_DRAIN, nullptr);
    }
  } else {
    const int quad = warp & 3;
    Stager sg{sStg + (warp - 2) * 2 * GEMM_STG_BYTES, 0u, lane, 2};
    if (lane == 0) prefetch_tmap(&tmC);
    int acc = 0;
    uint32_t aph = 0;
    for (int tile = cluster; tile < num_tiles; tile += n_clusters) {
      const int m0 = (tile / num_n) * 256 + (int)rank * 128, n_block = tile % num_n;
      const int y0 = m0 + quad * 32;
      const int row = y0 + lane;
      RopeRow rr;
      if constexpr (EPI == EPI_ROPE) rope_prefetch(args, row, row < args.M, n_block * BN, rr);
      if (!mbar_wait_warp(&tfull[acc], aph, args.status, DEV_TIMEOUT_EPILOGUE, abort_flag)) break;
      tc_fence_after();
      const uint32_t t = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      gemm_epilogue_tile<BN, EPI>(args, &tmC, sg, t, row, row < args.M, y0, n_block * BN, n_block, 0, 1, rr);
      tc_fence_before();
      mbar_arrive_cluster(map_to_rank(smem_u32(&tempty[acc]), 0));
      acc ^= 1;
      if (acc == 0) aph ^= 1u;
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while the other may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, TMEM_COLS);
  }
}

}  // namespace s1c
