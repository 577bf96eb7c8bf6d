// Cluster split-K bf16 GEMM for few output tiles (small token counts: the single-request path).
//
// A GEMM with M of one or two 128-row blocks has too few output tiles to put every SM on the
// weights. Here a thread-block cluster of C CTAs (C = 1, 2 or 4, CSK_MAX_C) computes one 128 x BN output
// tile (BN = 64 or 128): CTA r of the cluster accumulates the tile over K blocks
// [r * nk / C, (r + 1) * nk / C) in its own TMEM. Rows [s * 128 / C, (s + 1) * 128 / C) of the
// result belong to CTA s: as soon as its accumulator is ready, every CTA stages its partial tile
// from TMEM in its (now idle) pipeline shared memory and sends each owner its rows with one bulk
// copy into the owner's receive buffer (slot = sender's rank), counted on the owner's mbarrier.
// The owner waits for all C slots, adds them in rank order (so the sum does not depend on
// scheduling), applies the GEMM's epilogue and stores to global memory. No workspace, no second
// kernel, and no data leaves the cluster before it is final. Staged rows use a 16-byte-chunk XOR
// swizzle (chunk ^ (row & 7)) so that one-row-per-thread stores do not conflict on banks; the bulk
// copy moves the bytes unchanged and the owner reads them through the same swizzle.
//
// Roles (192 threads):
//   warp 0      TMA producer. The weight (B) tiles of the first stages are requested before the
//               programmatic-dependent-launch wait, since no earlier kernel writes weights; the
//               activation (A) tiles follow once the previous kernel has finished.
//   warp 1      TMEM allocation (BN columns) and tcgen05.mma issue (M = 128, N = BN, K = 16).
//   warps 2..5  TMEM -> staging (one row per thread), then one bulk copy per owner and warp.
//   all         the rank-order sum and the epilogue (8 output columns per work item); each
//               thread fetches the side inputs of its next item (residual rows, RoPE sin / cos,
//               bias) while the partial tiles are still on their way.
//
// Epilogues are those of the persistent kernel (gemm_sm100.cuh): EPI_STORE (bias, ReLU / GELU,
// bf16 or fp32 out), EPI_ROPE (rotate-half RoPE of q/k heads, split_rope.metal:46-76), EPI_GEGLU
// (gelu_erf(input) * gate, lib.rs:494-510; a 128-wide tile is 64 input rows of Wi loaded next to
// the 64 matching gate rows, two TMA boxes of the 128 | 128 interleaved weight), EPI_RESID
// (fp32 residual += result, lib.rs:1375-1390; one owner per element, so one deterministic add) and
// EPI_RESID16 (the f16 residual stream: f16(residual + result), one rounding).
//
// Every wait is bounded (common.cuh); on a timeout a role stops issuing work, but every thread still
// passes both cluster barrier phases, so no CTA of the cluster is left waiting.
#pragma once
#include "gemm_sm100.cuh"
#include "gemm_sm100_2cta.cuh"

namespace s1c {

struct CskArgs {
  int M, N, K;
  int C;              // CTAs per cluster = K splits (1, 2 or 4); the grid is tiles * C CTAs
  void* out;          // bf16 output, fp32 (EPI_RESID, or EPI_STORE with out_f32), f16 (EPI_RESID16)
  int ldo;            // output row pitch in elements
  const float* bias;  // EPI_STORE / EPI_RESID / EPI_RESID16, optional
  int act;            // EPI_STORE
  int out_f32;        // EPI_STORE
  const int* pos;     // EPI_ROPE
  const float* inv_freq;
  int rope_cols;
  int out_cols;       // EPI_GEGLU: I
  int* status;
  // The next GEMM's weights, prefetched into L2 while this one runs (null = none); a multiple of
  // 16 bytes at a 16-byte-aligned address.
  const void* pf;
  size_t pf_bytes;
};

// Largest cluster the launch plan uses. In the single-request forward (CUDA graph, weights streaming from HBM) clusters of 8 measured slower than
// clusters of at most 4 (128 tokens: 1.53 vs 1.26 ms per forward; 200 tokens: 2.03 vs 1.51 ms): the
// partial-tile exchange grows with C while the weight stream is already spread over the SMs.
constexpr int CSK_MAX_C = 4;

template <int BN>
__host__ __device__ constexpr size_t csk_smem_bytes() {
  // pipeline stages + receive buffer (C slots x 128/C rows x BN fp32 = 128 x BN fp32) + barriers
  return (size_t)GEMM_STAGES * (GEMM_BM * GEMM_BK * 2 + BN * GEMM_BK * 2) + (size_t)GEMM_BM * BN * 4 +
         1024 /*align*/ + 256 /*barriers*/;
}

S1C_DEV void cluster_arrive_release() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
S1C_DEV void cluster_wait_acquire() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

S1C_DEV void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }

// Bulk copy of `bytes` (a multiple of 16) from this CTA's shared memory into the shared memory of a
// CTA of this cluster; the bytes are counted (complete_tx) on the mbarrier at `remote_bar`, which
// lives in the same CTA as `remote_dst`.
S1C_DEV void bulk_copy_to_peer(uint32_t remote_dst, const void* src, uint32_t bytes, uint32_t remote_bar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   remote_dst),
               "r"(smem_u32(src)), "r"(bytes), "r"(remote_bar)
               : "memory");
}

// Warp-collective bounded wait on a barrier that other CTAs of the cluster complete; acquire at
// cluster scope so their stores are visible afterwards.
S1C_DEV bool mbar_wait_cluster_warp(uint64_t* bar, uint32_t parity, int* status, int code, volatile int* abort) {
  const uint32_t a = smem_u32(bar);
  const int lane = threadIdx.x & 31;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (__all_sync(0xffffffffu, ok != 0)) return true;
    if ((it & 63u) == 63u) {
      int give_up = 0;
      if (lane == 0) {
        const uint64_t now = globaltimer();
        if (t0 == 0) t0 = now;
        if (now - t0 > S1C_WAIT_BUDGET_NS) give_up = 1;
      }
      give_up = __shfl_sync(0xffffffffu, give_up, 0);
      if (give_up) {
        if (lane == 0) {
          report(status, code);
          if (abort) *abort = 1;
        }
        return false;
      }
    }
  }
}

S1C_DEV void store_bf16x8(__nv_bfloat16* dst, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                              pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

// Rank-order sum over the C received slots of the 8 floats [c, c + 8) (c a multiple of 8) of row
// `lr` of a slot; rows are BN floats with 16-byte chunks swizzled by (row & 7).
template <int BN>
S1C_DEV void csk_sum8(const float* recv, int C, uint32_t slot_floats, int lr, int c, float (&v)[8]) {
  const int sw = lr & 7;
  const uint32_t o0 = (uint32_t)lr * BN + (uint32_t)((((c >> 2)) ^ sw) << 2);
  const uint32_t o1 = (uint32_t)lr * BN + (uint32_t)((((c >> 2) + 1) ^ sw) << 2);
  float4 a = *reinterpret_cast<const float4*>(recv + o0), b = *reinterpret_cast<const float4*>(recv + o1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
#pragma unroll 1
  for (int s = 1; s < C; ++s) {
    a = *reinterpret_cast<const float4*>(recv + (size_t)s * slot_floats + o0);
    b = *reinterpret_cast<const float4*>(recv + (size_t)s * slot_floats + o1);
    v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w; v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
  }
}

// One epilogue work item: row `lr` of this CTA's share, unit `u` (8 output columns; RoPE: 8
// columns of a head's first half and their partners 32 columns on). `side` holds what the item
// needs from global memory besides the partial sums, fetched ahead: the residual row values
// (EPI_RESID), the bias (EPI_STORE / EPI_RESID), or cos / sin of the RoPE angles (EPI_ROPE).
struct CskItem {
  int lr, u, grow, col;  // col: output column of the first element; -1 = nothing to do
  float side[16];
};

template <int BN, int EPI>
S1C_DEV int csk_units() { return EPI == EPI_ROPE || EPI == EPI_GEGLU ? BN / 16 : BN / 8; }

template <int BN, int EPI>
S1C_DEV void csk_prepare(const CskArgs& args, int it, int R, int row0, int n0, int n_block, CskItem& x) {
  constexpr int UNITS = EPI == EPI_ROPE || EPI == EPI_GEGLU ? BN / 16 : BN / 8;
  x.col = -1;
  if (it >= R * UNITS) return;
  x.lr = it / UNITS;
  x.u = it % UNITS;
  x.grow = row0 + x.lr;
  if (x.grow >= args.M) return;
  if constexpr (EPI == EPI_ROPE) {
    const int hh = x.u >> 2, j0 = (x.u & 3) * 8, gcol = n0 + hh * 64 + j0;
    if (gcol >= args.N) return;
    x.col = gcol;
    if (n0 + hh * 64 < args.rope_cols) {
      const float p = (float)__ldg(args.pos + x.grow);
#pragma unroll
      for (int i = 0; i < 8; ++i) sincosf(p * __ldg(args.inv_freq + j0 + i), &x.side[8 + i], &x.side[i]);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        x.side[i] = 1.f;
        x.side[8 + i] = 0.f;
      }
    }
  } else if constexpr (EPI == EPI_GEGLU) {
    const int ocol = n_block * (BN / 2) + x.u * 8;
    if (ocol >= args.out_cols) return;
    x.col = ocol;
  } else {
    const int gcol = n0 + x.u * 8;
    if (gcol >= args.N) return;
    x.col = gcol;
    if (args.bias) {
      const float4 b0 = __ldg(reinterpret_cast<const float4*>(args.bias + gcol));
      const float4 b1 = __ldg(reinterpret_cast<const float4*>(args.bias + gcol + 4));
      x.side[0] = b0.x; x.side[1] = b0.y; x.side[2] = b0.z; x.side[3] = b0.w;
      x.side[4] = b1.x; x.side[5] = b1.y; x.side[6] = b1.z; x.side[7] = b1.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) x.side[i] = 0.f;
    }
    if constexpr (EPI == EPI_RESID) {
      const float4* o = reinterpret_cast<const float4*>(static_cast<const float*>(args.out) + (size_t)x.grow * args.ldo + gcol);
      const float4 h0 = o[0], h1 = o[1];
      x.side[8] = h0.x; x.side[9] = h0.y; x.side[10] = h0.z; x.side[11] = h0.w;
      x.side[12] = h1.x; x.side[13] = h1.y; x.side[14] = h1.z; x.side[15] = h1.w;
    } else if constexpr (EPI == EPI_RESID16) {
      const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const __half*>(args.out) + (size_t)x.grow * args.ldo + gcol);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_f16x2(w[i]);
        x.side[8 + 2 * i] = f.x;
        x.side[9 + 2 * i] = f.y;
      }
    }
  }
}

template <int BN, int EPI>
S1C_DEV void csk_finish(const CskArgs& args, const float* recv, int C, uint32_t slot_floats, const CskItem& x) {
  if (x.col < 0) return;
  if constexpr (EPI == EPI_ROPE) {
    const int col = (x.u >> 2) * 64 + (x.u & 3) * 8;
    float a[8], b[8];
    csk_sum8<BN>(recv, C, slot_floats, x.lr, col, a);
    csk_sum8<BN>(recv, C, slot_floats, x.lr, col + 32, b);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float p = a[i], q = b[i], cs = x.side[i], sn = x.side[8 + i];
      a[i] = p * cs - q * sn;
      b[i] = p * sn + q * cs;
    }
    __nv_bfloat16* o = static_cast<__nv_bfloat16*>(args.out) + (size_t)x.grow * args.ldo + x.col;
    store_bf16x8(o, a);
    store_bf16x8(o + 32, b);
  } else if constexpr (EPI == EPI_GEGLU) {
    float a[8], g[8];
    csk_sum8<BN>(recv, C, slot_floats, x.lr, x.u * 8, a);
    csk_sum8<BN>(recv, C, slot_floats, x.lr, BN / 2 + x.u * 8, g);
#pragma unroll
    for (int i = 0; i < 8; ++i) a[i] = gelu_erf(a[i]) * g[i];
    store_bf16x8(static_cast<__nv_bfloat16*>(args.out) + (size_t)x.grow * args.ldo + x.col, a);
  } else {
    float v[8];
    csk_sum8<BN>(recv, C, slot_floats, x.lr, x.u * 8, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] += x.side[i];
    if constexpr (EPI == EPI_RESID) {
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(args.out) + (size_t)x.grow * args.ldo + x.col);
      o[0] = make_float4(x.side[8] + v[0], x.side[9] + v[1], x.side[10] + v[2], x.side[11] + v[3]);
      o[1] = make_float4(x.side[12] + v[4], x.side[13] + v[5], x.side[14] + v[6], x.side[15] + v[7]);
    } else if constexpr (EPI == EPI_RESID16) {
      // f16(residual + (acc + bias)): the sum rounded once
      *reinterpret_cast<uint4*>(static_cast<__half*>(args.out) + (size_t)x.grow * args.ldo + x.col) =
          make_uint4(pack_f16x2(x.side[8] + v[0], x.side[9] + v[1]), pack_f16x2(x.side[10] + v[2], x.side[11] + v[3]),
                     pack_f16x2(x.side[12] + v[4], x.side[13] + v[5]), pack_f16x2(x.side[14] + v[6], x.side[15] + v[7]));
    } else {
      if (args.act == ACT_RELU) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = fmaxf(v[i], 0.f);
      } else if (args.act == ACT_GELU) {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = gelu_erf(v[i]);
      }
      if (args.out_f32) {
        float4* o = reinterpret_cast<float4*>(static_cast<float*>(args.out) + (size_t)x.grow * args.ldo + x.col);
        o[0] = make_float4(v[0], v[1], v[2], v[3]);
        o[1] = make_float4(v[4], v[5], v[6], v[7]);
      } else {
        store_bf16x8(static_cast<__nv_bfloat16*>(args.out) + (size_t)x.grow * args.ldo + x.col, v);
      }
    }
  }
}

// tmB: the weight with boxes of BN rows (GeGLU: of BN / 2 rows, loaded twice per stage).
template <int BN, int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_csk_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const CskArgs args) {
  constexpr int BM = GEMM_BM, BK = GEMM_BK, STAGES = GEMM_STAGES;
  constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
  static_assert(BN == 64 || BN == 128, "cluster split-K tiles are 128 x 64 or 128 x 128");
  static_assert(EPI != EPI_GEGLU || BN == 128, "GeGLU tiles are 64 input + 64 gate columns");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_u + 1023u) & ~1023u) - raw_u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  float* recv = reinterpret_cast<float*>(sB + STAGES * B_BYTES);  // [C][128 / C][BN]
  uint64_t* full = reinterpret_cast<uint64_t*>(recv + BM * BN);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* drain = tfull + 1;
  uint64_t* rbar = drain + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = args.C;
  const int rank = (int)cluster_ctarank();
  const int tile = blockIdx.x / C;
  const int num_n = (args.N + BN - 1) / BN;
  const int m0 = (tile / num_n) * BM, n_block = tile % num_n, n0 = n_block * BN;
  const int nk = (args.K + BK - 1) / BK;
  const int kb0 = rank * nk / C, nkb = (rank + 1) * nk / C - kb0;
  const int R = BM / C;  // rows owned by each CTA
  const uint32_t slot_floats = (uint32_t)(R * BN);

  // The next GEMM's weights into L2 (independent of every earlier kernel, so before the dependency
  // wait), issued by an epilogue thread that is idle until the mainloop ends.
  if (threadIdx.x == 64 && args.pf) prefetch_l2_share(args.pf, args.pf_bytes);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(drain, 1);
    mbar_init(rbar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    // The whole tile's worth of partial rows (C senders x R rows x BN fp32) completes the barrier.
    mbar_arrive_expect_tx(rbar, (uint32_t)(BM * BN * 4));
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // Phase 1 of the cluster barrier: every CTA's receive barrier is initialised (and the init fenced
  // at cluster scope above) before any CTA copies into it; the matching wait comes right before
  // the first copy.
  cluster_arrive_relaxed();
  const uint32_t tmem_base = *tmem_slot;
  pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmA);
      prefetch_tmap(&tmB);
      auto load_b = [&](int s, int kb) {
        if constexpr (EPI == EPI_GEGLU) {
          // tile n_block: Wi rows (n_block / 2) * 256 + (n_block % 2) * 64 + [0, 64) and the gate
          // rows 128 further; output columns n_block * 64 + [0, 64)
          const int r0 = (n_block >> 1) * 256 + (n_block & 1) * 64;
          tma_load_2d(sB + s * B_BYTES, &tmB, &full[s], kb * BK, r0);
          tma_load_2d(sB + s * B_BYTES + B_BYTES / 2, &tmB, &full[s], kb * BK, r0 + 128);
        } else {
          tma_load_2d(sB + s * B_BYTES, &tmB, &full[s], kb * BK, n0);
        }
      };
      const int pre = nkb < STAGES ? nkb : STAGES;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], STAGE_BYTES);
        load_b(i, kb0 + i);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) tma_load_2d(sA + i * A_BYTES, &tmA, &full[i], (kb0 + i) * BK, m0);
      int issued = pre;
      for (int i = pre; i < nkb; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&empty[s], ((i / STAGES) & 1) ^ 1u, args.status, DEV_TIMEOUT_PRODUCER, abort_flag)) break;
        mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
        load_b(s, kb0 + i);
        tma_load_2d(sA + s * A_BYTES, &tmA, &full[s], (kb0 + i) * BK, m0);
        ++issued;
      }
      // Loads in flight land before the CTA exits.
      for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
        mbar_wait(&full[j % STAGES], (j / STAGES) & 1, args.status, DEV_TIMEOUT_DRAIN, nullptr);
    }
    __syncwarp();
    cluster_wait_acquire();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      bool ok = true;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait(&full[s], (i / STAGES) & 1, args.status, DEV_TIMEOUT_MMA_FULL, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a0 = smem_u32(sA + s * A_BYTES), b0 = smem_u32(sB + s * B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          umma_bf16(tmem_base, sdesc_kmajor_sw128(a0 + k * 32), sdesc_kmajor_sw128(b0 + k * 32), idesc,
                    (i != 0 || k != 0) ? 1u : 0u);
        umma_commit(&empty[s]);
      }
      if (ok) umma_commit(tfull);
      umma_commit(drain);
      mbar_wait(drain, 0, args.status, DEV_TIMEOUT_DRAIN, nullptr);
    }
    __syncwarp();
    cluster_wait_acquire();
  } else {
    const int quad = warp & 3;  // TMEM lanes [32 * quad, 32 * quad + 32) = tile rows
    const int row = quad * 32 + lane;
    const bool ok = mbar_wait_warp(tfull, 0, args.status, DEV_TIMEOUT_EPILOGUE, abort_flag);
    cluster_wait_acquire();
    if (ok) {
      tc_fence_after();
      // Stage this warp's 32 rows of the partial tile in the idle pipeline buffers (every MMA of
      // this CTA has completed, so every load has landed and no tensor-core read is pending).
      float* stg = reinterpret_cast<float*>(smem);
      const uint32_t t = tmem_base + ((uint32_t)(quad * 32) << 16);
      float* dst = stg + (size_t)row * BN;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        float v[32];
        tmem_ld32(t + c * 32, v);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(dst + (((c * 8 + j) ^ (row & 7)) << 2)) =
              make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
      }
      fence_proxy_async();  // the staged rows are read next by the bulk-copy (async) proxy
      __syncwarp();
      if (lane == 0) {
        // rows [32 quad, 32 quad + 32) go to owners row / R, one contiguous copy per owner
        for (int r = quad * 32; r < quad * 32 + 32;) {
          const int o = r / R, r_end = min(quad * 32 + 32, (o + 1) * R), lr = r - o * R;
          const uint32_t d = map_to_rank(smem_u32(recv + (size_t)rank * slot_floats + (size_t)lr * BN), (uint32_t)o);
          bulk_copy_to_peer(d, stg + (size_t)r * BN, (uint32_t)((r_end - r) * BN * 4), map_to_rank(smem_u32(rbar), (uint32_t)o));
          r = r_end;
        }
        bulk_commit();
        bulk_wait_all();  // the staged rows have been read (and delivered) before the CTA moves on
      }
      __syncwarp();
    }
    tc_fence_before();
  }

  // ---- rank-order sum of the received slots and the epilogue: rows [rank * R, rank * R + R) ---
  pdl_wait();  // every thread passes the dependency wait before touching global memory
  {
    const int total = R * csk_units<BN, EPI>();
    CskItem cur, nxt;
    csk_prepare<BN, EPI>(args, threadIdx.x, R, m0 + rank * R, n0, n_block, cur);
    if (mbar_wait_cluster_warp(rbar, 0, args.status, DEV_TIMEOUT_EPILOGUE, abort_flag)) {
#pragma unroll 1
      for (int it = threadIdx.x; it < total; it += GEMM_THREADS) {
        csk_prepare<BN, EPI>(args, it + GEMM_THREADS, R, m0 + rank * R, n0, n_block, nxt);
        csk_finish<BN, EPI>(args, recv, C, slot_floats, cur);
        cur = nxt;
      }
    }
  }
  // Phase 2: no CTA leaves while a peer may still push into its shared memory.
  __syncwarp();
  cluster_arrive_release();
  cluster_wait_acquire();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, BN);
  }
}

}  // namespace s1c
