// Varlen flash attention on the 5th-generation tensor cores (tcgen05), head_dim 64.
//
// Same contract as attention.cuh (the key sets of the reference's masked SDPA calls,
// runtime/crates/laya-mlx/src/lib.rs:1644-1657, :1399-1417, :1711-1760): a query at position i of
// a row attends the keys j of the same row, all of them (global layers, head layers) or those
// with |i - j| <= window (local layers); softmax in fp32, output bf16.
//
// One CTA = one tile of up to 128 query rows x ATTC_HEADS heads, processed head after head so
// the TMA/MMA pipeline never drains between heads; two CTAs share an SM (96 KB of shared memory
// and 256 TMEM columns each). 192 threads:
//   warp 0      TMA producer: Q tile [128 x 64] per head (double buffered), K and V tiles
//               [64 keys x 64] per key step (2-stage ring), 128-byte swizzle.
//   warp 1      TMEM owner and MMA issuer:
//                 S = Q K^T        M=128 N=64 K=64   (K-major A and B)          -> TMEM cols [0,64)
//                 O_j = P_j V_j    M=128 N=64 K=64   (P K-major from smem, V MN-major) -> TMEM
//                                  cols [64,128) / [128,192) alternating
//               S of the next key step is issued as soon as the softmax has read the current S.
//   warps 2..5  softmax, one query row per thread (TMEM lane = row): masks only on tiles that
//               cross a row's key range, online max / sum in fp32 with p = 2^(s*scale - m) (one
//               FFMA and one ex2 per score), P rounded to bf16 into one of two shared-memory
//               buffers in the swizzled K-major layout the MMA reads, O_j folded into a register
//               accumulator with the running correction, final O / l stored bf16.
#pragma once
#include <cuda.h>
#include "common.cuh"

namespace s1c {

constexpr int ATTC_BQ = 128, ATTC_BK = 64, ATTC_THREADS = 192, ATTC_HEADS = 4, ATTC_KV_STAGES = 2;
constexpr uint32_t ATTC_Q_BYTES = ATTC_BQ * 64 * 2;       // 16 KB
constexpr uint32_t ATTC_KV_BYTES = ATTC_BK * 64 * 2;      // 8 KB each for K and V
constexpr uint32_t ATTC_P_BYTES = ATTC_BQ * ATTC_BK * 2;  // 16 KB: one swizzled [128 x 64] block (x2)
constexpr size_t ATTC_SMEM =
    2 * ATTC_Q_BYTES + ATTC_KV_STAGES * 2 * ATTC_KV_BYTES + 2 * ATTC_P_BYTES + 1024 + 256;

struct AttnTcArgs {
  const int* cu_seqlens;
  const int4* items;     // {seq, q_first, q_count, mode}; mode 1 = gathered query rows
  __nv_bfloat16* o;
  int o_stride;
  int q_col0, k_col0, v_col0;  // column of head 0 of q, k, v in their tensor maps
  int heads;                   // total heads (block b covers heads [(b % groups) * ATTC_HEADS, ...))
  int window;                  // < 0: global
  float scale_log2;
  int* status;
};

// Shared-memory descriptor of a V tile used as the MN-major B operand: rows are keys (the K
// dimension, 128 B apart, 8-row atoms of 1024 B), the 64 head dims (N) contiguous in a row.
S1C_DEV uint64_t sdesc_mnmajor_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)(8192u >> 4) << 16;   // leading byte offset: next 64-wide N block (unused, N = 64)
  d |= (uint64_t)(1024u >> 4) << 32;   // stride byte offset: next 8-key group
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// kind::f16 instruction descriptor with B MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32_bmn(int M, int N) {
  return idesc_bf16_f32(M, N) | (1u << 16);
}

S1C_DEV float ex2f_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__global__ void __launch_bounds__(ATTC_THREADS, 2)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmKV,
                        const AttnTcArgs args) {
  constexpr int NS = ATTC_KV_STAGES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_u + 1023u) & ~1023u) - raw_u);
  uint8_t* sQ = smem;                              // [2][16 KB]
  uint8_t* sK = sQ + 2 * ATTC_Q_BYTES;             // [NS][8 KB]
  uint8_t* sV = sK + NS * ATTC_KV_BYTES;           // [NS][8 KB]
  uint8_t* sP = sV + NS * ATTC_KV_BYTES;           // [2][16 KB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * ATTC_P_BYTES);
  uint64_t* q_full = bars + 0;    // [2]
  uint64_t* q_empty = bars + 2;   // [2]
  uint64_t* kv_full = bars + 4;   // [NS]
  uint64_t* kv_empty = bars + 4 + NS;
  uint64_t* s_full = bars + 4 + 2 * NS;
  uint64_t* s_free = s_full + 1;
  uint64_t* p_full = s_full + 2;  // [2]
  uint64_t* p_free = s_full + 4;  // [2]
  uint64_t* o_full = s_full + 6;  // [2]
  uint64_t* o_free = s_full + 8;  // [2]
  uint64_t* drain = s_full + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int groups = (args.heads + ATTC_HEADS - 1) / ATTC_HEADS;  // block b: item b / groups
  const int4 item = args.items[blockIdx.x / groups];
  const int seq = item.x, q_first = item.y, q_count = item.z, mode = item.w;
  const int s_begin = args.cu_seqlens[seq], s_end = args.cu_seqlens[seq + 1];
  const int h0 = (blockIdx.x % groups) * ATTC_HEADS;
  const int nh = min(ATTC_HEADS, args.heads - h0);
  const bool local = args.window >= 0 && mode == 0;
  int k_lo = s_begin, k_hi = s_end;
  if (local) {
    k_lo = max(s_begin, q_first - args.window);
    k_hi = min(s_end, q_first + q_count + args.window);
  }
  const int nt = (k_hi - k_lo + ATTC_BK - 1) / ATTC_BK;
  const int nsteps = nh * nt;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&p_free[i], 1);
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 128);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0 && nsteps > 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmKV);
      int issued_q = 0, issued_kv = 0;
      bool ok = true;
      for (int hi = 0; ok && hi < nh; ++hi) {
        const int h = h0 + hi, qb = hi & 1;
        if (!mbar_wait(&q_empty[qb], ((hi >> 1) & 1) ^ 1u, args.status, DEV_TIMEOUT_PRODUCER, abort_flag)) break;
        mbar_arrive_expect_tx(&q_full[qb], ATTC_Q_BYTES);
        tma_load_2d(sQ + qb * ATTC_Q_BYTES, &tmQ, &q_full[qb], args.q_col0 + h * 64, q_first);
        ++issued_q;
        for (int j = 0; j < nt; ++j) {
          const int step = hi * nt + j, s = step % NS;
          if (!mbar_wait(&kv_empty[s], ((step / NS) & 1) ^ 1u, args.status, DEV_TIMEOUT_PRODUCER, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[s], 2 * ATTC_KV_BYTES);
          tma_load_2d(sK + s * ATTC_KV_BYTES, &tmKV, &kv_full[s], args.k_col0 + h * 64, k_lo + j * ATTC_BK);
          tma_load_2d(sV + s * ATTC_KV_BYTES, &tmKV, &kv_full[s], args.v_col0 + h * 64, k_lo + j * ATTC_BK);
          ++issued_kv;
        }
      }
      // Loads still in flight land before the CTA exits.
      for (int i = max(0, issued_q - 2); i < issued_q; ++i)
        mbar_wait(&q_full[i & 1], (i >> 1) & 1, args.status, DEV_TIMEOUT_DRAIN, nullptr);
      for (int i = max(0, issued_kv - NS); i < issued_kv; ++i)
        mbar_wait(&kv_full[i % NS], (i / NS) & 1, args.status, DEV_TIMEOUT_DRAIN, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0 && nsteps > 0) {
      constexpr uint32_t idS = idesc_bf16_f32(128, ATTC_BK);
      constexpr uint32_t idO = idesc_bf16_f32_bmn(128, 64);
      const uint32_t tS = tmem, tO = tmem + 64;
      bool ok = true;
      // S for step `st`: needs Q of its head and K of its stage.
      auto issue_s = [&](int st) -> bool {
        const int hi = st / nt, j = st % nt, s = st % NS, qb = hi & 1;
        if (j == 0 && !mbar_wait(&q_full[qb], (hi >> 1) & 1, args.status, DEV_TIMEOUT_MMA_FULL, abort_flag))
          return false;
        if (!mbar_wait(&kv_full[s], (st / NS) & 1, args.status, DEV_TIMEOUT_MMA_FULL, abort_flag)) return false;
        if (st > 0 && !mbar_wait(s_free, (st - 1) & 1, args.status, DEV_TIMEOUT_MMA_TEMPTY, abort_flag)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ + qb * ATTC_Q_BYTES), ka = smem_u32(sK + s * ATTC_KV_BYTES);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_bf16(tS, sdesc_kmajor_sw128(qa + k * 32), sdesc_kmajor_sw128(ka + k * 32), idS, k ? 1u : 0u);
        umma_commit(s_full);
        if (j == nt - 1) umma_commit(&q_empty[qb]);  // Q of this head is no longer read
        return true;
      };
      ok = issue_s(0);
      for (int st = 0; ok && st < nsteps; ++st) {
        if (st + 1 < nsteps && !issue_s(st + 1)) break;
        const int s = st % NS, ob = st & 1;
        if (!mbar_wait(&p_full[ob], (st >> 1) & 1, args.status, DEV_TIMEOUT_MMA_FULL, abort_flag)) break;
        if (st >= 2 && !mbar_wait(&o_free[ob], ((st >> 1) - 1) & 1, args.status, DEV_TIMEOUT_MMA_TEMPTY, abort_flag))
          break;
        tc_fence_after();
        const uint32_t pa = smem_u32(sP + ob * ATTC_P_BYTES), va = smem_u32(sV + s * ATTC_KV_BYTES);
#pragma unroll
        for (int k = 0; k < ATTC_BK / 16; ++k)
          umma_bf16(tO + ob * 64, sdesc_kmajor_sw128(pa + k * 32), sdesc_mnmajor_sw128(va + k * 2048), idO,
                    k ? 1u : 0u);
        umma_commit(&o_full[ob]);
        umma_commit(&kv_empty[s]);
        umma_commit(&p_free[ob]);
      }
      umma_commit(drain);
      mbar_wait(drain, 0, args.status, DEV_TIMEOUT_DRAIN, nullptr);
    }
  } else {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row of this thread
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t tS = tmem + lane_off, tO = tmem + lane_off + 64;
    const int qtok = q_first + r;  // query token (mode 0)
    const float sc = args.scale_log2;
    float o[64];
    float m = -INFINITY, l = 0.f, corr_prev = 0.f;
    for (int st = 0; st < nsteps; ++st) {
      const int hi = st / nt, j = st % nt;
      if (j == 0) {
#pragma unroll
        for (int i = 0; i < 64; ++i) o[i] = 0.f;
        m = -INFINITY;
        l = 0.f;
      }
      if (!mbar_wait_warp(s_full, st & 1, args.status, DEV_TIMEOUT_EPILOGUE, abort_flag)) break;
      tc_fence_after();
      float s[64];
      tmem_ld32(tS, *reinterpret_cast<float(*)[32]>(s));
      tmem_ld32(tS + 32, *reinterpret_cast<float(*)[32]>(s + 32));
      tc_fence_before();
      mbar_arrive(s_free);
      // Keys this row may see, as column offsets [lo, hi) inside the tile.
      const int kt0 = k_lo + j * ATTC_BK;
      int lo = 0, hi_c = k_hi - kt0;
      if (local) {
        lo = max(lo, qtok - args.window - kt0);
        hi_c = min(hi_c, qtok + args.window + 1 - kt0);
      }
      if (!__all_sync(0xffffffffu, lo <= 0 && hi_c >= ATTC_BK)) {
#pragma unroll
        for (int c = 0; c < 64; ++c) s[c] = (c >= lo && c < hi_c) ? s[c] : -INFINITY;
      }
      float pm[8];  // 8 independent partial maxima, then a tree
#pragma unroll
      for (int i = 0; i < 8; ++i) pm[i] = s[i];
#pragma unroll
      for (int c = 8; c < 64; ++c) pm[c & 7] = fmaxf(pm[c & 7], s[c]);
      float mx = fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])), fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7])));
      mx = fmaxf(m, mx * sc);
      const float base = (mx == -INFINITY) ? 0.f : mx;
      const float corr = ex2f_approx(m - base);
      m = mx;
      // P row -> shared memory buffer st & 1 (one swizzled [128 x 64] block), once the PV MMA of
      // step st - 2 has read that buffer.
      const int pb = st & 1;
      if (st >= 2 &&
          !mbar_wait_warp(&p_free[pb], ((st >> 1) - 1) & 1, args.status, DEV_TIMEOUT_EPILOGUE, abort_flag))
        break;
      uint8_t* prow = sP + pb * ATTC_P_BYTES + r * 128;
      float rsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float p[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          p[i] = ex2f_approx(fmaf(s[8 * q + i], sc, -base));
          rsum[i] += p[i];
        }
        *reinterpret_cast<uint4*>(prow + ((q ^ (r & 7)) << 4)) =
            make_uint4(pack_bf16x2(p[0], p[1]), pack_bf16x2(p[2], p[3]), pack_bf16x2(p[4], p[5]),
                       pack_bf16x2(p[6], p[7]));
      }
      const float rs = ((rsum[0] + rsum[1]) + (rsum[2] + rsum[3])) + ((rsum[4] + rsum[5]) + (rsum[6] + rsum[7]));
      l = l * corr + rs;
      fence_proxy_async();
      mbar_arrive(&p_full[pb]);
      // Fold a finished O_j (same head) into the register accumulator, 32 columns at a time.
      auto fold = [&](int sj, float cr) -> bool {
        const int ob = sj & 1;
        if (!mbar_wait_warp(&o_full[ob], (sj >> 1) & 1, args.status, DEV_TIMEOUT_EPILOGUE, abort_flag)) return false;
        tc_fence_after();
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float t[32];
          tmem_ld32(tO + ob * 64 + half * 32, t);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[half * 32 + i] = o[half * 32 + i] * cr + t[i];
        }
        tc_fence_before();
        mbar_arrive(&o_free[ob]);
        return true;
      };
      if (j > 0 && !fold(st - 1, corr_prev)) break;
      corr_prev = corr;
      if (j == nt - 1) {
        if (!fold(st, corr)) break;
        // O / l -> bf16, row q_first + r of the output, columns of head h0 + hi
        if (r < q_count) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          uint4* dst = reinterpret_cast<uint4*>(args.o + (size_t)(q_first + r) * args.o_stride + (h0 + hi) * 64);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            dst[q] = make_uint4(pack_bf16x2(o[8 * q] * inv, o[8 * q + 1] * inv),
                                pack_bf16x2(o[8 * q + 2] * inv, o[8 * q + 3] * inv),
                                pack_bf16x2(o[8 * q + 4] * inv, o[8 * q + 5] * inv),
                                pack_bf16x2(o[8 * q + 6] * inv, o[8 * q + 7] * inv));
        }
      }
    }
  }
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace s1c
