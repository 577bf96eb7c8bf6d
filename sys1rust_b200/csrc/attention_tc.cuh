// Varlen flash attention on the 5th-generation tensor cores (tcgen05), head_dim 64.
//
// Same contract as attention.cuh (the key sets of the reference's masked SDPA calls,
// runtime/crates/laya-mlx/src/lib.rs:1644-1657, :1399-1417, :1711-1760): a query at position i of
// a row attends the keys j of the same row, all of them (global layers, head layers) or those
// with |i - j| <= window (local layers); softmax in fp32, output bf16.
//
// Persistent: a unit of work is one head of one tile of up to 128 query rows (unit u = item
// u / heads, head u % heads; items sorted longest first); the grid is two CTAs per SM (98 KB of
// shared memory and 256 TMEM columns each) and CTA b takes one unit of every round of grid units
// (b, then grid - 1 - b of the next round, ...) back to back, so the TMA/MMA pipeline never drains between units and the last wave is one unit
// deep, not four heads. 192 threads:
//   warp 0      TMA producer: Q tile [128 x 64] per unit (double buffered, so the next unit's Q
//               arrives while this one runs), K and V tiles [64 keys x 64] per key step (4-stage
//               ring), 128-byte swizzle.
//   warp 1      TMEM owner and MMA issuer:
//                 S = Q K^T     M=128 N=64 K=64 (K-major A and B from shared memory)
//                               -> TMEM cols [0,64) for even key steps, [64,128) for odd ones
//                 O += P V      M=128 N=64 K=64 (P from TMEM, V MN-major from shared memory)
//                               -> TMEM cols [128,192) for even units, [192,256) for odd units
//               The softmax writes P over the first 32 columns of its step's S buffer (bf16
//               pairs), and S of step st + 2 is issued into the same buffer right after P V of
//               step st: this thread's tcgen05 operations run in issue order, so P V has read P
//               before S overwrites it. S of a step is thus issued a whole key step ahead,
//               without waiting for the softmax to read the previous S.
//   warps 2..5  softmax, one query row per thread (TMEM lane = row). Per key step: the row's
//               maximum m; p = 2^(s * scale - m_ref) with a reference maximum m_ref that is only
//               raised when m exceeds it by more than 2^8 (p stays <= 256, exact in fp32 and
//               bf16-representable like any p), in which case the running sum and the O
//               accumulator in TMEM are rescaled by 2^(m_ref_old - m_ref) once the previous
//               P V has completed. P is rounded to bf16 pairs and written to TMEM over the S it
//               came from, where the P V MMA reads it as its A operand: no shared-memory round
//               trip and no proxy fence.
//               32-column halves of S that no row of a warp may see (window edges, a row's
//               last partial key tile) are neither read nor exponentiated; keys past a row's
//               bounds are masked only in halves where some row of the warp has a boundary.
//               A finished unit's O / l is read from TMEM and stored bf16 during the next key
//               step, after its exponentials, by which time the unit's last P V has completed.
#pragma once
#include <cuda.h>
#include "common.cuh"

namespace s1c {

constexpr int ATTC_BQ = 128, ATTC_BK = 64, ATTC_THREADS = 192, ATTC_KV_STAGES = 4;
// `attn=auto` picks this kernel when a launch has at least ATTC_HEADS units per SM.
constexpr int ATTC_HEADS = 4;
// TMEM columns: S (then P, bf16 pairs, over its first 32 columns) of even key steps [0,64), of odd
// key steps [64,128); O of even heads [128,192), of odd heads [192,256)
constexpr uint32_t ATTC_TMEM_COLS = 256;
constexpr uint32_t ATTC_TMEM_O = 128;
constexpr uint32_t ATTC_Q_BYTES = ATTC_BQ * 64 * 2;       // 16 KB
constexpr uint32_t ATTC_KV_BYTES = ATTC_BK * 64 * 2;      // 8 KB each for K and V
constexpr size_t ATTC_SMEM = 2 * ATTC_Q_BYTES + ATTC_KV_STAGES * 2 * ATTC_KV_BYTES + 1024 + 256;
constexpr float ATTC_RESCALE_LOG2 = 8.0f;  // raise the reference maximum only past 2^8

struct AttnTcArgs {
  const int* cu_seqlens;
  const int4* items;     // {seq, q_first, q_count, mode}; mode 1 = gathered query rows
  __nv_bfloat16* o;
  int o_stride;
  int q_col0, k_col0, v_col0;  // column of head 0 of q, k, v in their tensor maps
  int heads;                   // heads per item: unit u of the launch is (item u / heads, head u % heads)
  int window;                  // < 0: global
  float scale_log2;
  int* status;
  int n_items;                 // items in the work list (the grid strides over n_items * heads units)
};

// One unit of work: one head of one item (a tile of up to 128 query rows), with its key range
// [k_lo, k_hi) and its number of 64-key steps nt (0: an empty item, filled in to a bucket's fixed
// work-list length, or no keys; such units are skipped by every role alike).
struct AttcUnit {
  int q_first, q_count, mode, h, k_lo, k_hi, nt;
};
S1C_DEV AttcUnit attc_unit(const AttnTcArgs& args, int u) {
  AttcUnit w;
  const int4 item = args.items[u / args.heads];
  w.h = u % args.heads;
  w.q_first = item.y;
  w.q_count = item.z;
  w.mode = item.w;
  w.k_lo = w.k_hi = w.nt = 0;
  if (w.q_count <= 0) return w;
  const int s_begin = args.cu_seqlens[item.x], s_end = args.cu_seqlens[item.x + 1];
  w.k_lo = s_begin;
  w.k_hi = s_end;
  if (args.window >= 0 && w.mode == 0) {
    w.k_lo = max(s_begin, w.q_first - args.window);
    w.k_hi = min(s_end, w.q_first + w.q_count + args.window);
  }
  w.nt = max(0, w.k_hi - w.k_lo + ATTC_BK - 1) / ATTC_BK;
  return w;
}
// This CTA's unit of round k is k * grid + blockIdx.x in even rounds and k * grid + (grid - 1 -
// blockIdx.x) in odd ones: units come longest item first, so walking each round in the other
// direction evens out the CTAs' sums (the first CTAs would otherwise take the longest unit of every
// round). Advances k to the next round whose unit has work; false when none is left.
S1C_DEV bool attc_seek(const AttnTcArgs& args, int& k, AttcUnit& w) {
  const int n_units = args.n_items * args.heads, G = gridDim.x;
  for (; k * G < n_units; ++k) {
    const int u = k * G + ((k & 1) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x);
    if (u >= n_units) continue;
    w = attc_unit(args, u);
    if (w.nt > 0) return true;
  }
  return false;
}
// Grid of the persistent launch: two CTAs per SM, or one per unit when there are fewer units.
inline int attc_grid(int n_items, int heads, int num_sms) {
  const long units = (long)n_items * heads;
  return (int)(units < 2L * num_sms ? units : 2L * num_sms);
}

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

// Two 32-column TMEM loads with one wait: v[0..31] from taddr, v[32..63] from taddr + 32.
S1C_DEV void tmem_ld32x2(uint32_t taddr, bool lo, bool hi, float (&v)[64]) {
  uint32_t r[64];
  if (lo)
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
  else
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = 0xff800000u;  // -inf: this half is not read
  if (hi)
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
          "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
          "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
          "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr + 32));
  else
#pragma unroll
    for (int i = 32; i < 64; ++i) r[i] = 0xff800000u;
  // One hardware wait covers both loads; each asm names its half as read-write so that no use
  // is scheduled before it.
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[32]), "+r"(r[33]), "+r"(r[34]), "+r"(r[35]), "+r"(r[36]), "+r"(r[37]), "+r"(r[38]),
                 "+r"(r[39]), "+r"(r[40]), "+r"(r[41]), "+r"(r[42]), "+r"(r[43]), "+r"(r[44]), "+r"(r[45]),
                 "+r"(r[46]), "+r"(r[47]), "+r"(r[48]), "+r"(r[49]), "+r"(r[50]), "+r"(r[51]), "+r"(r[52]),
                 "+r"(r[53]), "+r"(r[54]), "+r"(r[55]), "+r"(r[56]), "+r"(r[57]), "+r"(r[58]), "+r"(r[59]),
                 "+r"(r[60]), "+r"(r[61]), "+r"(r[62]), "+r"(r[63])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 consecutive fp32 columns to TMEM (completion: tmem_st_wait).
S1C_DEV void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
      "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]),
      "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]),
      "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}
S1C_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D (TMEM) (+)= A (TMEM: row i in lane i, two bf16 of consecutive k per 32-bit column) * B (shared
// memory descriptor).
S1C_DEV void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
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
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + NS * ATTC_KV_BYTES);
  uint64_t* q_full = bars + 0;    // [2]
  uint64_t* q_empty = bars + 2;   // [2]
  uint64_t* o_full = bars + 4;    // [2]
  uint64_t* o_free = bars + 6;    // [2]
  uint64_t* kv_full = bars + 8;   // [NS]
  uint64_t* kv_empty = bars + 8 + NS;
  uint64_t* s_full = bars + 8 + 2 * NS;  // [2]: S of even / odd key steps computed
  uint64_t* p_full = s_full + 2;          // [2]: P of even / odd key steps written
  uint64_t* p_free = s_full + 4;          // [2]: P V of even / odd key steps completed
  uint64_t* drain = s_full + 6;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);  // one arrival per softmax warp
    }
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&p_free[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, ATTC_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tmap(&tmQ);
      prefetch_tmap(&tmKV);
      int issued_q = 0, issued_kv = 0;  // units (= Q loads) and key steps (= K/V stages) issued
      bool ok = true;
      AttcUnit w;
      for (int k = 0; ok && attc_seek(args, k, w); ++k) {
        const int qb = issued_q & 1;
        // Q buffer qb is free once the last S MMA of the unit two before has completed
        if (!mbar_wait(&q_empty[qb], ((issued_q >> 1) & 1) ^ 1u, args.status, DEV_TIMEOUT_PRODUCER, abort_flag)) break;
        mbar_arrive_expect_tx(&q_full[qb], ATTC_Q_BYTES);
        tma_load_2d(sQ + qb * ATTC_Q_BYTES, &tmQ, &q_full[qb], args.q_col0 + w.h * 64, w.q_first);
        ++issued_q;
        for (int j = 0; j < w.nt; ++j) {
          const int step = issued_kv, s = step % NS;
          if (!mbar_wait(&kv_empty[s], ((step / NS) & 1) ^ 1u, args.status, DEV_TIMEOUT_PRODUCER, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[s], 2 * ATTC_KV_BYTES);
          tma_load_2d(sK + s * ATTC_KV_BYTES, &tmKV, &kv_full[s], args.k_col0 + w.h * 64, w.k_lo + j * ATTC_BK);
          tma_load_2d(sV + s * ATTC_KV_BYTES, &tmKV, &kv_full[s], args.v_col0 + w.h * 64, w.k_lo + j * ATTC_BK);
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
    if (lane == 0) {
      constexpr uint32_t idS = idesc_bf16_f32(128, ATTC_BK);
      constexpr uint32_t idO = idesc_bf16_f32_bmn(128, 64);
      // S cursor: the next key step whose S is issued (unit su, its count sui among this CTA's
      // units, key step sj of it, global step sst). S of step st goes into TMEM buffer st & 1 and
      // is issued right after P V of step st - 2, which read the P held in that buffer.
      int su = 0, sui = 0, sj = 0, sst = 0;  // su: round
      AttcUnit sw;
      bool s_more = attc_seek(args, su, sw);
      auto issue_next_s = [&]() -> bool {
        if (!s_more) return true;
        const int qb = sui & 1, s = sst % NS, sb = sst & 1;
        if (sj == 0 && !mbar_wait(&q_full[qb], (sui >> 1) & 1, args.status, DEV_TIMEOUT_MMA_FULL, abort_flag))
          return false;
        if (!mbar_wait(&kv_full[s], (sst / NS) & 1, args.status, DEV_TIMEOUT_MMA_FULL, abort_flag)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(sQ + qb * ATTC_Q_BYTES), ka = smem_u32(sK + s * ATTC_KV_BYTES);
        const uint32_t tS = tmem + 64 * sb;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_bf16(tS, sdesc_kmajor_sw128(qa + k * 32), sdesc_kmajor_sw128(ka + k * 32), idS, k ? 1u : 0u);
        umma_commit(&s_full[sb]);
        if (sj == sw.nt - 1) umma_commit(&q_empty[qb]);  // Q of this unit is no longer read
        ++sst;
        if (++sj == sw.nt) {
          sj = 0;
          ++sui;
          ++su;
          s_more = attc_seek(args, su, sw);
        }
        return true;
      };
      bool ok = issue_next_s() && issue_next_s();
      int st = 0, pui = 0, pu = 0;  // pu: round
      AttcUnit pw;
      for (bool more = ok && attc_seek(args, pu, pw); ok && more; more = attc_seek(args, pu, pw)) {
        const int ob = pui & 1;
        for (int j = 0; j < pw.nt; ++j, ++st) {
          const int s = st % NS, sb = st & 1;
          if (!mbar_wait(&p_full[sb], (st >> 1) & 1, args.status, DEV_TIMEOUT_MMA_FULL, abort_flag)) {
            ok = false;
            break;
          }
          // the first P V of a unit overwrites its O buffer: the O of the unit two before must have been read
          if (j == 0 && pui >= 2 &&
              !mbar_wait(&o_free[ob], ((pui >> 1) - 1) & 1, args.status, DEV_TIMEOUT_MMA_TEMPTY, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t va = smem_u32(sV + s * ATTC_KV_BYTES), tO = tmem + ATTC_TMEM_O + 64 * ob;
          const uint32_t tP = tmem + 64 * sb;
#pragma unroll
          for (int k = 0; k < ATTC_BK / 16; ++k)
            umma_bf16_ts(tO, tP + 8 * k, sdesc_mnmajor_sw128(va + k * 2048), idO, (j > 0 || k > 0) ? 1u : 0u);
          umma_commit(&kv_empty[s]);
          umma_commit(&p_free[sb]);
          if (j == pw.nt - 1) umma_commit(&o_full[ob]);
          if (!issue_next_s()) {
            ok = false;
            break;
          }
        }
        ++pui;
        ++pu;
      }
      umma_commit(drain);
      mbar_wait(drain, 0, args.status, DEV_TIMEOUT_DRAIN, nullptr);
    }
  } else {
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row of this thread
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float sc = args.scale_log2;
    float m_ref = -INFINITY, l = 0.f;
    // O / l of a finished unit -> bf16, row pq_first + r, columns of head ph. Deferred to the next
    // step's exponentials so that the last P V of the unit has completed by then. `hd` is the
    // unit's count among this CTA's units (its O buffer and barrier phase).
    int pend = -1, pq_first = 0, pq_count = 0, ph = 0;
    float l_pend = 0.f;
    auto epilogue = [&](int hd, float lsum) -> bool {
      const int ob = hd & 1;
      if (!mbar_wait_warp(&o_full[ob], (hd >> 1) & 1, args.status, DEV_TIMEOUT_EPILOGUE, abort_flag)) return false;
      tc_fence_after();
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
      uint4* dst = reinterpret_cast<uint4*>(args.o + (size_t)(pq_first + r) * args.o_stride + ph * 64);
      const uint32_t tO = tmem + lane_off + ATTC_TMEM_O + 64 * ob;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float t[32];
        tmem_ld32(tO + half * 32, t);
        if (r < pq_count) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            dst[half * 4 + q] = make_uint4(pack_bf16x2(t[8 * q] * inv, t[8 * q + 1] * inv),
                                           pack_bf16x2(t[8 * q + 2] * inv, t[8 * q + 3] * inv),
                                           pack_bf16x2(t[8 * q + 4] * inv, t[8 * q + 5] * inv),
                                           pack_bf16x2(t[8 * q + 6] * inv, t[8 * q + 7] * inv));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[ob]);
      return true;
    };
    bool ok = true;
    int st = 0, ui = 0, u = 0;  // u: round
    AttcUnit w;
    for (; ok && attc_seek(args, u, w); ++u, ++ui) {
      m_ref = -INFINITY;
      l = 0.f;
      const bool local = args.window >= 0 && w.mode == 0;
      const int qtok = w.q_first + r;  // query token (mode 0)
      const int k_lo = w.k_lo, k_hi = w.k_hi, hi = ui;
      for (int j = 0; j < w.nt; ++j, ++st) {
        // Keys this row may see, as column offsets [lo, hi_c) inside the tile; which 32-column
        // halves any row of this warp may see.
        const int kt0 = k_lo + j * ATTC_BK;
        int lo = 0, hi_c = k_hi - kt0;
        if (local) {
          lo = max(lo, qtok - args.window - kt0);
          hi_c = min(hi_c, qtok + args.window + 1 - kt0);
        }
        const bool need0 = __any_sync(0xffffffffu, lo < 32 && hi_c > 0);
        const bool need1 = __any_sync(0xffffffffu, lo < 64 && hi_c > 32);
        const int sb = st & 1;
        const uint32_t tS = tmem + lane_off + 64 * sb;
        if (!mbar_wait_warp(&s_full[sb], (st >> 1) & 1, args.status, DEV_TIMEOUT_EPILOGUE, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float s[64];
        tmem_ld32x2(tS, need0, need1, s);
        // Keys outside [lo, hi_c) are masked only in the halves where some row of the warp has a
        // boundary (halves no row sees were not read and hold -inf): one bit test per column. Tiles
        // every row of the warp sees whole (most key steps of global layers) skip all of it.
        if (!__all_sync(0xffffffffu, lo <= 0 && hi_c >= ATTC_BK)) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const int c0 = half * 32;
            if ((half ? need1 : need0) && !__all_sync(0xffffffffu, lo <= c0 && hi_c >= c0 + 32)) {
              const int a = min(max(lo - c0, 0), 32), b = min(max(hi_c - c0, 0), 32);
              const uint32_t vis = (b >= 32 ? 0xffffffffu : (1u << b) - 1u) & ~(a >= 32 ? 0xffffffffu : (1u << a) - 1u);
#pragma unroll
              for (int c = 0; c < 32; ++c) s[c0 + c] = (vis & (1u << c)) ? s[c0 + c] : -INFINITY;
            }
          }
        }
        float pm[8];  // 8 independent partial maxima over the halves read, then a tree
#pragma unroll
        for (int i = 0; i < 8; ++i) pm[i] = -INFINITY;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          if (half ? need1 : need0) {
#pragma unroll
            for (int c = half * 32; c < half * 32 + 32; ++c) pm[c & 7] = fmaxf(pm[c & 7], s[c]);
          }
        }
        const float mx =
            fmaxf(fmaxf(fmaxf(pm[0], pm[1]), fmaxf(pm[2], pm[3])), fmaxf(fmaxf(pm[4], pm[5]), fmaxf(pm[6], pm[7]))) * sc;
        // Raise the reference maximum only when this tile's maximum passes it by more than 2^8.
        float factor = 1.f;
        bool rescale_o = false;
        if (mx > m_ref + ATTC_RESCALE_LOG2) {
          factor = ex2f_approx(m_ref - mx);  // 0 while m_ref is -inf
          rescale_o = l > 0.f;               // O holds earlier P V products of this unit
          l *= factor;
          m_ref = mx;
        }
        const float base = (m_ref == -INFINITY) ? 0.f : m_ref;
        float rsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          if (half ? need1 : need0) {
#pragma unroll
            for (int c = half * 32; c < half * 32 + 32; ++c) {
              s[c] = ex2f_approx(fmaf(s[c], sc, -base));
              rsum[c & 7] += s[c];
            }
          } else {
#pragma unroll
            for (int c = half * 32; c < half * 32 + 32; ++c) s[c] = 0.f;
          }
        }
        l += ((rsum[0] + rsum[1]) + (rsum[2] + rsum[3])) + ((rsum[4] + rsum[5]) + (rsum[6] + rsum[7]));
        if (pend >= 0) {
          if (!epilogue(pend, l_pend)) {
            ok = false;
            break;
          }
          pend = -1;
        }
        {
          // P over the S it came from (S of this step is in registers; P V of step st - 2, which
          // read the P held here before, ran ahead of the S MMA that wrote this step's S)
          float pk[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = __uint_as_float(pack_bf16x2(s[2 * i], s[2 * i + 1]));
          tmem_st32(tS, pk);
        }
        if (__any_sync(0xffffffffu, rescale_o)) {
          // O is rescaled after the previous step's P V has completed
          if (st > 0 &&
              !mbar_wait_warp(&p_free[sb ^ 1], ((st - 1) >> 1) & 1, args.status, DEV_TIMEOUT_EPILOGUE, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t tO = tmem + lane_off + ATTC_TMEM_O + 64 * (hi & 1);
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            float t[32];
            tmem_ld32(tO + half * 32, t);
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] *= factor;
            tmem_st32(tO + half * 32, t);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[sb]);
        if (j == w.nt - 1) {
          pend = hi;
          l_pend = l;
          pq_first = w.q_first;
          pq_count = w.q_count;
          ph = w.h;
        }
      }
    }
    if (ok && pend >= 0) epilogue(pend, l_pend);
  }
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ATTC_TMEM_COLS);
  }
}

}  // namespace s1c
