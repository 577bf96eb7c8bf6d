// Varlen flash attention, head_dim 64, bf16 in / bf16 out, fp32 softmax statistics.
//
// Replaces the reference's masked SDPA calls (runtime/crates/laya-mlx/src/lib.rs:1644-1657
// encoder global/local, :1432-1475 chunked local, :1711-1760 head layers). The reference pads
// rows and adds MASK_NEG (-1e4) to padded keys and to keys outside the window; here sequences
// are unpadded (cu_seqlens) and the same key set is selected exactly: a query at position i
// of a row sees the keys j of the same row with |i - j| <= window (local layers,
// lib.rs:1399-1417), or every key of the row (global layers, head layers). Keys the reference
// masks with -1e4 get exp(-1e4 - max) = 0 in fp32, so both select the same softmax.
//
// One CTA = 4 warps = 64 query rows of one head; K/V tiles of 64 keys stream through shared
// memory with cp.async (double buffered, XOR-swizzled 128-byte rows, ldmatrix fragments),
// QK^T and PV on mma.sync m16n8k16 bf16 with fp32 accumulation, online softmax in fp32.
//
// Work items {seq, q_first, q_count, mode}:
//   mode 0: query rows are the packed tokens q_first .. q_first + q_count - 1 of sequence
//           `seq`; Q and O are indexed by token.
//   mode 1: query rows are rows q_first .. of a separate (gathered) Q/O buffer, all of
//           sequence `seq`; used by the pruned last head layer (lib.rs:1728-1748), global only.
#pragma once
#include "common.cuh"

namespace s1c {

struct AttnArgs {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  __nv_bfloat16* o;
  int q_stride, k_stride, v_stride, o_stride;  // row pitches in elements
  const int* cu_seqlens;                        // [n + 1]
  const int4* items;                            // work items
  int window;                                   // < 0: global
  float scale_log2;                             // softmax scale * log2(e)
  int heads;                                    // block b works on item b / heads, head b % heads
};

constexpr int ATT_BQ = 64, ATT_BK = 64, ATT_D = 64, ATT_THREADS = 128;

S1C_DEV void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
S1C_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
S1C_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
S1C_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
S1C_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
S1C_DEV void mma_bf16_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                            uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2^x on the special-function unit (inputs of -inf give +0).
S1C_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Byte offset of 16-byte chunk `c` of row `r` in a [64][64] bf16 tile with XOR swizzle.
S1C_DEV uint32_t swz(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

// Load rows [row0, row0 + 64) of a [*, stride] bf16 matrix (columns col0 .. col0 + 63) into a
// swizzled tile; rows at or past `row_end` are zero-filled.
S1C_DEV void load_tile_async(uint32_t tile, const __nv_bfloat16* base, int stride, int col0, int row0, int row_end,
                             int tid) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = tid + i * ATT_THREADS;  // 512 chunks of 16 B
    const int r = idx >> 3, c = idx & 7;
    const int row = row0 + r;
    const bool ok = row < row_end;
    const __nv_bfloat16* src = base + (size_t)(ok ? row : 0) * stride + col0 + c * 8;
    cp_async16(tile + swz(r, c), src, ok ? 16u : 0u);
  }
}

__global__ void __launch_bounds__(ATT_THREADS, 4) attention_varlen_kernel(const AttnArgs args) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(128) __nv_bfloat16 sQ[ATT_BQ * ATT_D];
  __shared__ __align__(128) __nv_bfloat16 sK[2][ATT_BK * ATT_D];
  __shared__ __align__(128) __nv_bfloat16 sV[2][ATT_BK * ATT_D];

  const int4 item = args.items[blockIdx.x / args.heads];
  const int head = blockIdx.x % args.heads;
  const int seq = item.x, q_first = item.y, q_count = item.z, mode = item.w;
  if (q_count <= 0) return;  // an empty item (work lists filled up to a bucket's fixed length)
  const int s_begin = args.cu_seqlens[seq], s_end = args.cu_seqlens[seq + 1];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hcol = head * ATT_D;

  // Key range of this tile of queries.
  int k_lo = s_begin, k_hi = s_end;
  if (args.window >= 0 && mode == 0) {
    const int p0 = q_first - s_begin, p1 = p0 + q_count - 1;
    k_lo = max(s_begin, s_begin + p0 - args.window);
    k_hi = min(s_end, s_begin + p1 + args.window + 1);
  }
  const int n_tiles = max(0, k_hi - k_lo + ATT_BK - 1) / ATT_BK;

  const uint32_t q_s = smem_u32(sQ);
  const uint32_t k_s0 = smem_u32(sK[0]), v_s0 = smem_u32(sV[0]);
  constexpr uint32_t TILE_BYTES = ATT_BK * ATT_D * 2;

  load_tile_async(q_s, args.q, args.q_stride, hcol, q_first, q_first + q_count, tid);
  if (n_tiles > 0) {
    load_tile_async(k_s0, args.k, args.k_stride, hcol, k_lo, k_hi, tid);
    load_tile_async(v_s0, args.v, args.v_stride, hcol, k_lo, k_hi, tid);
  }
  cp_async_commit();

  const int g = lane >> 2, t4 = lane & 3;
  const bool local = args.window >= 0 && mode == 0;
  // Query positions of this thread's two rows (mode 0 only; used by the window test).
  const int qrow0 = warp * 16 + g;
  const int qpos0 = q_first - s_begin + qrow0, qpos1 = qpos0 + 8;

  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qa[4][4];

  for (int it = 0; it < n_tiles; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_tiles) {
      const int nb = buf ^ 1;
      load_tile_async(k_s0 + nb * TILE_BYTES, args.k, args.k_stride, hcol, k_lo + (it + 1) * ATT_BK, k_hi, tid);
      load_tile_async(v_s0 + nb * TILE_BYTES, args.v, args.v_stride, hcol, k_lo + (it + 1) * ATT_BK, k_hi, tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    if (it == 0) {
      // Q fragments for this warp's 16 rows, 4 k-steps of 16 dims.
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int r = warp * 16 + (lane & 15);
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(q_s + swz(r, c), qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3]);
      }
    }

    // Keys this thread's two rows may see, as column offsets [lo, hi) inside the tile: the
    // sequence's [k_lo, k_hi), narrowed to |i - j| <= window on local layers. Masking runs only
    // when some row of the warp does not see the whole tile (edge tiles).
    const int kt0 = k_lo + it * ATT_BK;
    int lo0 = 0, hi0 = k_hi - kt0, lo1 = 0, hi1 = k_hi - kt0;
    if (local) {
      lo0 = max(lo0, s_begin + qpos0 - args.window - kt0);
      hi0 = min(hi0, s_begin + qpos0 + args.window + 1 - kt0);
      lo1 = max(lo1, s_begin + qpos1 - args.window - kt0);
      hi1 = min(hi1, s_begin + qpos1 + args.window + 1 - kt0);
    }
    // 16-key blocks of this tile that some row of the warp sees: [blo, bhi). Blocks outside are
    // skipped entirely (their scores, exponentials and PV products would all be zero).
    int blo = min(lo0, lo1), bhi = max(hi0, hi1);
    blo = __reduce_min_sync(0xffffffffu, blo);
    bhi = __reduce_max_sync(0xffffffffu, bhi);
    blo = max(blo, 0) >> 4;
    bhi = min((max(bhi, 0) + 15) >> 4, ATT_BK / 16);

    // S = Q K^T for 64 keys: 8 groups of 8 keys; per k-step the four K fragments are loaded
    // before the eight MMAs that use them.
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      uint32_t kb[4][4];
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        // keys 16*jp .. 16*jp+15 (two groups), dims 16*ks .. 16*ks+15
        const int r = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 2 + ((lane >> 3) & 1);
        if (jp >= blo && jp < bhi) ldsm_x4(k_s0 + buf * TILE_BYTES + swz(r, c), kb[jp][0], kb[jp][1], kb[jp][2], kb[jp][3]);
      }
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        if (jp >= blo && jp < bhi) {
          mma_bf16_16816(s[2 * jp], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kb[jp][0], kb[jp][1]);
          mma_bf16_16816(s[2 * jp + 1], qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], kb[jp][2], kb[jp][3]);
        }
      }
    }
    const bool whole = lo0 <= 0 && hi0 >= ATT_BK && lo1 <= 0 && hi1 >= ATT_BK;
    if (!__all_sync(0xffffffffu, whole)) {
      const int b = 2 * t4;  // column of element (j, e) = j * 8 + b + (e & 1)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = j * 8 + (e & 1) + b;
          const bool ok = (e < 2) ? (c >= lo0 && c < hi0) : (c >= lo1 && c < hi1);
          s[j][e] = ok ? s[j][e] : -INFINITY;
        }
      }
    }

    // Online softmax (base 2) on raw scores: max first, then p = 2^(s * scale - max * scale).
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    mx0 = fmaxf(m0, mx0 * args.scale_log2);
    mx1 = fmaxf(m1, mx1 * args.scale_log2);
    const float base0 = (mx0 == -INFINITY) ? 0.f : mx0;
    const float base1 = (mx1 == -INFINITY) ? 0.f : mx1;
    const float corr0 = ex2_approx(m0 - base0), corr1 = ex2_approx(m1 - base1);
    m0 = mx0;
    m1 = mx1;
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pa[8][2];
    const float sc = args.scale_log2;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = ex2_approx(fmaf(s[j][0], sc, -base0)), p1 = ex2_approx(fmaf(s[j][1], sc, -base0));
      const float p2 = ex2_approx(fmaf(s[j][2], sc, -base1)), p3 = ex2_approx(fmaf(s[j][3], sc, -base1));
      rs0 += p0 + p1;
      rs1 += p2 + p3;
      pa[j][0] = pack_bf16x2(p0, p1);
      pa[j][1] = pack_bf16x2(p2, p3);
    }
    l0 = l0 * corr0 + rs0;
    l1 = l1 * corr1 + rs1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= corr0; o[j][1] *= corr0;
      o[j][2] *= corr1; o[j][3] *= corr1;
    }

    // O += P V: 4 k-steps of 16 keys (the blocks some row sees), 8 groups of 8 dims; the four
    // V fragments of a k-step are loaded before its eight MMAs.
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      if (ks < blo || ks >= bhi) continue;
      const uint32_t a0 = pa[2 * ks][0], a1 = pa[2 * ks][1], a2 = pa[2 * ks + 1][0], a3 = pa[2 * ks + 1][1];
      uint32_t vb[4][4];
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        // keys 16*ks .. +15, dims 16*jp .. +15 (two groups), transposed load
        const int r = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = jp * 2 + (lane >> 4);
        ldsm_x4_t(v_s0 + buf * TILE_BYTES + swz(r, c), vb[jp][0], vb[jp][1], vb[jp][2], vb[jp][3]);
      }
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {
        mma_bf16_16816(o[2 * jp], a0, a1, a2, a3, vb[jp][0], vb[jp][1]);
        mma_bf16_16816(o[2 * jp + 1], a0, a1, a2, a3, vb[jp][2], vb[jp][3]);
      }
    }
    __syncthreads();
  }

  // Row sums across the quad, normalise, store.
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int r0 = q_first + warp * 16 + g, r1 = r0 + 8;
  const int lim = q_first + q_count;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int col = hcol + j * 8 + 2 * t4;
    if (r0 < lim)
      *reinterpret_cast<uint32_t*>(args.o + (size_t)r0 * args.o_stride + col) =
          pack_bf16x2(o[j][0] * inv0, o[j][1] * inv0);
    if (r1 < lim)
      *reinterpret_cast<uint32_t*>(args.o + (size_t)r1 * args.o_stride + col) =
          pack_bf16x2(o[j][2] * inv1, o[j][3] * inv1);
  }
}

}  // namespace s1c
