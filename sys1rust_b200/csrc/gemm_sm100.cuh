// Persistent bf16 GEMM for sm_100a on the 5th-generation tensor cores:
//   out = epilogue( A[M, K] * B[N, K]^T )   (A and B K-major, as the weights are stored [out, in])
//
// Encoder GEMMs of the reference forward (runtime/crates/laya-mlx/src/lib.rs:1363-1390 `mm` and
// `lin_add`, :1600-1675 the layer loop) and the head's biased linears (:1726-1760) all run here.
//
// Structure (one CTA per SM, 64 + 32 x GEMM_EPI_WARPS threads):
//   warp 0      TMA producer: 128x64 A tile + BNx64 B tile per stage, 128-byte swizzle,
//               4-stage ring of shared-memory buffers guarded by full/empty mbarriers.
//   warp 1      allocates 2*BN TMEM columns and issues tcgen05.mma (M=128, N=BN, K=16 per
//               instruction, fp32 accumulation in TMEM); tcgen05.commit releases a stage when
//               the MMAs reading it are done and hands a finished accumulator to the epilogue.
//   warps 2..   epilogue, one (default) or two warps per TMEM lane quadrant (a warp may only read
//               the 32 TMEM lanes of quadrant warp % 4), each taking its share of the columns:
//               tcgen05.ld of the accumulator (one row per thread), the fused math, then each
//               warp writes its 32-row slice of a 128-byte-wide column block into a swizzled
//               shared-memory staging buffer and one lane hands it to TMA: a tensor store for
//               bf16 / fp32 outputs, a tensor reduce-add for the residual streams. Global
//               traffic is therefore fully coalesced whatever the row layout. Two accumulators
//               alternate, so the epilogue of tile i overlaps the MMAs of tile i+1 (see
//               GEMM_EPI_WARPS for what the overlap costs).
// Tiles are walked n-fastest (tile = m_block * n_blocks + n_block) so CTAs running together
// share their A rows and stream the whole weight from L2.
//
// Epilogues:
//   EPI_STORE  bias (optional), then identity / ReLU / erf-GELU, stored bf16 (or fp32).
//   EPI_ROPE   the encoder's qkv: rotate-half RoPE of the q and k heads at each row's position
//              (split_rope.metal:46-76), v copied; stored bf16 [M, 3d] (q | k | v, head-major).
//   EPI_GEGLU  the encoder's Wi with its rows interleaved per 128 (input 128 | gate 128 per
//              256-wide tile): out = gelu_erf(input) * gate (lib.rs:367-368, :494-510), bf16 [M, I].
//   EPI_RESID  fp32 residual stream update: out += acc (+ bias) (lib.rs:1375-1390), one fp32 add per
//              element performed by the TMA reduction (the head's residual streams).
//   EPI_RESID16 the encoder's residual stream, stored f16 as the reference stores it (its f16
//              model's `lin_add`, lib.rs:1373-1390): out += f16(acc (+ bias)), the f16 add performed
//              by the TMA reduction; half the bytes of the fp32 stream in the Wo / Wo2 epilogues and
//              the LayerNorms that read it.
#pragma once
#include <cuda.h>
#include "common.cuh"

namespace s1c {

enum Epi : int { EPI_STORE = 0, EPI_ROPE = 1, EPI_GEGLU = 2, EPI_RESID = 3, EPI_RESID16 = 4 };
enum Act : int { ACT_NONE = 0, ACT_RELU = 1, ACT_GELU = 2 };

struct GemmArgs {
  int M, N, K;
  const float* bias;      // [N] or null (EPI_STORE, EPI_RESID, EPI_RESID16)
  int act;                // EPI_STORE activation
  int out_f32;            // EPI_STORE: fp32 output (the output map is fp32, 32-column boxes)
  const int* pos;         // EPI_ROPE: position of each row inside its sequence
  const float* inv_freq;  // EPI_ROPE: [32] inverse frequencies of the layer's theta
  const float* rope_tab;  // EPI_ROPE, optional: [positions][64] cos | sin of p * inv_freq[j]
                          // (rope_table_kernel); when set the epilogue reads a row's 32 cos / sin
                          // pairs instead of evaluating them: 16 loads instead of 32 sincosf
  int rope_cols;          // EPI_ROPE: columns [0, rope_cols) hold q and k heads
  int out_cols;           // EPI_GEGLU: output width I
  int k_splits;           // > 1: split-K; split s stores its fp32 partial sums into rows
                          // [s * split_rows, ...) of the workspace the output map then describes;
                          // splitk_finalize sums the slices in order and applies the epilogue
  int split_rows;         // rows of one workspace slice (M rounded up to the tile height)
  int* status;
  const void* pf;         // cluster split-K only: the next GEMM's weights, prefetched into L2
  size_t pf_bytes;
};

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int GEMM_STAGES = 4;  // 128 x 256 tiles: 4 x 48 KB stages
// 128 x 128 tiles: 6 x 32 KB stages fit beside the staging buffers.
__host__ __device__ constexpr int gemm_stages(int BN) { return BN >= 256 ? GEMM_STAGES : 6; }
constexpr int GEMM_THREADS = 192;    // the two-CTA and cluster split-K kernels: 2 + 4 warps
// Epilogue warps of the persistent one-CTA kernel. The accumulator drains while the next tile's
// MMAs run, but the epilogue's work still slows the mainloop: without it the mainloop reaches
// ~1.6 PFLOP/s on the K = 1024 shapes, with it ~1.15-1.23. Measured: the epilogue warps that share
// an SM sub-partition with the MMA-issuing warp cost the most (a cheap epilogue on that quadrant
// alone gave +13 %), eight warps were slower than four on GeGLU (1177 vs 1235 TFLOP/s) and equal
// elsewhere, so four is the default; eight is kept as a build option.
#ifndef S1C_GEMM_EPI_WARPS
#define S1C_GEMM_EPI_WARPS 4
#endif
constexpr int GEMM_EPI_WARPS = S1C_GEMM_EPI_WARPS;  // the persistent one-CTA kernel: 2 + 4 or 2 + 8 warps
static_assert(GEMM_EPI_WARPS == 4 || GEMM_EPI_WARPS == 8, "one or two epilogue warps per TMEM lane quadrant");
constexpr int GEMM1_THREADS = 64 + 32 * GEMM_EPI_WARPS;
constexpr uint32_t GEMM_STG_BYTES = 4096;  // one staging buffer: 32 rows x 128 bytes

__host__ __device__ constexpr size_t gemm_smem_bytes(int BN) {
  return (size_t)gemm_stages(BN) * (GEMM_BM * GEMM_BK * 2 + BN * GEMM_BK * 2) + 8 * GEMM_STG_BYTES + 1024 /*align*/ +
         256 /*barriers*/;
}

// GELU(x) = x * Phi(x) = 0.5 x erfc(-x / sqrt(2)) (the reference's erf form, lib.rs:494-510).
// erfc(z), z >= 0, by the Chebyshev fit of Numerical Recipes (Press, Teukolsky, Vetterling and
// Flannery, 2nd ed., section 6.2, "erfcc"): erfc(z) = t exp(-z^2 + P(t)), t = 1 / (1 + z / 2), with
// fractional error below 1.2e-7 for every z; then Phi(x) = 1 - erfc(|x|/sqrt 2) / 2 for x >= 0 and
// erfc(|x|/sqrt 2) / 2 below. One reciprocal, one exp2 and eleven FMAs, no branch; the GELU's
// absolute error is below 2e-8 (checked against erf in double precision over [-12, 12]).
// The same GELU for two values at once: the scaling, the polynomial and the exp2 argument on packed
// fp32 pairs (f32x2 FMA / MUL, bit-identical per lane to the scalar form), the reciprocal, the exp2
// and the sign select per element. Measured +4 % on the Wi + GeGLU GEMM over the scalar form.
S1C_DEV void gelu_erf_x2(float& x0, float& x1) {
  float z0, z1, d0, d1;
  f2_unpack(f2_mul(f2_pack(fabsf(x0), fabsf(x1)), f2_splat(0.70710678118654752f)), z0, z1);
  const uint64_t z = f2_pack(z0, z1);
  f2_unpack(f2_fma(f2_splat(0.5f), z, f2_splat(1.0f)), d0, d1);
  float t0, t1;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t0) : "f"(d0));
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t1) : "f"(d1));
  const uint64_t t = f2_pack(t0, t1);
  uint64_t p = f2_splat(0.17087277f);
  p = f2_fma(p, t, f2_splat(-0.82215223f));
  p = f2_fma(p, t, f2_splat(1.48851587f));
  p = f2_fma(p, t, f2_splat(-1.13520398f));
  p = f2_fma(p, t, f2_splat(0.27886807f));
  p = f2_fma(p, t, f2_splat(-0.18628806f));
  p = f2_fma(p, t, f2_splat(0.09678418f));
  p = f2_fma(p, t, f2_splat(0.37409196f));
  p = f2_fma(p, t, f2_splat(1.00002368f));
  p = f2_fma(p, t, f2_splat(-1.26551223f));
  float a0, a1;
  f2_unpack(f2_mul(f2_fma(f2_pack(-z0, -z1), z, p), f2_splat(1.4426950408889634f)), a0, a1);
  float e0, e1;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(a0));
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(a1));
  float h0, h1;
  f2_unpack(f2_mul(f2_mul(f2_splat(0.5f), t), f2_pack(e0, e1)), h0, h1);
  x0 = x0 * (x0 >= 0.f ? 1.0f - h0 : h0);
  x1 = x1 * (x1 >= 0.f ? 1.0f - h1 : h1);
}

S1C_DEV float gelu_erf(float x) {
  const float z = fabsf(x) * 0.70710678118654752f;
  float t;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(t) : "f"(fmaf(0.5f, z, 1.0f)));
  float p = 0.17087277f;
  p = fmaf(p, t, -0.82215223f);
  p = fmaf(p, t, 1.48851587f);
  p = fmaf(p, t, -1.13520398f);
  p = fmaf(p, t, 0.27886807f);
  p = fmaf(p, t, -0.18628806f);
  p = fmaf(p, t, 0.09678418f);
  p = fmaf(p, t, 0.37409196f);
  p = fmaf(p, t, 1.00002368f);
  p = fmaf(p, t, -1.26551223f);
  float e;  // exp(-z^2 + p) = 2^((p - z^2) log2 e)
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(fmaf(-z, z, p) * 1.4426950408889634f));
  const float h = 0.5f * t * e;
  return x * (x >= 0.f ? 1.0f - h : h);
}

// TMA tensor store / reduce-add of a staged box, and the bulk-group bookkeeping.
S1C_DEV void tma_store_2d(const void* tmap, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
S1C_DEV void tma_reduce_add_2d(const void* tmap, const void* src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
S1C_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
S1C_DEV void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
S1C_DEV void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
S1C_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Per-warp staging of 32 rows x 128 bytes with the 128-byte swizzle the output tensor map uses:
// row r, 16-byte chunk c lives at r*128 + ((c ^ (r & 7)) * 16). Double buffered per warp.
struct Stager {
  uint8_t* base;   // this warp's buffers
  uint32_t count;  // units issued so far
  int lane;
  int nbuf;        // 1 or 2 buffers

  // Wait until the buffer about to be written is no longer read by an older store.
  S1C_DEV uint8_t* acquire() {
    if (nbuf == 1) {
      if (count >= 1) {
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
      }
      return base;
    }
    if (count >= 2) {
      if (lane == 0) bulk_wait_read1();
      __syncwarp();
    }
    return base + (count & 1) * GEMM_STG_BYTES;
  }
  S1C_DEV void put_f32x32(uint8_t* buf, const float (&v)[32]) {
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<float4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) =
          make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  }
  S1C_DEV void put_bf16x64(uint8_t* buf, const float* v) {
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) =
          make_uint4(pack_bf16x2(v[8 * c], v[8 * c + 1]), pack_bf16x2(v[8 * c + 2], v[8 * c + 3]),
                     pack_bf16x2(v[8 * c + 4], v[8 * c + 5]), pack_bf16x2(v[8 * c + 6], v[8 * c + 7]));
  }
  S1C_DEV void put_f16x64(uint8_t* buf, const float* v) {
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(buf + lane * 128 + ((c ^ (lane & 7)) << 4)) =
          make_uint4(pack_f16x2(v[8 * c], v[8 * c + 1]), pack_f16x2(v[8 * c + 2], v[8 * c + 3]),
                     pack_f16x2(v[8 * c + 4], v[8 * c + 5]), pack_f16x2(v[8 * c + 6], v[8 * c + 7]));
  }
  // 16 values as bf16 into the 16-byte chunks c and c + 1 of this lane's row.
  S1C_DEV void put_bf16x16(uint8_t* buf, int c, const float* v) {
#pragma unroll
    for (int k = 0; k < 2; ++k)
      *reinterpret_cast<uint4*>(buf + lane * 128 + (((c + k) ^ (lane & 7)) << 4)) =
          make_uint4(pack_bf16x2(v[8 * k], v[8 * k + 1]), pack_bf16x2(v[8 * k + 2], v[8 * k + 3]),
                     pack_bf16x2(v[8 * k + 4], v[8 * k + 5]), pack_bf16x2(v[8 * k + 6], v[8 * k + 7]));
  }
  // Hand the staged box at (x, y) to TMA.
  S1C_DEV void issue(const void* tmap, const uint8_t* buf, int x, int y, bool reduce) {
    fence_proxy_async();
    __syncwarp();
    if (lane == 0) {
      if (reduce) tma_reduce_add_2d(tmap, buf, x, y);
      else tma_store_2d(tmap, buf, x, y);
      bulk_commit();
    }
    ++count;
  }
};

S1C_DEV void add_bias32(float* v, const float* bias, int col) {
  const float4* b4 = reinterpret_cast<const float4*>(bias + col);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 b = __ldg(b4 + i);
    v[4 * i] += b.x; v[4 * i + 1] += b.y; v[4 * i + 2] += b.z; v[4 * i + 3] += b.w;
  }
}

// Split-K partial sums: the raw fp32 accumulators of one split, stored (32-column units) into that
// split's slice of the workspace. Each element of a slice is written by exactly one tile.
// `part` of `parts` (1 or 2) epilogue warps sharing a TMEM lane quadrant takes that share of the
// tile's column units.
template <int BN>
__device__ __forceinline__ void gemm_epilogue_partial(const GemmArgs& args, const CUtensorMap* tmC, Stager& sg,
                                                      uint32_t t, int y0, int n0, int part, int parts) {
#pragma unroll 1
  for (int c = part * (BN / 32) / parts; c < (part + 1) * (BN / 32) / parts; ++c) {
    float v[32];
    tmem_ld32(t + c * 32, v);
    const int col = n0 + c * 32;
    if (col >= args.N) continue;
    uint8_t* buf = sg.acquire();
    sg.put_f32x32(buf, v);
    sg.issue(tmC, buf, col, y0, false);
  }
}

// cos / sin of one row's RoPE angles (32 pairs, the angle p * inv_freq[j] formed in fp32,
// split_rope.metal:46-76), fetched for a tile before its accumulator is ready so that the table's
// latency overlaps the tile's MMAs: from the per-position table, else by sincosf. Tiles of the v
// columns (n0 >= rope_cols) fetch nothing.
struct RopeRow {
  float cs[32], sn[32];
};
S1C_DEV void rope_prefetch(const GemmArgs& args, int row, bool m_ok, int n0, RopeRow& rr) {
  if (n0 >= args.rope_cols) return;
  const int pi = m_ok ? __ldg(args.pos + row) : 0;
  if (args.rope_tab) {
    const float4* tb = reinterpret_cast<const float4*>(args.rope_tab + (size_t)pi * 64);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 c4 = __ldg(tb + i), s4 = __ldg(tb + 8 + i);
      rr.cs[4 * i] = c4.x; rr.cs[4 * i + 1] = c4.y; rr.cs[4 * i + 2] = c4.z; rr.cs[4 * i + 3] = c4.w;
      rr.sn[4 * i] = s4.x; rr.sn[4 * i + 1] = s4.y; rr.sn[4 * i + 2] = s4.z; rr.sn[4 * i + 3] = s4.w;
    }
  } else {
    const float p = (float)pi;
#pragma unroll
    for (int j = 0; j < 32; ++j) sincosf(p * __ldg(args.inv_freq + j), &rr.sn[j], &rr.cs[j]);
  }
}

template <int BN, int EPI>
__device__ __forceinline__ void gemm_epilogue_tile(const GemmArgs& args, const CUtensorMap* tmC, Stager& sg,
                                                   uint32_t t, int row, bool m_ok, int y0, int n0, int n_block,
                                                   int part, int parts, const RopeRow& rr) {
  if constexpr (EPI == EPI_RESID || EPI == EPI_STORE || EPI == EPI_RESID16) {
    const bool f32 = (EPI == EPI_RESID) || (EPI == EPI_STORE && args.out_f32);
    if (f32) {
      // fp32 output: 32-column units. Rows past M add (or store) zeros.
#pragma unroll 1
      for (int c = part * (BN / 32) / parts; c < (part + 1) * (BN / 32) / parts; ++c) {
        float v[32];
        tmem_ld32(t + c * 32, v);
        const int col = n0 + c * 32;
        if (col >= args.N) continue;  // warp-uniform
        if (args.bias) add_bias32(v, args.bias, col);
        if constexpr (EPI == EPI_STORE) {
          if (args.act == ACT_RELU) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.0f);
          } else if (args.act == ACT_GELU) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
          }
        }
        if (!m_ok) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = 0.f;
        }
        uint8_t* buf = sg.acquire();
        sg.put_f32x32(buf, v);
        sg.issue(tmC, buf, col, y0, EPI == EPI_RESID);
      }
    } else {
      // 16-bit output, 64-column units: bf16 stores, or the f16 residual stream's reduce-add
      // (rows past M add zeros).
#pragma unroll 1
      for (int c = part * (BN / 64) / parts; c < (part + 1) * (BN / 64) / parts; ++c) {
        float v[64];
        tmem_ld32(t + c * 64, *reinterpret_cast<float(*)[32]>(v));
        tmem_ld32(t + c * 64 + 32, *reinterpret_cast<float(*)[32]>(v + 32));
        const int col = n0 + c * 64;
        if (col >= args.N) continue;
        if (args.bias) {
          add_bias32(v, args.bias, col);
          if (col + 32 < args.N) add_bias32(v + 32, args.bias, col + 32);
        }
        if constexpr (EPI == EPI_RESID16) {
          if (!m_ok) {
#pragma unroll
            for (int j = 0; j < 64; ++j) v[j] = 0.f;
          }
        } else {
          if (args.act == ACT_RELU) {
#pragma unroll
            for (int j = 0; j < 64; ++j) v[j] = fmaxf(v[j], 0.0f);
          } else if (args.act == ACT_GELU) {
#pragma unroll
            for (int j = 0; j < 64; ++j) v[j] = gelu_erf(v[j]);
          }
        }
        uint8_t* buf = sg.acquire();
        if constexpr (EPI == EPI_RESID16) sg.put_f16x64(buf, v);
        else sg.put_bf16x64(buf, v);
        sg.issue(tmC, buf, col, y0, EPI == EPI_RESID16);
      }
    }
  } else if constexpr (EPI == EPI_ROPE) {
    // Rotate-half RoPE of every 64-wide q/k head in the tile at this row's position, with the
    // row's cos / sin (`rr`, fetched by rope_prefetch before the accumulator wait) shared by the
    // tile's heads.
    const bool rope = n0 < args.rope_cols;  // uniform: q/k tiles never straddle the v columns
    const float(&cs)[32] = rr.cs;
    const float(&sn)[32] = rr.sn;
#pragma unroll 1
    for (int hh = part * (BN / 64) / parts; hh < (part + 1) * (BN / 64) / parts; ++hh) {
      const int col = n0 + hh * 64;
      if (col >= args.N) continue;  // warp-uniform
      uint8_t* buf = sg.acquire();
      // the head in two passes of 16 rotate-half pairs (j, j + 32): fewer live registers
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        float lo[16], hi[16];
        tmem_ld16(t + hh * 64 + q * 16, lo);
        tmem_ld16(t + hh * 64 + 32 + q * 16, hi);
        if (rope) {
          // lo' = a cos - b sin, hi' = a sin + b cos on packed pairs of columns (f32x2)
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const uint64_t a = f2_pack(lo[j], lo[j + 1]), b = f2_pack(hi[j], hi[j + 1]);
            const uint64_t c = f2_pack(cs[q * 16 + j], cs[q * 16 + j + 1]);
            const uint64_t sv = f2_pack(sn[q * 16 + j], sn[q * 16 + j + 1]);
            f2_unpack(f2_fma(a, c, f2_mul(f2_pack(-hi[j], -hi[j + 1]), sv)), lo[j], lo[j + 1]);
            f2_unpack(f2_fma(a, sv, f2_mul(b, c)), hi[j], hi[j + 1]);
          }
        }
        sg.put_bf16x16(buf, 2 * q, lo);
        sg.put_bf16x16(buf, 4 + 2 * q, hi);
      }
      sg.issue(tmC, buf, col, y0, false);
    }
  } else {  // EPI_GEGLU, BN == 256: columns [0,128) input, [128,256) gate
    static_assert(EPI != EPI_GEGLU || BN == 256, "GeGLU tiles are 128 input + 128 gate columns");
#pragma unroll 1
    for (int u = part * 2 / parts; u < (part + 1) * 2 / parts; ++u) {
      const int ocol = n_block * 128 + u * 64;
      if (ocol >= args.out_cols) continue;  // warp-uniform
      uint8_t* buf = sg.acquire();
#pragma unroll
      for (int h = 0; h < 4; ++h) {  // 16 input columns and their 16 gate columns at a time
        float a[16], g[16];
        tmem_ld16(t + u * 64 + h * 16, a);
        tmem_ld16(t + 128 + u * 64 + h * 16, g);
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          gelu_erf_x2(a[j], a[j + 1]);
          float p0, p1;
          f2_unpack(f2_mul(f2_pack(a[j], a[j + 1]), f2_pack(g[j], g[j + 1])), p0, p1);
          a[j] = p0;
          a[j + 1] = p1;
        }
        sg.put_bf16x16(buf, 2 * h, a);
      }
      sg.issue(tmC, buf, ocol, y0, false);
    }
  }
}

template <int BN, int EPI>
__global__ void __launch_bounds__(GEMM1_THREADS, 1)
    gemm_bf16_sm100(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const GemmArgs args) {
  constexpr int BM = GEMM_BM, BK = GEMM_BK, STAGES = gemm_stages(BN);
  constexpr uint32_t A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  static_assert(TMEM_COLS == 32 || TMEM_COLS == 64 || TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512,
                "TMEM allocations are powers of two from 32 to 512 columns");
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "tcgen05 M=128 needs N % 16 == 0, 16..256");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_u + 1023u) & ~1023u) - raw_u);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sStg = sB + STAGES * B_BYTES;  // 8 warps x 1 buffer x 4 KB, 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(sStg + 8 * GEMM_STG_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (args.M + BM - 1) / BM, num_n = (args.N + BN - 1) / BN;
  const int ksp = args.k_splits > 1 ? args.k_splits : 1;  // host keeps ksp <= nk
  const int num_tiles = num_m * num_n * ksp;
  const int nk = (args.K + BK - 1) / BK;
  // tile -> (m block, n block, k split); the split covers k blocks [kb0, kb1)
  auto decode = [&](int tile, int& m_block, int& n_block, int& kb0, int& kb1) {
    const int mn = tile / ksp, ks = tile % ksp;
    m_block = mn / num_n;
    n_block = mn % num_n;
    kb0 = ks * nk / ksp;
    kb1 = (ks + 1) * nk / ksp;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 32 * GEMM_EPI_WARPS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
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
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        int mb, nb, kb0, kb1;
        decode(tile, mb, nb, kb0, kb1);
        const int m0 = mb * BM, n0 = nb * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1u, args.status, DEV_TIMEOUT_PRODUCER, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(sA + s * A_BYTES, &tmA, &full[s], kb * BK, m0);
          tma_load_2d(sB + s * B_BYTES, &tmB, &full[s], kb * BK, n0);
          ++issued;
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      // Every load this thread issued must land before the CTA exits; only the last STAGES
      // can still be in flight.
      int back = issued < STAGES ? issued : STAGES;
      int ss = s;
      uint32_t pp = ph;
      for (int i = 0; i < back; ++i) {
        if (--ss < 0) {
          ss = STAGES - 1;
          pp ^= 1u;
        }
        mbar_wait(&full[ss], pp, args.status, DEV_TIMEOUT_DRAIN, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(BM, BN);
      // The MMA issue loop is kept short: it shares its SM sub-partition with epilogue warps, and
      // every instruction it waits to issue is a gap in the tensor pipe. Descriptors of stage 0
      // are built once; a stage's are these plus its byte offset (the start-address field holds
      // address >> 4, and no stage crosses the field's 256 KB range).
      const uint64_t adesc0 = sdesc_kmajor_sw128(smem_u32(sA)), bdesc0 = sdesc_kmajor_sw128(smem_u32(sB));
      int s = 0, acc = 0;
      uint32_t ph = 0, aph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], aph ^ 1u, args.status, DEV_TIMEOUT_MMA_TEMPTY, abort_flag)) break;
        tc_fence_after();
        const uint32_t d = tmem_base + (uint32_t)(acc * BN);
        int mb, nb, kb0, kb1;
        decode(tile, mb, nb, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[s], ph, args.status, DEV_TIMEOUT_MMA_FULL, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Stepping K by 16 elements adds 32 bytes (2 in the descriptor's >>4 address field).
          const uint64_t ad = adesc0 + (uint64_t)(s * (A_BYTES >> 4)), bd = bdesc0 + (uint64_t)(s * (B_BYTES >> 4));
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d, ad + 2u * k, bd + 2u * k, idesc, (kb != kb0 || k != 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) aph ^= 1u;
      }
      // All MMAs this thread issued complete before TMEM is released.
      umma_commit(drain);
      mbar_wait(drain, 0, args.status, DEV_TIMEOUT_DRAIN, nullptr);
    }
  } else {
    const int quad = warp & 3;  // TMEM lanes this warp may read: [32*quad, 32*quad + 32)
    constexpr int PARTS = GEMM_EPI_WARPS / 4, NBUF = 8 / GEMM_EPI_WARPS;
    const int part = (warp - 2) / 4;  // which share of the tile's columns
    Stager sg{sStg + (warp - 2) * NBUF * GEMM_STG_BYTES, 0u, lane, NBUF};
    if (lane == 0) prefetch_tmap(&tmC);
    int acc = 0;
    uint32_t aph = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, n_block, kb0, kb1;
      decode(tile, mb, n_block, kb0, kb1);
      const int m0 = mb * BM;
      const int y0 = m0 + quad * 32;
      const int row = y0 + lane;
      RopeRow rr;
      if constexpr (EPI == EPI_ROPE) {
        if (ksp == 1) rope_prefetch(args, row, row < args.M, n_block * BN, rr);
      }
      if (!mbar_wait_warp(&tfull[acc], aph, args.status, DEV_TIMEOUT_EPILOGUE, abort_flag)) break;
      tc_fence_after();
      const uint32_t t = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
      if (ksp > 1)
        gemm_epilogue_partial<BN>(args, &tmC, sg, t, (tile % ksp) * args.split_rows + y0, n_block * BN, part, PARTS);
      else
        gemm_epilogue_tile<BN, EPI>(args, &tmC, sg, t, row, row < args.M, y0, n_block * BN, n_block, part, PARTS,
                                    rr);
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) aph ^= 1u;
    }
    // Stores in flight finish (and stop reading shared memory) before the CTA exits.
    if (lane == 0) bulk_wait_all();
  }
  __syncwarp();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// cos | sin of the RoPE angles p * inv_freq[j] for positions [0, P): row p holds cos for
// j = 0..31 then sin for j = 0..31, each from the fp32 angle exactly as the epilogue forms it.
__global__ void rope_table_kernel(float* __restrict__ tab, int P, const float* __restrict__ inv_freq) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P * 32) return;
  const int p = i >> 5, j = i & 31;
  float sn, cs;
  sincosf((float)p * inv_freq[j], &sn, &cs);
  tab[(size_t)p * 64 + j] = cs;
  tab[(size_t)p * 64 + 32 + j] = sn;
}

}  // namespace s1c
