// Finalisation of a split-K GEMM: split s stored its fp32 partial sums in slice s of a workspace
// [splits][rows][N]; this kernel adds the slices in split order (so the result does not depend on
// scheduling), applies the GEMM's epilogue (bias / activation, RoPE, GeGLU, or the residual add)
// and writes the real output. Used for GEMMs with too few output tiles to occupy the GPU (small
// token counts: the single-request latency path), where splitting K puts every SM on the weights.
#pragma once
#include "gemm_sm100.cuh"

namespace s1c {

struct SplitKFinal {
  const float* ws;    // [splits][rows][N] fp32 partial sums
  int splits, rows;   // slices and rows per slice
  int M, N;
  void* out;          // output (bf16, or fp32 when out_f32 / EPI_RESID, f16 for EPI_RESID16)
  int ldo;            // output row pitch, elements
  const float* bias;  // EPI_STORE / EPI_RESID / EPI_RESID16
  int act, out_f32;   // EPI_STORE
  const int* pos;     // EPI_ROPE
  const float* inv_freq;
  int rope_cols;
  int out_cols;       // EPI_GEGLU: I; workspace columns are the interleaved Wi rows
};

// Sum of the split slices at (r, c .. c+7), in split order.
S1C_DEV void slice_sum8(const SplitKFinal& f, int r, int c, float (&v)[8]) {
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = 0.f;
  for (int s = 0; s < f.splits; ++s) {
    const float4* p = reinterpret_cast<const float4*>(f.ws + ((size_t)s * f.rows + r) * f.N + c);
    const float4 a = p[0], b = p[1];
    v[0] += a.x; v[1] += a.y; v[2] += a.z; v[3] += a.w; v[4] += b.x; v[5] += b.y; v[6] += b.z; v[7] += b.w;
  }
}

// One thread per (row, 8 consecutive output columns).
template <int EPI>
__global__ void splitk_finalize_kernel(const SplitKFinal f) {
  pdl_trigger();
  pdl_wait();
  const int groups = (EPI == EPI_GEGLU ? f.out_cols : f.N) / 8;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)f.M * groups) return;
  const int r = (int)(idx / groups), g = (int)(idx % groups);
  float v[8];
  if constexpr (EPI == EPI_GEGLU) {
    const int o = g * 8, t = o / 128, j = o % 128;
    float in[8], gt[8];
    slice_sum8(f, r, t * 256 + j, in);
    slice_sum8(f, r, t * 256 + 128 + j, gt);
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = gelu_erf(in[i]) * gt[i];
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(f.out) + (size_t)r * f.ldo + o;
    *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  } else if constexpr (EPI == EPI_ROPE) {
    // 8 columns of one 64-wide head: rotate-half pairs (j, j + 32) live in the same head, so the
    // thread holding columns of the first half rotates them with their partners from the second.
    const int c = g * 8, head0 = c & ~63, j0 = c & 63;
    if (j0 >= 32) return;
    float a[8], b[8];
    slice_sum8(f, r, c, a);
    slice_sum8(f, r, c + 32, b);
    if (head0 < f.rope_cols) {
      const float p = (float)f.pos[r];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float sn, cs;
        sincosf(p * f.inv_freq[j0 + i], &sn, &cs);
        const float u = a[i], w = b[i];
        a[i] = u * cs - w * sn;
        b[i] = u * sn + w * cs;
      }
    }
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(f.out) + (size_t)r * f.ldo + c;
    *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(a[0], a[1]), pack_bf16x2(a[2], a[3]),
                                                pack_bf16x2(a[4], a[5]), pack_bf16x2(a[6], a[7]));
    *reinterpret_cast<uint4*>(dst + 32) = make_uint4(pack_bf16x2(b[0], b[1]), pack_bf16x2(b[2], b[3]),
                                                     pack_bf16x2(b[4], b[5]), pack_bf16x2(b[6], b[7]));
  } else if constexpr (EPI == EPI_RESID) {
    const int c = g * 8;
    slice_sum8(f, r, c, v);
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(f.out) + (size_t)r * f.ldo + c);
    float4 a = dst[0], b = dst[1];
    const float* bias = f.bias;
    a.x += v[0] + (bias ? bias[c] : 0.f); a.y += v[1] + (bias ? bias[c + 1] : 0.f);
    a.z += v[2] + (bias ? bias[c + 2] : 0.f); a.w += v[3] + (bias ? bias[c + 3] : 0.f);
    b.x += v[4] + (bias ? bias[c + 4] : 0.f); b.y += v[5] + (bias ? bias[c + 5] : 0.f);
    b.z += v[6] + (bias ? bias[c + 6] : 0.f); b.w += v[7] + (bias ? bias[c + 7] : 0.f);
    dst[0] = a;
    dst[1] = b;
  } else if constexpr (EPI == EPI_RESID16) {
    // f16(residual + (sum + bias)): the sum rounded once
    const int c = g * 8;
    slice_sum8(f, r, c, v);
    uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(f.out) + (size_t)r * f.ldo + c);
    const uint4 u = *dst;
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 h = unpack_f16x2(w[i]);
      o[i] = pack_f16x2(h.x + (v[2 * i] + (f.bias ? f.bias[c + 2 * i] : 0.f)),
                        h.y + (v[2 * i + 1] + (f.bias ? f.bias[c + 2 * i + 1] : 0.f)));
    }
    *dst = make_uint4(o[0], o[1], o[2], o[3]);
  } else {  // EPI_STORE
    const int c = g * 8;
    slice_sum8(f, r, c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float x = v[i] + (f.bias ? f.bias[c + i] : 0.f);
      if (f.act == ACT_RELU) x = fmaxf(x, 0.f);
      else if (f.act == ACT_GELU) x = gelu_erf(x);
      v[i] = x;
    }
    if (f.out_f32) {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(f.out) + (size_t)r * f.ldo + c);
      dst[0] = make_float4(v[0], v[1], v[2], v[3]);
      dst[1] = make_float4(v[4], v[5], v[6], v[7]);
    } else {
      __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(f.out) + (size_t)r * f.ldo + c;
      *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                  pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
    }
  }
}

}  // namespace s1c
