// Finalisation of a split-K GEMM: the splits have reduce-added their fp32 partial sums into a
// workspace [rows, N]; this kernel applies the GEMM's epilogue (bias / activation, RoPE, GeGLU)
// to the sums, writes the real output, and zeroes the workspace again so that it is ready for the
// next split-K GEMM. Used for GEMMs with too few output tiles to occupy the GPU (small token counts:
// the single-request latency path), where splitting K is what puts every SM on the weight stream.
#pragma once
#include "gemm_sm100.cuh"

namespace s1c {

struct SplitKFinal {
  float* ws;          // [M, N] fp32 partial sums, row pitch N; zeroed on exit
  int M, N;
  void* out;          // output (bf16, or fp32 when out_f32)
  int ldo;            // output row pitch, elements
  const float* bias;  // EPI_STORE
  int act, out_f32;   // EPI_STORE
  const int* pos;     // EPI_ROPE
  const float* inv_freq;
  int rope_cols;
  int out_cols;       // EPI_GEGLU: I; workspace columns are the interleaved Wi rows
};

// One thread per (row, 8 consecutive output columns).
template <int EPI>
__global__ void splitk_finalize_kernel(const SplitKFinal f) {
  const int groups = (EPI == EPI_GEGLU ? f.out_cols : f.N) / 8;
  const long idx = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long)f.M * groups) return;
  const int r = (int)(idx / groups), g = (int)(idx % groups);
  float* wrow = f.ws + (size_t)r * f.N;
  float v[8];
  if constexpr (EPI == EPI_GEGLU) {
    const int o = g * 8, t = o / 128, j = o % 128;
    float* in = wrow + t * 256 + j;
    float* gt = wrow + t * 256 + 128 + j;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      v[i] = gelu_erf(in[i]) * gt[i];
      in[i] = 0.f;
      gt[i] = 0.f;
    }
    __nv_bfloat16* dst = static_cast<__nv_bfloat16*>(f.out) + (size_t)r * f.ldo + o;
    *reinterpret_cast<uint4*>(dst) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
  } else if constexpr (EPI == EPI_ROPE) {
    // 8 columns of one 64-wide head: rotate-half pairs (j, j + 32) live in the same head, so a
    // thread with columns in the first half rotates them with their partners from the second.
    const int c = g * 8, head0 = c & ~63, j0 = c & 63;
    if (j0 >= 32) return;  // the first-half thread of the pair writes both halves
    float* x1 = wrow + c;
    float* x2 = wrow + c + 32;
    float a[8], b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      a[i] = x1[i];
      b[i] = x2[i];
      x1[i] = 0.f;
      x2[i] = 0.f;
    }
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
  } else {  // EPI_STORE
    const int c = g * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float x = wrow[c + i] + (f.bias ? f.bias[c + i] : 0.f);
      if (f.act == ACT_RELU) x = fmaxf(x, 0.f);
      else if (f.act == ACT_GELU) x = gelu_erf(x);
      v[i] = x;
      wrow[c + i] = 0.f;
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
