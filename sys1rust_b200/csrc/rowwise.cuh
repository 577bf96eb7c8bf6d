// Row-wise memory-bound kernels: one warp per row of d values, 16-byte vector accesses,
// warp-shuffle reductions, two-pass (mean, then centred variance) LayerNorm statistics in fp32.
//
//   embed_ln      tok_emb gather + bias-free emb_norm (lib.rs:1534-1551); writes the encoder's
//                 residual stream (f16, the reference's storage type) and its bf16 copy (layer
//                 0's attn_norm is the identity, lib.rs:993-997, so that copy is the first Wqkv
//                 input).
//   layernorm     f16 (encoder) or fp32 (head) rows -> LayerNorm (weight, optional bias) -> bf16
//                 (lib.rs:630-641), optionally through a row gather (the scorer's marker rows,
//                 lib.rs:1787-1795).
//   final_to_head final_norm (lib.rs:1689), + type_emb of the row's qtype (lib.rs:1702-1708),
//                 then the first head layer's norm1 (lib.rs:1735): one pass over the row.
//   gather_rows   fp32 row gather (pooled rows, the pruned head layer's residual rows).
//   scorer_logits the scorer's last Linear(S -> 1) + bias, and the -1e4 fill of marker slots
//                 past marker_count (lib.rs:1799, :1851-1857).
#pragma once
#include "common.cuh"

namespace s1c {

template <int D>
struct RowVec {
  static_assert(D % 256 == 0, "row width must be a multiple of 256");
  static constexpr int CHUNKS = D / 256;  // 8-element chunks per lane
  float v[CHUNKS * 8];
};

template <int D>
S1C_DEV void load_row_f32(const float* src, RowVec<D>& r, int lane) {
#pragma unroll
  for (int c = 0; c < RowVec<D>::CHUNKS; ++c) {
    const float4* p = reinterpret_cast<const float4*>(src + c * 256 + lane * 8);
    const float4 a = p[0], b = p[1];
    float* o = r.v + c * 8;
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w; o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
  }
}
template <int D>
S1C_DEV void load_row_bf16(const __nv_bfloat16* src, RowVec<D>& r, int lane) {
#pragma unroll
  for (int c = 0; c < RowVec<D>::CHUNKS; ++c) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + c * 256 + lane * 8);
    float* o = r.v + c * 8;
    o[0] = bf16_lo(u.x); o[1] = bf16_hi(u.x); o[2] = bf16_lo(u.y); o[3] = bf16_hi(u.y);
    o[4] = bf16_lo(u.z); o[5] = bf16_hi(u.z); o[6] = bf16_lo(u.w); o[7] = bf16_hi(u.w);
  }
}
template <int D>
S1C_DEV void load_row_f16(const __half* src, RowVec<D>& r, int lane) {
#pragma unroll
  for (int c = 0; c < RowVec<D>::CHUNKS; ++c) {
    const uint4 u = *reinterpret_cast<const uint4*>(src + c * 256 + lane * 8);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float* o = r.v + c * 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack_f16x2(w[i]);
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
}
template <int D>
S1C_DEV void load_row(const float* src, RowVec<D>& r, int lane) { load_row_f32<D>(src, r, lane); }
template <int D>
S1C_DEV void load_row(const __half* src, RowVec<D>& r, int lane) { load_row_f16<D>(src, r, lane); }
template <int D>
S1C_DEV void store_row_f16(__half* dst, const RowVec<D>& r, int lane) {
#pragma unroll
  for (int c = 0; c < RowVec<D>::CHUNKS; ++c) {
    const float* o = r.v + c * 8;
    *reinterpret_cast<uint4*>(dst + c * 256 + lane * 8) =
        make_uint4(pack_f16x2(o[0], o[1]), pack_f16x2(o[2], o[3]), pack_f16x2(o[4], o[5]), pack_f16x2(o[6], o[7]));
  }
}
template <int D>
S1C_DEV void store_row_f32(float* dst, const RowVec<D>& r, int lane) {
#pragma unroll
  for (int c = 0; c < RowVec<D>::CHUNKS; ++c) {
    float4* p = reinterpret_cast<float4*>(dst + c * 256 + lane * 8);
    const float* o = r.v + c * 8;
    p[0] = make_float4(o[0], o[1], o[2], o[3]);
    p[1] = make_float4(o[4], o[5], o[6], o[7]);
  }
}
template <int D>
S1C_DEV void store_row_bf16(__nv_bfloat16* dst, const RowVec<D>& r, int lane) {
#pragma unroll
  for (int c = 0; c < RowVec<D>::CHUNKS; ++c) {
    const float* o = r.v + c * 8;
    uint4 u;
    u.x = pack_bf16x2(o[0], o[1]);
    u.y = pack_bf16x2(o[2], o[3]);
    u.z = pack_bf16x2(o[4], o[5]);
    u.w = pack_bf16x2(o[6], o[7]);
    *reinterpret_cast<uint4*>(dst + c * 256 + lane * 8) = u;
  }
}

S1C_DEV float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// In-place LayerNorm of a register row: (x - mean) * rsqrt(var + eps) * w (+ b).
template <int D>
S1C_DEV void layernorm_row(RowVec<D>& r, const float* w, const float* b, float eps, int lane) {
  constexpr int N = RowVec<D>::CHUNKS * 8;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) s += r.v[i];
  const float mean = warp_sum(s) * (1.0f / D);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float d = r.v[i] - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(warp_sum(q) * (1.0f / D) + eps);
#pragma unroll
  for (int c = 0; c < RowVec<D>::CHUNKS; ++c) {
    const float4* w4 = reinterpret_cast<const float4*>(w + c * 256 + lane * 8);
    const float4 wa = __ldg(w4), wb = __ldg(w4 + 1);
    const float wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
    float bv[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (b) {
      const float4* b4 = reinterpret_cast<const float4*>(b + c * 256 + lane * 8);
      const float4 ba = __ldg(b4), bb = __ldg(b4 + 1);
      bv[0] = ba.x; bv[1] = ba.y; bv[2] = ba.z; bv[3] = ba.w; bv[4] = bb.x; bv[5] = bb.y; bv[6] = bb.z; bv[7] = bb.w;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) r.v[c * 8 + j] = (r.v[c * 8 + j] - mean) * rstd * wv[j] + bv[j];
  }
}

template <int D>
__global__ void embed_ln_kernel(const uint32_t* __restrict__ ids, int T, const __nv_bfloat16* __restrict__ tok_emb,
                                int vocab, const float* __restrict__ w, float eps, __half* __restrict__ h,
                                __nv_bfloat16* __restrict__ x, int* status) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  uint32_t id = ids[row];
  if (id >= (uint32_t)vocab) {  // the host validates ids; never read outside the table
    if (lane == 0) report(status, DEV_BAD_INDEX);
    id = 0;
  }
  RowVec<D> r;
  load_row_bf16<D>(tok_emb + (size_t)id * D, r, lane);
  layernorm_row<D>(r, w, nullptr, eps, lane);
  store_row_f16<D>(h + (size_t)row * D, r, lane);
  store_row_bf16<D>(x + (size_t)row * D, r, lane);
}

// In-place LayerNorm of a register row with the weight (and bias) already in registers.
template <int D, bool HAS_B>
S1C_DEV void layernorm_row_w(RowVec<D>& r, const RowVec<D>& w, const RowVec<D>& b, float eps) {
  constexpr int N = RowVec<D>::CHUNKS * 8;
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) s += r.v[i];
  const float mean = warp_sum(s) * (1.0f / D);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float d = r.v[i] - mean;
    q += d * d;
  }
  const float rstd = rsqrtf(warp_sum(q) * (1.0f / D) + eps);
#pragma unroll
  for (int i = 0; i < N; ++i) r.v[i] = (r.v[i] - mean) * rstd * w.v[i] + (HAS_B ? b.v[i] : 0.f);
}

// Grid-stride over rows, one warp per row at a time, two rows in flight per warp: the grid is
// sized to the SMs (every SM gets the same share of rows, no partial last wave), and the
// LayerNorm weight / bias are read once per warp into registers -- before the dependency wait,
// since no kernel of the forward writes them. (Prefetching each warp's next two rows into L2 with
// a bulk prefetch measured 4-5 % slower in the forward.)
template <int D, bool HAS_B, typename TIn>
__global__ void __launch_bounds__(256) layernorm_kernel(const TIn* __restrict__ in, const int* __restrict__ gather,
                                                        int rows, const float* __restrict__ w,
                                                        const float* __restrict__ b, float eps,
                                                        __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  RowVec<D> wv, bv;
  load_row_f32<D>(w, wv, lane);
  if constexpr (HAS_B) load_row_f32<D>(b, bv, lane);
  pdl_wait();
  const int nw = gridDim.x * (blockDim.x >> 5);
  int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  for (; row + nw < rows; row += 2 * nw) {
    const int r1 = row + nw;
    RowVec<D> x0, x1;
    load_row<D>(in + (size_t)(gather ? gather[row] : row) * D, x0, lane);
    load_row<D>(in + (size_t)(gather ? gather[r1] : r1) * D, x1, lane);
    layernorm_row_w<D, HAS_B>(x0, wv, bv, eps);
    store_row_bf16<D>(out + (size_t)row * D, x0, lane);
    layernorm_row_w<D, HAS_B>(x1, wv, bv, eps);
    store_row_bf16<D>(out + (size_t)r1 * D, x1, lane);
  }
  if (row < rows) {
    RowVec<D> x0;
    load_row<D>(in + (size_t)(gather ? gather[row] : row) * D, x0, lane);
    layernorm_row_w<D, HAS_B>(x0, wv, bv, eps);
    store_row_bf16<D>(out + (size_t)row * D, x0, lane);
  }
}

template <int D>
__global__ void final_to_head_kernel(const __half* __restrict__ h, int T, const float* __restrict__ final_w, float eps,
                                     float* __restrict__ hidden_out, int hidden_rows, const int* __restrict__ token_row,
                                     const uint32_t* __restrict__ qtype, const float* __restrict__ type_emb,
                                     const float* __restrict__ n1w, const float* __restrict__ n1b,
                                     float* __restrict__ h2, __nv_bfloat16* __restrict__ x) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  RowVec<D> r;
  load_row_f16<D>(h + (size_t)row * D, r, lane);
  layernorm_row<D>(r, final_w, nullptr, eps, lane);
  if (hidden_out && row < hidden_rows) store_row_f32<D>(hidden_out + (size_t)row * D, r, lane);
  const uint32_t qt = qtype[token_row[row]];
  RowVec<D> te;
  load_row_f32<D>(type_emb + (size_t)qt * D, te, lane);
#pragma unroll
  for (int i = 0; i < RowVec<D>::CHUNKS * 8; ++i) r.v[i] += te.v[i];
  store_row_f32<D>(h2 + (size_t)row * D, r, lane);
  layernorm_row<D>(r, n1w, n1b, 1e-5f, lane);
  store_row_bf16<D>(x + (size_t)row * D, r, lane);
}

__global__ void gather_rows_f32_kernel(const float* __restrict__ in, const int* __restrict__ idx, int rows, int d,
                                       float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  if (row >= rows) return;
  const float4* s = reinterpret_cast<const float4*>(in + (size_t)idx[row] * d);
  float4* o = reinterpret_cast<float4*>(out + (size_t)row * d);
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) o[i] = s[i];
}

__global__ void gather_rows_bf16_kernel(const __nv_bfloat16* __restrict__ in, const int* __restrict__ idx, int rows,
                                        int d, __nv_bfloat16* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  if (row >= rows) return;
  const uint4* s = reinterpret_cast<const uint4*>(in + (size_t)idx[row] * d);
  uint4* o = reinterpret_cast<uint4*>(out + (size_t)row * d);
  for (int i = threadIdx.x; i < d / 8; i += blockDim.x) o[i] = s[i];
}

// logits[r] = dot(hid[r, :S], w3) + b3 for r < n * kmax; slots past marker_count are -1e4.
__global__ void scorer_logits_kernel(const float* __restrict__ hid, int R, int S, const float* __restrict__ w3,
                                     const float* __restrict__ b3, const int* __restrict__ marker_count, int kmax,
                                     float* __restrict__ logits) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= R) return;
  float s = 0.f;
  for (int i = lane; i < S; i += 32) s += hid[(size_t)row * S + i] * __ldg(w3 + i);
  s = warp_sum(s);
  if (lane == 0) {
    const int seq = row / kmax, k = row % kmax;
    logits[row] = (k < marker_count[seq]) ? s + b3[0] : -1e4f;
  }
}

}  // namespace s1c
