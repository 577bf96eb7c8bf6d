// libs1c: the C ABI of include/s1c.h and the host runtime that drives the sm_100a kernels.
//
// One s1c_backend per GPU: weights resident in HBM (bf16 matrices, fp32 vectors), activation
// buffers sized for a packed-token capacity, TMA descriptors built once per buffer, one CUDA
// stream. A forward packs the batch on the host (Packing::new, laya-mlx/src/lib.rs:906-930),
// uploads a small metadata arena, and enqueues the whole model on the stream:
//   embed_ln -> 28 x [LN, GEMM+RoPE, attention, GEMM+residual, LN, GEMM+GeGLU, GEMM+residual]
//   -> final LN + type embedding + head norm1 -> head layers (last one pruned to the scorer's
//   rows, lib.rs:1728-1748) -> scorer -> logits / pooled.
// The encoder's residual stream is stored f16, as the reference's f16 model stores it (the
// residual GEMMs add into it in place); the head's residual streams are fp32.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <nvtx3/nvToolsExt.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/s1c.h"
#include "attention.cuh"
#include "attention_tc.cuh"
#include "gemm_sm100.cuh"
#include "gemm_sm100_2cta.cuh"
#include "gemm_sm100_csk.cuh"
#include "splitk.cuh"
#include "rowwise.cuh"
#include "safetensors.h"
#include "server.h"
#include "decode.h"

using namespace s1c;
typedef __nv_bfloat16 bf16;

namespace {

// ---------------------------------------------------------------------------------------------
// errors

struct S1cError : std::runtime_error {
  s1c_status code;
  S1cError(s1c_status c, const std::string& m) : std::runtime_error(m), code(c) {}
};

#define CK(call)                                                                                  \
  do {                                                                                            \
    cudaError_t e_ = (call);                                                                      \
    if (e_ != cudaSuccess)                                                                        \
      throw S1cError(S1C_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));          \
  } while (0)

thread_local std::string g_create_error;

// ---------------------------------------------------------------------------------------------
// host numerics

uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40);  // quiet NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float f16_bits_to_f32(uint16_t h) {
  const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
  uint32_t u;
  if (e == 0) {
    if (m == 0) {
      u = s;
    } else {  // subnormal
      int sh = 0;
      while (!(m & 0x400u)) {
        m <<= 1;
        ++sh;
      }
      m &= 0x3ffu;
      u = s | ((uint32_t)(127 - 15 - sh + 1) << 23) | (m << 13);
    }
  } else if (e == 31) {
    u = s | 0x7f800000u | (m << 13);
  } else {
    u = s | ((e + 127 - 15) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
uint16_t f32_to_f16_bits(float f) {
  const __half_raw r = __float2half_rn(f);  // round to nearest even (cuda_fp16, host side)
  return r.x;
}
float bf16_bits_to_f32(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
float elem_f32(const s1c_tensor& t, size_t i) {
  switch (t.dtype) {
    case S1C_DT_F32: return static_cast<const float*>(t.data)[i];
    case S1C_DT_F16: return f16_bits_to_f32(static_cast<const uint16_t*>(t.data)[i]);
    case S1C_DT_BF16: return bf16_bits_to_f32(static_cast<const uint16_t*>(t.data)[i]);
    case S1C_DT_F64: return (float)static_cast<const double*>(t.data)[i];
  }
  throw S1cError(S1C_ERR_WEIGHTS, std::string(t.name) + ": unsupported dtype");
}

// ---------------------------------------------------------------------------------------------
// TMA descriptors

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  if (!fn) throw S1cError(S1C_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  return fn;
}

// 2D row-major matrix [rows, cols] (row pitch `ld` elements) tiled in boxes of box_rows x 128 bytes
// with the 128-byte swizzle: bf16 / f16 boxes are 64 elements wide, fp32 boxes 32.
CUtensorMap make_tmap_dt(const void* ptr, CUtensorMapDataType dt, uint64_t rows, uint64_t cols, uint64_t ld,
                         uint32_t box_rows) {
  const uint64_t es = dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * es) % 16)
    throw S1cError(S1C_ERR_ARG, "TMA operand must be 16-byte aligned with a 16-byte multiple row pitch");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * es};
  cuuint32_t box[2] = {(cuuint32_t)(128 / es), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw S1cError(S1C_ERR_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return m;
}
CUtensorMap make_tmap_t(const void* ptr, bool f32, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
  return make_tmap_dt(ptr, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rows, cols, ld,
                      box_rows);
}
// K-major bf16 GEMM / attention operand [rows, k], boxes of box_rows x 64 elements.
CUtensorMap make_tmap(const void* ptr, uint64_t rows, uint64_t k, uint64_t ld, uint32_t box_rows) {
  return make_tmap_t(ptr, false, rows, k, ld, box_rows);
}
// A weight (B operand) with its TMA maps: 256-row boxes for the one-CTA kernel, 128-row boxes
// for the two-CTA kernel (each CTA of a pair loads half of the 256-row tile) and the 128-wide
// cluster split-K tiles, 64-row boxes for the 64-wide cluster split-K tiles and the GeGLU halves.
struct WeightMap {
  CUtensorMap full, half, quarter;
};
WeightMap make_wmap(const void* ptr, uint64_t rows, uint64_t k, uint64_t ld) {
  return WeightMap{make_tmap(ptr, rows, k, ld, 256), make_tmap(ptr, rows, k, ld, 128), make_tmap(ptr, rows, k, ld, 64)};
}
// GEMM output map: boxes of 32 rows x 128 bytes (one epilogue warp's slice).
CUtensorMap make_out_tmap(const void* ptr, bool f32, uint64_t rows, uint64_t cols, uint64_t ld) {
  return make_tmap_t(ptr, f32, rows, cols, ld, 32);
}
// The same for an f16 output (the encoder's residual stream, EPI_RESID16).
CUtensorMap make_out_tmap_f16(const void* ptr, uint64_t rows, uint64_t cols, uint64_t ld) {
  return make_tmap_dt(ptr, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, rows, cols, ld, 32);
}

// ---------------------------------------------------------------------------------------------
// kernel launch helpers

// Launch with programmatic stream serialisation when `t_pdl` is set (see pdl_trigger / pdl_wait in
// common.cuh): the kernel may start while its predecessor drains, and waits on the device before
// touching the predecessor's data.
thread_local bool t_pdl = true;
// GEMM kernels the load check turned off for the handle whose forward is being enqueued on this
// thread (launch_gemm's shape rule then never picks them).
constexpr int GEMM_OFF_2CTA = 1, GEMM_OFF_CSK = 2;
thread_local int t_gemm_off = 0;
template <typename... P, typename... A>
void launch_k(void (*kernel)(P...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = t_pdl ? 1 : 0;
  CK(cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...));
}

constexpr int GEMM_BN = 256;

template <int EPI>
void set_gemm_smem() {
  CK(cudaFuncSetAttribute(gemm_bf16_sm100<GEMM_BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)gemm_smem_bytes(GEMM_BN)));
  if constexpr (EPI != EPI_GEGLU)
    CK(cudaFuncSetAttribute(gemm_bf16_sm100<128, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                            (int)gemm_smem_bytes(128)));
  CK(cudaFuncSetAttribute(gemm2_bf16_sm100<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)gemm2_smem_bytes()));
}
template <int BN, int EPI>
void set_csk_smem() {
  CK(cudaFuncSetAttribute(gemm_csk_sm100<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                          (int)csk_smem_bytes<BN>()));
}
void set_all_gemm_smem() {
  set_csk_smem<128, EPI_STORE>();
  set_csk_smem<128, EPI_ROPE>();
  set_csk_smem<128, EPI_GEGLU>();
  set_csk_smem<128, EPI_RESID>();
  set_csk_smem<128, EPI_RESID16>();
  set_csk_smem<64, EPI_STORE>();
  set_csk_smem<64, EPI_ROPE>();
  set_csk_smem<64, EPI_RESID>();
  set_csk_smem<64, EPI_RESID16>();
  set_gemm_smem<EPI_STORE>();
  set_gemm_smem<EPI_ROPE>();
  set_gemm_smem<EPI_GEGLU>();
  set_gemm_smem<EPI_RESID>();
  set_gemm_smem<EPI_RESID16>();
}

// Where a GEMM's output goes, for the split-K path: the output buffer and its row pitch (the
// residual stream for residual GEMMs), and the fp32 workspace that holds one slice of partial sums
// per split.
struct SplitCtx {
  float* ws;
  size_t ws_bytes;
  void* out;
  int ldo;
};

// Split-K factor for a GEMM with few output tiles: enough splits to cover the SMs, at least one
// 64-wide K block per split, at most 16 splits, partial-sum traffic bounded by the weight traffic,
// slices within the workspace. 1 = no split.
int pick_k_splits(int M, int N, int K, int num_sms, size_t ws_bytes) {
  const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * ((N + GEMM_BN - 1) / GEMM_BN);
  const int nk = (K + GEMM_BK - 1) / GEMM_BK;
  if (tiles * 2 > num_sms) return 1;
  const int rows = (M + GEMM_BM - 1) / GEMM_BM * GEMM_BM;
  // Partial sums of all splits (splits x rows x N fp32) stay within twice the weight bytes (N x K
  // bf16): at most K / rows splits.
  int ksp = std::max(1, std::min({num_sms / tiles, nk, 16, K / rows}));
  const size_t slice = (size_t)rows * N * 4;
  while (ksp > 1 && (size_t)ksp * slice > ws_bytes) --ksp;
  return ksp;
}

// Cluster split-K plan (gemm_sm100_csk.cuh) for a GEMM with few output tiles: the tile width
// (128, or 64 when that puts more SMs on the weights; GeGLU tiles are always 128 wide) and the
// cluster size C (1, 2, 4 or 8 CTAs, each a K split of at least one 64-wide block), as many CTAs
// as fit on the SMs in one wave.
struct CskPlan {
  int bn = 128, C = 1, tiles = 0;
};
CskPlan plan_csk(int M, int N, int K, int num_sms, bool geglu) {
  CskPlan best;
  const int nk = (K + GEMM_BK - 1) / GEMM_BK;
  for (int bn : {128, 64}) {
    if (geglu && bn != 128) continue;
    const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * ((N + bn - 1) / bn);
    int C = CSK_MAX_C;
    while (C > 1 && (C > nk || tiles * C > num_sms)) C >>= 1;
    if (best.tiles == 0 || tiles * C > best.tiles * best.C) best = CskPlan{bn, C, tiles};
  }
  return best;
}

template <int BN, int EPI>
void launch_csk_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CskArgs& a, int tiles, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(tiles * a.C));
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = csk_smem_bytes<BN>();
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)a.C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = t_pdl ? 2 : 1;
  CK(cudaLaunchKernelEx(&cfg, gemm_csk_sm100<BN, EPI>, ta, tb, a));
}

template <int EPI>
void launch_csk(const CUtensorMap& ta, const WeightMap& tb, const GemmArgs& g, const SplitCtx& sk, int num_sms,
                cudaStream_t st) {
  const CskPlan p = plan_csk(g.M, g.N, g.K, num_sms, EPI == EPI_GEGLU);
  CskArgs a{};
  a.M = g.M; a.N = g.N; a.K = g.K; a.C = p.C;
  a.out = sk.out; a.ldo = sk.ldo;
  a.bias = g.bias; a.act = g.act; a.out_f32 = g.out_f32;
  a.pos = g.pos; a.inv_freq = g.inv_freq; a.rope_cols = g.rope_cols; a.out_cols = g.out_cols;
  a.status = g.status;
  a.pf = g.pf; a.pf_bytes = g.pf_bytes;
  if constexpr (EPI == EPI_GEGLU) {
    launch_csk_bn<128, EPI>(ta, tb.quarter, a, p.tiles, st);
  } else {
    if (p.bn == 128) launch_csk_bn<128, EPI>(ta, tb.half, a, p.tiles, st);
    else launch_csk_bn<64, EPI>(ta, tb.quarter, a, p.tiles, st);
  }
}

// GEMM variant: 0 = by shape (cluster split-K when there are few tiles, an output context is
// given and K splits over a cluster, else the one- or two-CTA kernel), 1 = one-CTA 128 x 256, 2 = two-CTA, 3 = one-CTA split-K
// through the fp32 workspace and a finalize kernel (at least 2 splits), 4 = cluster split-K,
// 5 = one-CTA 128 x 128 (not for GeGLU). The 128 x 128 tiles would fill the last wave of the SMs
// better on N = 1024 (6.92 instead of 3.46 waves at 16k tokens) but measured 22 % slower there
// (half the MMA work per A tile loaded), so the shape rule never picks them.
template <int EPI>
void launch_gemm(const CUtensorMap& ta, const WeightMap& tb, const CUtensorMap& tc, const GemmArgs& a0, int num_sms,
                 cudaStream_t st, int variant = 0, const SplitCtx* sk = nullptr, int64_t* extra_launches = nullptr) {
  if (a0.M <= 0) return;
  GemmArgs a = a0;
  a.k_splits = 1;
  // Few output tiles (small token counts): the cluster split-K kernel, one launch per GEMM, when
  // its plan really splits K over a cluster (C >= 2). With C = 1 every CTA would walk the whole K
  // range of a 128-wide tile: the plain kernels are faster there (measured at 16k-SM scale: Wqkv
  // M = 512 9.8 vs 20.6 us, Wo2 M = 2048 18.6 vs 39.0 us).
  bool csk = sk && variant == 4;
  if (sk && variant == 0 && !(t_gemm_off & GEMM_OFF_CSK) &&
      ((a.M + GEMM_BM - 1) / GEMM_BM) * ((a.N + GEMM_BN - 1) / GEMM_BN) * 2 <= num_sms)
    csk = plan_csk(a.M, a.N, a.K, num_sms, EPI == EPI_GEGLU).C >= 2;
  if (csk) {
    launch_csk<EPI>(ta, tb, a, *sk, num_sms, st);
    CK(cudaGetLastError());
    return;
  }
  int ksp = 1;
  const int rows = (a.M + GEMM_BM - 1) / GEMM_BM * GEMM_BM;
  if (sk && sk->ws && variant == 3) {
    ksp = pick_k_splits(a.M, a.N, a.K, num_sms, sk->ws_bytes);
    if (variant == 3 && ksp < 2 && (a.K + GEMM_BK - 1) / GEMM_BK >= 2 && 2 * (size_t)rows * a.N * 4 <= sk->ws_bytes)
      ksp = 2;
  }
  if (ksp > 1) {
    a.k_splits = ksp;
    a.split_rows = rows;
    const int tiles = (rows / GEMM_BM) * ((a.N + GEMM_BN - 1) / GEMM_BN) * ksp;
    const int grid = std::min(tiles, num_sms);
    const CUtensorMap tw = make_out_tmap(sk->ws, true, (uint64_t)ksp * rows, a.N, a.N);
    launch_k(gemm_bf16_sm100<GEMM_BN, EPI>, dim3(grid), dim3(GEMM1_THREADS), gemm_smem_bytes(GEMM_BN), st, ta, tb.full, tw, a);
    CK(cudaGetLastError());
    SplitKFinal f{sk->ws, ksp, rows, a.M, a.N, sk->out, sk->ldo, a.bias, a.act, a.out_f32, a.pos, a.inv_freq,
                  a.rope_cols, a.out_cols};
    const long work = (long)a.M * ((EPI == EPI_GEGLU ? a.out_cols : a.N) / 8);
    launch_k(splitk_finalize_kernel<EPI>, dim3((unsigned)((work + 255) / 256)), dim3(256), 0, st, f);
    CK(cudaGetLastError());
    if (extra_launches) ++*extra_launches;
    return;
  }
  // By shape: the two-CTA kernel for the RoPE, residual and plain stores once its 256 x 256 tiles
  // fill the SMs (measured at 16k tokens: Wqkv 1253 vs 1212, Wo2 1187 vs 1126, Wo 952 vs 905
  // TFLOP/s), the one-CTA kernel for GeGLU (1245 vs 1219) and for fewer tiles.
  const bool two = variant == 2 ||
                   (variant == 0 && EPI != EPI_GEGLU && !(t_gemm_off & GEMM_OFF_2CTA) &&
                    ((a.M + 255) / 256) * ((a.N + GEMM_BN - 1) / GEMM_BN) * 2 >= num_sms);
  if (two) {
    const int tiles = ((a.M + 255) / 256) * ((a.N + GEMM_BN - 1) / GEMM_BN);
    const int clusters = std::min(tiles, num_sms / 2);
    launch_k(gemm2_bf16_sm100<EPI>, dim3(2 * clusters), dim3(GEMM_THREADS), gemm2_smem_bytes(), st, ta, tb.half, tc, a);
  } else if (EPI != EPI_GEGLU && variant == 5) {
    if constexpr (EPI != EPI_GEGLU) {
      const int tiles = ((a.M + GEMM_BM - 1) / GEMM_BM) * ((a.N + 127) / 128);
      const int grid = std::min(tiles, num_sms);
      launch_k(gemm_bf16_sm100<128, EPI>, dim3(grid), dim3(GEMM1_THREADS), gemm_smem_bytes(128), st, ta, tb.half, tc, a);
    }
  } else {
    const int tiles = ((a.M + GEMM_BM - 1) / GEMM_BM) * ((a.N + GEMM_BN - 1) / GEMM_BN);
    const int grid = std::min(tiles, num_sms);
    launch_k(gemm_bf16_sm100<GEMM_BN, EPI>, dim3(grid), dim3(GEMM1_THREADS), gemm_smem_bytes(GEMM_BN), st, ta, tb.full, tc, a);
  }
  CK(cudaGetLastError());
}

template <int D, typename TIn>
void launch_ln(const TIn* in, const int* gather, int rows, const float* w, const float* b, float eps, bf16* out,
               cudaStream_t st, int num_sms) {
  if (rows <= 0) return;
  // 8 warps per block, one wave of resident blocks at most (register-limited), rows spread evenly
  // over the grid.
  auto resident = [](auto kernel) {
    int n = 0;
    CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, 256, 0));
    return std::max(n, 1);
  };
  static const int per_sm_b = resident(layernorm_kernel<D, true, TIn>),
                   per_sm_nb = resident(layernorm_kernel<D, false, TIn>);
  const int blocks = std::max(1, std::min((rows + 7) / 8, (b ? per_sm_b : per_sm_nb) * num_sms));
  if (b) launch_k(layernorm_kernel<D, true, TIn>, dim3(blocks), dim3(256), 0, st, in, gather, rows, w, b, eps, out);
  else launch_k(layernorm_kernel<D, false, TIn>, dim3(blocks), dim3(256), 0, st, in, gather, rows, w, b, eps, out);
  CK(cudaGetLastError());
}

__global__ void prep_tokens_kernel(const int* __restrict__ cu, int n, int T, int* __restrict__ pos,
                                   int* __restrict__ row) {
  pdl_trigger();
  pdl_wait();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  int lo = 0, hi = n - 1;  // largest r with cu[r] <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid - 1;
  }
  pos[t] = t - cu[lo];
  row[t] = lo;
}

// ---------------------------------------------------------------------------------------------
// the backend

struct DevBuf {
  void* p = nullptr;
  size_t bytes = 0;
  ~DevBuf() { if (p) cudaFree(p); }
  void ensure(size_t b) {
    if (b <= bytes) return;
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
    CK(cudaMalloc(&p, b));
    bytes = b;
  }
  template <class T> T* as() const { return static_cast<T*>(p); }
};

struct ProfRec {
  const char* name;
  double flops, bytes;
  size_t ev;
};
struct ProfStat {
  int64_t launches = 0;
  double ms = 0, flops = 0, bytes = 0;
};

struct EncLayer {
  bf16 *wqkv = nullptr, *wo = nullptr, *wi = nullptr, *wo2 = nullptr;
  float *attn_norm = nullptr, *mlp_norm = nullptr;
  bool local = false;
  WeightMap tm_wqkv, tm_wo, tm_wi, tm_wo2;
};

struct HeadLayer {
  bf16 *in_w = nullptr, *out_w = nullptr, *l1_w = nullptr, *l2_w = nullptr;
  float *in_b = nullptr, *out_b = nullptr, *l1_b = nullptr, *l2_b = nullptr;
  float *n1w = nullptr, *n1b = nullptr, *n2w = nullptr, *n2b = nullptr;
  WeightMap tm_in, tm_in_q, tm_in_kv, tm_out, tm_l1, tm_l2;
};

}  // namespace

struct s1c_backend {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  std::string name = "cuda(sm_100a,bf16)";
  std::string kernels =
      "gemm_tcgen05_tma(rope,geglu,residual,bias_act),attention_varlen_mma,embed_ln,layernorm,final_to_head,"
      "scorer_logits";
  std::string last_error;
  int64_t launches = 0;
  cudaStream_t own_stream = nullptr;

  // per-launch profiling (s1c_profile; the `ops` trace turns it on for its forwards)
  bool prof_on = false;
  bool prof_user = false;  // s1c_profile(on)
  // Tracing (`trace=1`, `layers=1`, `ops=1`, the reference's knobs of those names,
  // laya-mlx/src/lib.rs:75-80, :1555-1579, :1842-1850): per forward one stderr line with the
  // shape, the graph use, the host enqueue time and the device time (`trace`); the device time of
  // every encoder layer (`layers`); the summed device time of every kernel (`ops`). `layers` and
  // `ops` launch kernel by kernel (no graphs), like the reference's per-layer evaluation.
  bool trace = false, trace_layers = false, trace_ops = false;
  cudaEvent_t tr_ev[2] = {nullptr, nullptr};
  std::vector<cudaEvent_t> layer_ev;
  double tr_enqueue_us = 0;
  bool tr_pending = false;
  std::string tr_desc;
  std::vector<cudaEvent_t> ev_pool;
  size_t ev_used = 0;
  std::vector<ProfRec> prof_pending;
  std::map<std::string, ProfStat> prof_stats;

  // config
  int V = 0, d = 0, L = 0, H = 0, I = 0, Ipad = 0, F = 0, S = 0, n_head = 0, window = 64, max_pos = 0;
  float eps = 1e-5f;
  std::vector<uint8_t> local;

  // weights
  std::vector<void*> allocs;
  bf16* tok_emb = nullptr;
  float *emb_norm = nullptr, *final_norm = nullptr, *type_emb = nullptr;
  std::vector<EncLayer> layers;
  std::vector<HeadLayer> head;
  float *sc_nw = nullptr, *sc_nb = nullptr, *sc_b1 = nullptr, *sc_w3 = nullptr, *sc_b3 = nullptr;
  bf16* sc_w1 = nullptr;
  WeightMap tm_sc1;
  float* inv_freq[2] = {nullptr, nullptr};  // 0 global theta, 1 local theta
  float* rope_tab[2] = {nullptr, nullptr};  // [max_pos][64] cos | sin per theta

  // activations (capacity in rows, multiples of 128)
  int gemm_variant = 0;   // `gemm=auto|1cta|2cta|splitk|csk`
  bool pdl = true;        // `pdl=0|1`: programmatic dependent launch between the forward's kernels
  // Attention kernel per call: `attn=auto` (default) runs the tcgen05 kernel (attention_tc.cuh) on
  // the encoder and head layer 0 (global and sliding window) when its grid fills the SMs, and the
  // mma.sync kernel (attention.cuh) on the pruned head rows (1 + kmax queries per row, where its
  // 64-row tiles waste less) and on small batches; `attn=tc|mma` force one kernel everywhere.
  enum AttnMode { ATTN_AUTO, ATTN_TC, ATTN_MMA } attn_mode = ATTN_AUTO;
  // Load-time kernel self-check (`check=0|1`, `check_fail=`; selfcheck()).
  bool check = true;
  bool checked = false;
  int gemm_off = 0;          // GEMM_OFF_* bits set by the check
  std::string check_fail;    // kernels whose check gets a planted wrong expected value ('+'-separated)
  std::string check_report;  // kernels the check turned off ('+'-separated)
  int cap_T = 0, cap_R = 0;
  DevBuf h, x, qkv, att, act;          // [cap_T, ...]; h: the encoder's residual stream, f16
  DevBuf h2;                           // head residual stream [cap_T, d] fp32
  DevBuf xs, qs, atts, hs, fs, xm, sh; // scorer rows [cap_R, ...]
  CUtensorMap tm_x, tm_att, tm_act_i, tm_act_f, tm_xs, tm_atts, tm_fs, tm_xm;
  // tcgen05 attention maps: Q boxes of ATTC_BQ rows, K/V boxes of ATTC_BK rows
  CUtensorMap tm_qkv_att, tm_qkv_kv, tm_kv_att, tm_qs_att;
  // GEMM output maps (32-row boxes): bf16 qkv as [T,3d] and [T,2d], act as [T,I] and [T,F];
  // residual streams h (f16) and h2 (fp32); scorer-row buffers.
  CUtensorMap to_qkv3, to_kv2, to_act_i, to_act_f, to_h, to_h2, to_qs, to_hs, to_fs, to_sh;

  // Metadata: a forward's small host arrays (and the token ids when they come from the host) are
  // staged in a pinned host slot and copied in one transfer into `meta_dev`, a device arena whose
  // address only changes when it grows. Host slots form a ring; a slot is reused once its copy has
  // completed (event), so forwards can be enqueued back to back without a host sync.
  struct MetaSlot {
    void* host = nullptr;
    size_t host_bytes = 0;
    cudaEvent_t copied = nullptr;
    bool pending = false;
  };
  static constexpr int META_SLOTS = 4;
  MetaSlot meta[META_SLOTS];
  int meta_next = 0;
  DevBuf meta_dev;
  DevBuf tok;         // pos [cap_T] + token_row [cap_T] int32
  int* d_status = nullptr;
  int* h_status = nullptr;
  DevBuf out_stage;   // logits and pooled of the current forward (copied out by the entry points)
  DevBuf splitk_ws;   // split-K fp32 partial sums, one slice per split
  float* h_out = nullptr;  // pinned host outputs
  size_t h_out_bytes = 0;

  // CUDA graphs of whole forwards, keyed by the shape that fixes every launch configuration and
  // every buffer offset: (tokens, rows, kmax, attention items, pruned-row items). Kernel arguments
  // point only at the backend's own buffers, so a graph replays any batch of that shape. A bucket
  // shape is captured the first time it is seen, any other shape the second time; at most
  // MAX_GRAPHS graphs are kept (the least recently replayed one goes first) and at most MAX_SEEN
  // shapes are remembered; all graphs are dropped when a buffer moves.
  bool use_graphs = true;
  struct Graph {
    cudaGraphExec_t exec = nullptr;
    int64_t launches = 0;
    uint64_t last_used = 0;
  };
  static constexpr size_t MAX_GRAPHS = 128, MAX_SEEN = 4096;
  std::map<std::vector<int>, Graph> graphs;
  std::map<std::vector<int>, int> seen;
  uint64_t graph_clock = 0;
  void drop_graphs() {
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second.exec);
    graphs.clear();
    seen.clear();
  }
  void evict_graphs(size_t keep) {
    if (graphs.size() > keep && stream) cudaStreamSynchronize(stream);  // no evicted graph still runs
    while (graphs.size() > keep) {
      auto lru = graphs.begin();
      for (auto i = graphs.begin(); i != graphs.end(); ++i)
        if (i->second.last_used < lru->second.last_used) lru = i;
      cudaGraphExecDestroy(lru->second.exec);
      graphs.erase(lru);
    }
  }
  // Packed-token buckets (`buckets=`, ascending; empty: exact shapes) and the row counts that
  // s1c_warmup runs at every bucket (`warm=`).
  std::vector<int> buckets = {128, 256, 384, 512, 640, 768, 896, 1024, 1280, 1536, 1792, 2048};
  std::vector<int> warm_rows = {1};

  ~s1c_backend() {
    if (stream) cudaStreamSynchronize(stream);
    if (own_stream) cudaStreamSynchronize(own_stream);
    for (cudaEvent_t e : ev_pool) cudaEventDestroy(e);
    for (cudaEvent_t e : layer_ev) cudaEventDestroy(e);
    for (cudaEvent_t e : tr_ev)
      if (e) cudaEventDestroy(e);
    for (void* p : allocs) cudaFree(p);
    if (d_status) cudaFree(d_status);
    if (h_status) cudaFreeHost(h_status);
    for (auto& sl : meta) {
      if (sl.host) cudaFreeHost(sl.host);
      if (sl.copied) cudaEventDestroy(sl.copied);
    }
    drop_graphs();
    if (h_out) cudaFreeHost(h_out);
    if (own_stream) cudaStreamDestroy(own_stream);
  }

  template <class T>
  T* dalloc(size_t n) {
    void* p = nullptr;
    CK(cudaMalloc(&p, std::max<size_t>(n, 1) * sizeof(T)));
    allocs.push_back(p);
    return static_cast<T*>(p);
  }
};

namespace {

struct TensorTable {
  std::map<std::string, const s1c_tensor*> by_name;
  const s1c_tensor& get(const std::string& n, std::vector<int64_t> shape) const {
    auto it = by_name.find(n);
    if (it == by_name.end()) throw S1cError(S1C_ERR_WEIGHTS, n + ": missing tensor");
    const s1c_tensor& t = *it->second;
    bool ok = (int)shape.size() == t.ndim;
    for (size_t i = 0; ok && i < shape.size(); ++i) ok = shape[i] == t.shape[i];
    if (!ok) {
      std::string want, got;
      for (auto s : shape) want += std::to_string(s) + ",";
      for (int i = 0; i < t.ndim; ++i) got += std::to_string(t.shape[i]) + ",";
      throw S1cError(S1C_ERR_WEIGHTS, n + ": shape [" + got + "] where [" + want + "] is needed");
    }
    if (!t.data) throw S1cError(S1C_ERR_WEIGHTS, n + ": null data");
    return t;
  }
  bool has(const std::string& n) const { return by_name.count(n) != 0; }
};

// Matrix [rows, cols] -> bf16 on the device, rows padded with zeros to a multiple of 256 so
// that every TMA box lies inside the tensor.
bf16* upload_matrix(s1c_backend& B, const s1c_tensor& t, int64_t rows, int64_t cols, const int64_t* row_map = nullptr,
                    int64_t out_rows = -1) {
  if (out_rows < 0) out_rows = rows;
  const int64_t padded = (out_rows + 255) / 256 * 256;
  std::vector<uint16_t> hbuf((size_t)padded * cols, 0);
  for (int64_t r = 0; r < out_rows; ++r) {
    const int64_t src = row_map ? row_map[r] : r;
    if (src < 0) continue;
    for (int64_t c = 0; c < cols; ++c) hbuf[(size_t)r * cols + c] = f32_to_bf16_bits(elem_f32(t, (size_t)src * cols + c));
  }
  bf16* d = B.dalloc<bf16>(hbuf.size());
  CK(cudaMemcpy(d, hbuf.data(), hbuf.size() * 2, cudaMemcpyHostToDevice));
  return d;
}
float* upload_vector(s1c_backend& B, const s1c_tensor& t, int64_t n, int64_t offset = 0) {
  std::vector<float> hbuf((size_t)n);
  for (int64_t i = 0; i < n; ++i) hbuf[i] = elem_f32(t, (size_t)(offset + i));
  float* d = B.dalloc<float>(n);
  CK(cudaMemcpy(d, hbuf.data(), n * 4, cudaMemcpyHostToDevice));
  return d;
}

// RoPE inverse frequencies exp2(-(i / 32) * log2(theta)), i = 0..31, in fp32 as the reference
// kernel computes them (split_rope.metal:46-76). The GEMM epilogue forms the angle p * inv_freq
// in fp32 and takes its cos/sin. Returns a fresh device allocation of 32 floats.
float* make_inv_freq_raw(float theta) {
  float t[32];
  const float lbase = std::log2(theta);
  for (int i = 0; i < 32; ++i) t[i] = std::exp2(-((float)i / 32.0f) * lbase);
  float* d = nullptr;
  CK(cudaMalloc(&d, sizeof t));
  cudaError_t e = cudaMemcpy(d, t, sizeof t, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(d);
    throw S1cError(S1C_ERR_CUDA, std::string("inv_freq upload: ") + cudaGetErrorString(e));
  }
  return d;
}
float* make_inv_freq(s1c_backend& B, float theta) {
  float* d = make_inv_freq_raw(theta);
  B.allocs.push_back(d);
  return d;
}
// The cos | sin table of rope_table_kernel for positions [0, P) (a fresh device allocation).
float* make_rope_table_raw(const float* d_inv_freq, int P) {
  float* d = nullptr;
  CK(cudaMalloc(&d, (size_t)P * 64 * sizeof(float)));
  rope_table_kernel<<<(P * 32 + 255) / 256, 256>>>(d, P, d_inv_freq);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(d);
    throw S1cError(S1C_ERR_CUDA, std::string("RoPE table: ") + cudaGetErrorString(e));
  }
  return d;
}

void ensure_capacity(s1c_backend& B, int T, int R) {
  const int want_T = (std::max(T, 128) + 127) / 128 * 128;
  const int want_R = (std::max(R, 128) + 127) / 128 * 128;
  if (want_T > B.cap_T) {
    const int cap = std::max(want_T, B.cap_T + B.cap_T / 2 / 128 * 128);
    CK(cudaStreamSynchronize(B.stream));
    B.drop_graphs();
    const size_t wide = (size_t)std::max(B.Ipad / 2, B.F);
    B.h.ensure((size_t)cap * B.d * 2);
    B.h2.ensure((size_t)cap * B.d * 4);
    B.x.ensure((size_t)cap * B.d * 2);
    B.qkv.ensure((size_t)cap * 3 * B.d * 2);
    B.att.ensure((size_t)cap * B.d * 2);
    B.act.ensure((size_t)cap * wide * 2);
    B.tok.ensure((size_t)cap * 2 * 4);
    B.cap_T = cap;
    // Rows past a forward's token count are read (and discarded) by full tiles: keep them finite.
    CK(cudaMemsetAsync(B.qkv.p, 0, B.qkv.bytes, B.stream));
    CK(cudaMemsetAsync(B.x.p, 0, B.x.bytes, B.stream));
    CK(cudaMemsetAsync(B.att.p, 0, B.att.bytes, B.stream));
    CK(cudaMemsetAsync(B.act.p, 0, B.act.bytes, B.stream));
    B.tm_x = make_tmap(B.x.p, cap, B.d, B.d, GEMM_BM);
    B.tm_qkv_att = make_tmap(B.qkv.p, cap, 3 * B.d, 3 * B.d, ATTC_BQ);
    B.tm_qkv_kv = make_tmap(B.qkv.p, cap, 3 * B.d, 3 * B.d, ATTC_BK);
    B.tm_kv_att = make_tmap(B.qkv.p, cap, 2 * B.d, 2 * B.d, ATTC_BK);
    B.to_qkv3 = make_out_tmap(B.qkv.p, false, cap, 3 * B.d, 3 * B.d);
    B.to_kv2 = make_out_tmap(B.qkv.p, false, cap, 2 * B.d, 2 * B.d);
    B.to_act_i = make_out_tmap(B.act.p, false, cap, B.I, B.I);
    B.to_act_f = make_out_tmap(B.act.p, false, cap, B.F, B.F);
    B.to_h = make_out_tmap_f16(B.h.p, cap, B.d, B.d);
    B.to_h2 = make_out_tmap(B.h2.p, true, cap, B.d, B.d);
    B.tm_att = make_tmap(B.att.p, cap, B.d, B.d, GEMM_BM);
    B.tm_act_i = make_tmap(B.act.p, cap, B.I, B.I, GEMM_BM);
    B.tm_act_f = make_tmap(B.act.p, cap, B.F, B.F, GEMM_BM);
  }
  if (want_R > B.cap_R) {
    const int cap = std::max(want_R, B.cap_R + B.cap_R / 2 / 128 * 128);
    CK(cudaStreamSynchronize(B.stream));
    B.drop_graphs();
    B.xs.ensure((size_t)cap * B.d * 2);
    B.qs.ensure((size_t)cap * B.d * 2);
    B.atts.ensure((size_t)cap * B.d * 2);
    B.hs.ensure((size_t)cap * B.d * 4);
    B.fs.ensure((size_t)cap * B.F * 2);
    B.xm.ensure((size_t)cap * B.d * 2);
    B.sh.ensure((size_t)cap * B.S * 4);
    B.cap_R = cap;
    CK(cudaMemsetAsync(B.qs.p, 0, B.qs.bytes, B.stream));
    CK(cudaMemsetAsync(B.xs.p, 0, B.xs.bytes, B.stream));
    B.tm_xs = make_tmap(B.xs.p, cap, B.d, B.d, GEMM_BM);
    B.tm_qs_att = make_tmap(B.qs.p, cap, B.d, B.d, ATTC_BQ);
    B.to_qs = make_out_tmap(B.qs.p, false, cap, B.d, B.d);
    B.to_hs = make_out_tmap(B.hs.p, true, cap, B.d, B.d);
    B.to_fs = make_out_tmap(B.fs.p, false, cap, B.F, B.F);
    B.to_sh = make_out_tmap(B.sh.p, true, cap, B.S, B.S);
    B.tm_atts = make_tmap(B.atts.p, cap, B.d, B.d, GEMM_BM);
    B.tm_fs = make_tmap(B.fs.p, cap, B.F, B.F, GEMM_BM);
    B.tm_xm = make_tmap(B.xm.p, cap, B.d, B.d, GEMM_BM);
  }
}

void build(s1c_backend& B, const s1c_model_desc& D, const s1c_tensor* tensors, int n_tensors) {
  B.V = D.vocab_size;
  B.d = D.hidden_size;
  B.L = D.num_layers;
  B.H = D.num_heads;
  B.I = D.intermediate_size;
  B.eps = D.norm_eps;
  B.window = D.local_attention / 2;
  B.max_pos = D.max_position > 0 ? D.max_position : 8192;
  B.n_head = D.head_layers;
  if (B.d != 256 && B.d != 768 && B.d != 1024)
    throw S1cError(S1C_ERR_CONFIG, "hidden_size " + std::to_string(B.d) + " is not one of 256, 768, 1024");
  if (B.H <= 0 || B.d % B.H || B.d / B.H != 64)
    throw S1cError(S1C_ERR_CONFIG, "the attention kernels need head_dim 64 (hidden_size / num_heads)");
  if (B.I <= 0 || B.I % 32) throw S1cError(S1C_ERR_CONFIG, "intermediate_size must be a positive multiple of 32");
  if (D.local_attention < 2) throw S1cError(S1C_ERR_CONFIG, "local_attention must be at least 2");
  if (B.n_head < 1) throw S1cError(S1C_ERR_CONFIG, "head_layers must be at least 1");
  if (B.L < 1 || !D.layer_is_local) throw S1cError(S1C_ERR_CONFIG, "num_layers / layer_is_local");
  B.local.assign(D.layer_is_local, D.layer_is_local + B.L);
  B.Ipad = (B.I + 127) / 128 * 256;

  TensorTable tt;
  for (int i = 0; i < n_tensors; ++i) {
    if (!tensors[i].name) throw S1cError(S1C_ERR_ARG, "tensor with a null name");
    tt.by_name[tensors[i].name] = &tensors[i];
  }
  const int64_t d = B.d, I = B.I;
  B.tok_emb = upload_matrix(B, tt.get("encoder.embeddings.tok_embeddings.weight", {B.V, d}), B.V, d);
  B.emb_norm = upload_vector(B, tt.get("encoder.embeddings.norm.weight", {d}), d);
  B.final_norm = upload_vector(B, tt.get("encoder.final_norm.weight", {d}), d);
  B.type_emb = upload_vector(B, tt.get("type_emb.weight", {3, d}), 3 * d);

  // Wi rows interleaved per 128: tile t holds input rows [128t, 128t+128) then gate rows
  // [I + 128t, ...), zero past the end, so one 256-wide output tile carries both GeGLU halves.
  std::vector<int64_t> wi_map((size_t)B.Ipad);
  for (int64_t r = 0; r < B.Ipad; ++r) {
    const int64_t t = r / 256, j = r % 256;
    const int64_t c = 128 * t + (j < 128 ? j : j - 128);  // output column this row feeds
    wi_map[r] = c < I ? (j < 128 ? c : I + c) : -1;
  }
  B.layers.resize(B.L);
  for (int i = 0; i < B.L; ++i) {
    const std::string p = "encoder.layers." + std::to_string(i);
    EncLayer& l = B.layers[i];
    l.local = B.local[i] != 0;
    if (i > 0) l.attn_norm = upload_vector(B, tt.get(p + ".attn_norm.weight", {d}), d);
    l.mlp_norm = upload_vector(B, tt.get(p + ".mlp_norm.weight", {d}), d);
    l.wqkv = upload_matrix(B, tt.get(p + ".attn.Wqkv.weight", {3 * d, d}), 3 * d, d);
    l.wo = upload_matrix(B, tt.get(p + ".attn.Wo.weight", {d, d}), d, d);
    l.wi = upload_matrix(B, tt.get(p + ".mlp.Wi.weight", {2 * I, d}), 2 * I, d, wi_map.data(), B.Ipad);
    l.wo2 = upload_matrix(B, tt.get(p + ".mlp.Wo.weight", {d, I}), d, I);
    l.tm_wqkv = make_wmap(l.wqkv, 3 * d, d, d);
    l.tm_wo = make_wmap(l.wo, (d + 255) / 256 * 256, d, d);
    l.tm_wi = make_wmap(l.wi, B.Ipad, d, d);
    l.tm_wo2 = make_wmap(l.wo2, (d + 255) / 256 * 256, I, I);
  }
  const std::string h0 = "head.layers.0.linear1.weight";
  if (!tt.has(h0)) throw S1cError(S1C_ERR_WEIGHTS, h0 + ": missing tensor");
  B.F = (int)tt.by_name[h0]->shape[0];
  if (B.F <= 0 || B.F % 256) throw S1cError(S1C_ERR_CONFIG, "head FFN width must be a multiple of 256");
  B.head.resize(B.n_head);
  for (int j = 0; j < B.n_head; ++j) {
    const std::string p = "head.layers." + std::to_string(j);
    HeadLayer& hl = B.head[j];
    const s1c_tensor& inw = tt.get(p + ".self_attn.in_proj_weight", {3 * d, d});
    hl.in_w = upload_matrix(B, inw, 3 * d, d);
    hl.in_b = upload_vector(B, tt.get(p + ".self_attn.in_proj_bias", {3 * d}), 3 * d);
    hl.out_w = upload_matrix(B, tt.get(p + ".self_attn.out_proj.weight", {d, d}), d, d);
    hl.out_b = upload_vector(B, tt.get(p + ".self_attn.out_proj.bias", {d}), d);
    hl.l1_w = upload_matrix(B, tt.get(p + ".linear1.weight", {B.F, d}), B.F, d);
    hl.l1_b = upload_vector(B, tt.get(p + ".linear1.bias", {B.F}), B.F);
    hl.l2_w = upload_matrix(B, tt.get(p + ".linear2.weight", {d, B.F}), d, B.F);
    hl.l2_b = upload_vector(B, tt.get(p + ".linear2.bias", {d}), d);
    hl.n1w = upload_vector(B, tt.get(p + ".norm1.weight", {d}), d);
    hl.n1b = upload_vector(B, tt.get(p + ".norm1.bias", {d}), d);
    hl.n2w = upload_vector(B, tt.get(p + ".norm2.weight", {d}), d);
    hl.n2b = upload_vector(B, tt.get(p + ".norm2.bias", {d}), d);
    hl.tm_in = make_wmap(hl.in_w, 3 * d, d, d);
    hl.tm_in_q = make_wmap(hl.in_w, d, d, d);
    hl.tm_in_kv = make_wmap(hl.in_w + d * d, 2 * d, d, d);
    hl.tm_out = make_wmap(hl.out_w, (d + 255) / 256 * 256, d, d);
    hl.tm_l1 = make_wmap(hl.l1_w, B.F, d, d);
    hl.tm_l2 = make_wmap(hl.l2_w, (d + 255) / 256 * 256, B.F, B.F);
  }
  if (!tt.has("scorer.1.weight")) throw S1cError(S1C_ERR_WEIGHTS, "scorer.1.weight: missing tensor");
  B.S = (int)tt.by_name["scorer.1.weight"]->shape[0];
  if (B.S <= 0 || B.S % 32) throw S1cError(S1C_ERR_CONFIG, "scorer hidden width must be a multiple of 32");
  B.sc_nw = upload_vector(B, tt.get("scorer.0.weight", {d}), d);
  B.sc_nb = upload_vector(B, tt.get("scorer.0.bias", {d}), d);
  B.sc_w1 = upload_matrix(B, tt.get("scorer.1.weight", {B.S, d}), B.S, d);
  B.sc_b1 = upload_vector(B, tt.get("scorer.1.bias", {B.S}), B.S);
  B.sc_w3 = upload_vector(B, tt.get("scorer.3.weight", {1, B.S}), B.S);
  B.sc_b3 = upload_vector(B, tt.get("scorer.3.bias", {1}), 1);
  B.tm_sc1 = make_wmap(B.sc_w1, (B.S + 255) / 256 * 256, d, d);

  B.inv_freq[0] = make_inv_freq(B, D.global_rope_theta);
  B.inv_freq[1] = make_inv_freq(B, D.local_rope_theta);
  for (int t = 0; t < 2; ++t) {
    B.rope_tab[t] = make_rope_table_raw(B.inv_freq[t], std::max(B.max_pos, 1));
    B.allocs.push_back(B.rope_tab[t]);
  }
  CK(cudaMalloc(&B.d_status, sizeof(int)));
  CK(cudaMemset(B.d_status, 0, sizeof(int)));
  B.splitk_ws.ensure((size_t)32 << 20);
  CK(cudaMallocHost(&B.h_status, sizeof(int)));
  ensure_capacity(B, std::max(D.max_tokens, 128), 128);
}

// ---------------------------------------------------------------------------------------------
// forward

struct HostMeta {
  int n = 0, kmax = 0, T = 0, R = 0, M = 0;  // rows, kmax, tokens, scorer rows n(1+kmax), markers n*kmax
  int hidden_rows = 0;                        // tokens whose final hidden state is written out
  double pairs_global = 0, pairs_local = 0, pairs_rows = 0;  // attended (query, key) pairs per head-set
  std::vector<int> cu, srows, mrows, prows, mcount;
  // attention key range of every row, (begin, end) token pairs: the row's own tokens, or with
  // `real_len` its real tokens only (padding tokens attend them but are never keys); a work
  // item's x field is 2 * row, so the kernels read its range at acu[x], acu[x + 1]
  std::vector<int> acu;
  std::vector<uint32_t> qtype;
  // attention work lists for the two query-tile heights: full rows (encoder, head layer 0) and
  // the pruned head rows, tiles of 64 (mma.sync kernel) and 128 (tcgen05 kernel)
  std::vector<int4> items_full, items_rows, items_full_tc, items_rows_tc;
};

void validate_varlen(const s1c_backend& B, const s1c_varlen& in) {
  if (in.n < 0 || in.kmax < 0) throw S1cError(S1C_ERR_ARG, "n and kmax must be non-negative");
  if (in.n == 0) return;
  if (!in.cu_seqlens || !in.marker_count || !in.qtype || (in.kmax > 0 && !in.marker_pos))
    throw S1cError(S1C_ERR_ARG, "null batch array");
  if (in.cu_seqlens[0] != 0) throw S1cError(S1C_ERR_ARG, "cu_seqlens[0] must be 0");
  for (int r = 0; r < in.n; ++r) {
    const int len = in.cu_seqlens[r + 1] - in.cu_seqlens[r];
    if (len < 1) throw S1cError(S1C_ERR_ARG, "row " + std::to_string(r) + ": every row needs at least one token");
    if (len > B.max_pos)
      throw S1cError(S1C_ERR_ARG, "row " + std::to_string(r) + ": length " + std::to_string(len) +
                                      " exceeds max_position " + std::to_string(B.max_pos));
    if (in.qtype[r] > 2) throw S1cError(S1C_ERR_ARG, "row " + std::to_string(r) + ": qtype must be 0, 1 or 2");
    const int mc = in.marker_count[r];
    if (mc < 0 || mc > in.kmax) throw S1cError(S1C_ERR_ARG, "row " + std::to_string(r) + ": marker_count outside 0..kmax");
    for (int k = 0; k < in.kmax; ++k)
      if ((int64_t)in.marker_pos[(size_t)r * in.kmax + k] >= len)
        throw S1cError(S1C_ERR_ARG, "row " + std::to_string(r) + ": marker position past the row");
  }
}

// Attention work items with the longest sequences first. The attention grids launch item-major
// (all heads of one item in consecutive blocks), so the tiles with the most keys start in the
// first wave and the short ones fill the tail (longest-processing-time order).
static void longest_first(std::vector<int4>& items, const int* acu) {
  std::stable_sort(items.begin(), items.end(), [acu](const int4& a, const int4& b) {
    return acu[a.x + 1] - acu[a.x] > acu[b.x + 1] - acu[b.x];
  });
}

// Work items (query tiles) of the first `n_items` rows only; with `pad` set, every list is then
// filled with empty items (q_count 0, which the attention kernels skip) up to the fixed lengths of
// a bucket shape, so that the grids of a bucket's captured graph fit any batch of the bucket.
struct ItemPad {
  bool on = false;
  int full = 0, rows = 0, full_tc = 0, rows_tc = 0;
};
HostMeta make_meta(const s1c_varlen& in, int window, int n_items, const ItemPad& pad, const int* real_len = nullptr) {
  HostMeta m;
  m.n = in.n;
  m.kmax = in.kmax;
  m.T = in.n ? in.cu_seqlens[in.n] : 0;
  m.R = in.n * (1 + in.kmax);
  m.M = in.n * in.kmax;
  m.cu.assign(in.cu_seqlens, in.cu_seqlens + in.n + 1);
  m.qtype.assign(in.qtype, in.qtype + in.n);
  m.mcount.assign(in.marker_count, in.marker_count + in.n);
  m.srows.resize(m.R);
  m.prows.resize(in.n);
  m.mrows.resize(m.M);
  m.acu.resize(2 * (size_t)in.n);
  for (int r = 0; r < in.n; ++r) {
    const int base = m.cu[r];
    m.acu[2 * r] = base;
    m.acu[2 * r + 1] = real_len ? base + real_len[r] : m.cu[r + 1];
    m.srows[r * (1 + in.kmax)] = base;
    m.prows[r] = r * (1 + in.kmax);
    for (int k = 0; k < in.kmax; ++k) {
      m.srows[r * (1 + in.kmax) + 1 + k] = base + (int)in.marker_pos[(size_t)r * in.kmax + k];
      m.mrows[r * in.kmax + k] = r * (1 + in.kmax) + 1 + k;
    }
    if (r >= n_items) continue;
    const int len = m.cu[r + 1] - base;
    m.pairs_global += (double)len * len;
    m.pairs_rows += (double)(1 + in.kmax) * len;
    for (int i = 0; i < len; ++i) m.pairs_local += std::min(i, window) + std::min(len - 1 - i, window) + 1;
    const int rows = 1 + in.kmax;
    for (int q = 0; q < len; q += ATT_BQ)
      m.items_full.push_back(make_int4(2 * r, base + q, std::min(ATT_BQ, len - q), 0));
    for (int q = 0; q < rows; q += ATT_BQ)
      m.items_rows.push_back(make_int4(2 * r, r * rows + q, std::min(ATT_BQ, rows - q), 1));
    for (int q = 0; q < len; q += ATTC_BQ)
      m.items_full_tc.push_back(make_int4(2 * r, base + q, std::min(ATTC_BQ, len - q), 0));
    for (int q = 0; q < rows; q += ATTC_BQ)
      m.items_rows_tc.push_back(make_int4(2 * r, r * rows + q, std::min(ATTC_BQ, rows - q), 1));
  }
  longest_first(m.items_full, m.acu.data());
  longest_first(m.items_rows, m.acu.data());
  longest_first(m.items_full_tc, m.acu.data());
  longest_first(m.items_rows_tc, m.acu.data());
  if (pad.on) {
    auto fill = [](std::vector<int4>& v, int count, int mode) {
      if ((int)v.size() > count) throw S1cError(S1C_ERR_ARG, "internal: bucket work list overflow");
      v.resize(count, make_int4(0, 0, 0, mode));
    };
    fill(m.items_full, pad.full, 0);
    fill(m.items_rows, pad.rows, 1);
    fill(m.items_full_tc, pad.full_tc, 0);
    fill(m.items_rows_tc, pad.rows_tc, 1);
  }
  return m;
}

struct DevMeta {
  const uint32_t* ids;
  const int* cu;
  const int* acu;
  const int* srows;
  const int* mrows;
  const int* prows;
  const int* mcount;
  const uint32_t* qtype;
  const int4* items_full;
  const int4* items_rows;
  const int4* items_full_tc;
  const int4* items_rows_tc;
};

// Stage the metadata (and optionally the ids) in pinned memory and copy it in one transfer.
DevMeta upload_meta(s1c_backend& B, const HostMeta& m, const uint32_t* host_ids) {
  struct Part {
    const void* src;
    size_t bytes;
  };
  // The ids region is always reserved (ids that are already on the device are copied into it).
  std::vector<Part> parts = {
      {host_ids, (size_t)m.T * 4},
      {m.cu.data(), m.cu.size() * 4},
      {m.srows.data(), m.srows.size() * 4},
      {m.mrows.data(), m.mrows.size() * 4},
      {m.prows.data(), m.prows.size() * 4},
      {m.mcount.data(), m.mcount.size() * 4},
      {m.qtype.data(), m.qtype.size() * 4},
      {m.items_full.data(), m.items_full.size() * 16},
      {m.items_rows.data(), m.items_rows.size() * 16},
      {m.items_full_tc.data(), m.items_full_tc.size() * 16},
      {m.items_rows_tc.data(), m.items_rows_tc.size() * 16},
      {m.acu.data(), m.acu.size() * 4},
  };
  std::vector<size_t> off(parts.size());
  size_t total = 0;
  for (size_t i = 0; i < parts.size(); ++i) {
    off[i] = total;
    total += (parts[i].bytes + 255) / 256 * 256;
  }
  total = std::max<size_t>(total, 256);
  s1c_backend::MetaSlot& sl = B.meta[B.meta_next];
  B.meta_next = (B.meta_next + 1) % s1c_backend::META_SLOTS;
  if (!sl.copied) CK(cudaEventCreateWithFlags(&sl.copied, cudaEventDisableTiming));
  if (sl.pending) CK(cudaEventSynchronize(sl.copied));  // the slot's previous copy has left the host buffer
  sl.pending = false;
  if (total > sl.host_bytes) {
    if (sl.host) cudaFreeHost(sl.host);
    sl.host = nullptr;
    sl.host_bytes = 0;
    CK(cudaMallocHost(&sl.host, total * 2));
    sl.host_bytes = total * 2;
  }
  if (total > B.meta_dev.bytes) {
    CK(cudaStreamSynchronize(B.stream));  // kernels of earlier forwards may still read the arena
    B.drop_graphs();
    B.meta_dev.ensure(total * 2);
  }
  // Only the metadata proper is copied when the ids come from the device.
  const size_t skip = host_ids ? 0 : off[1];
  char* hs = static_cast<char*>(sl.host);
  for (size_t i = 0; i < parts.size(); ++i)
    if (parts[i].bytes && parts[i].src) std::memcpy(hs + off[i], parts[i].src, parts[i].bytes);
  CK(cudaMemcpyAsync(B.meta_dev.as<char>() + skip, hs + skip, total - skip, cudaMemcpyHostToDevice, B.stream));
  CK(cudaEventRecord(sl.copied, B.stream));
  sl.pending = true;
  char* dv = B.meta_dev.as<char>();
  DevMeta dm;
  dm.ids = reinterpret_cast<const uint32_t*>(dv + off[0]);
  dm.cu = reinterpret_cast<const int*>(dv + off[1]);
  dm.srows = reinterpret_cast<const int*>(dv + off[2]);
  dm.mrows = reinterpret_cast<const int*>(dv + off[3]);
  dm.prows = reinterpret_cast<const int*>(dv + off[4]);
  dm.mcount = reinterpret_cast<const int*>(dv + off[5]);
  dm.qtype = reinterpret_cast<const uint32_t*>(dv + off[6]);
  dm.items_full = reinterpret_cast<const int4*>(dv + off[7]);
  dm.items_rows = reinterpret_cast<const int4*>(dv + off[8]);
  dm.items_full_tc = reinterpret_cast<const int4*>(dv + off[9]);
  dm.items_rows_tc = reinterpret_cast<const int4*>(dv + off[10]);
  dm.acu = reinterpret_cast<const int*>(dv + off[11]);
  return dm;
}

// Per-launch CUDA-event timing (s1c_profile): every launch of a forward is bracketed by two
// events on the forward's stream and attributed to a named kernel with its algorithmic FLOPs
// and bytes; the totals are read back after the forward's final synchronisation.
void prof_collect(s1c_backend& B) {
  for (const auto& r : B.prof_pending) {
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, B.ev_pool[r.ev], B.ev_pool[r.ev + 1]));
    ProfStat& st = B.prof_stats[r.name];
    st.launches += 1;
    st.ms += ms;
    st.flops += r.flops;
    st.bytes += r.bytes;
  }
  B.prof_pending.clear();
  B.ev_used = 0;
}

template <class F>
void launch(s1c_backend& B, int64_t& nl, const char* name, double flops, double bytes, F&& f) {
  size_t ev = 0;
  if (B.prof_on) {
    if (B.ev_used + 2 > B.ev_pool.size()) {
      for (int i = 0; i < 64; ++i) {
        cudaEvent_t e;
        CK(cudaEventCreate(&e));
        B.ev_pool.push_back(e);
      }
    }
    ev = B.ev_used;
    B.ev_used += 2;
    CK(cudaEventRecord(B.ev_pool[ev], B.stream));
  }
  f();
  CK(cudaGetLastError());
  if (B.prof_on) {
    CK(cudaEventRecord(B.ev_pool[ev + 1], B.stream));
    B.prof_pending.push_back(ProfRec{name, flops, bytes, ev});
  }
  ++nl;
}

template <int D>
void run_forward(s1c_backend& B, const HostMeta& m, const DevMeta& dm, const uint32_t* d_ids, float* d_logits,
                 float* d_pooled, float* d_hidden) {
  cudaStream_t st = B.stream;
  const int T = m.T, d = B.d, nsm = B.num_sms;
  const double Td = (double)T * d;
  int64_t nl = 0;
  int* pos = B.tok.as<int>();
  int* trow = pos + B.cap_T;
  __half* h = B.h.as<__half>();
  float* h2 = B.h2.as<float>();
  bf16* x = B.x.as<bf16>();
  bf16* qkv = B.qkv.as<bf16>();
  bf16* att = B.att.as<bf16>();
  bf16* act = B.act.as<bf16>();
  const float scale_log2 = (1.0f / 8.0f) * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)

  launch(B, nl, "prep_tokens", 0, 8.0 * T, [&] {
    launch_k(prep_tokens_kernel, dim3((T + 255) / 256), dim3(256), 0, st, dm.cu, m.n, T, pos, trow);
  });
  launch(B, nl, "embed_ln", 0, 6.0 * Td, [&] {
    launch_k(embed_ln_kernel<D>, dim3((T + 7) / 8), dim3(256), 0, st, d_ids, T, B.tok_emb, B.V, B.emb_norm, B.eps, h, x, B.d_status);
  });

  // Attention over the items' query tiles: the tcgen05 kernel reads Q/K/V through TMA maps
  // (tq with q at column q_col0, tkv with k at k_col0 and v at v_col0); the mma.sync kernel
  // through the raw pointers and row pitches.
  // `rows`: the pruned head rows (work lists items_rows*), else full rows (items_full*).
  auto attn = [&](const char* name, const CUtensorMap& tq, const CUtensorMap& tkv, int q_col0, int k_col0,
                  int v_col0, const bf16* q, const bf16* k, const bf16* v, bf16* o, int qs, int ks, int vs, int os,
                  bool rows, int window, double pairs) {
    // auto: the tcgen05 kernel when its work (query tiles of 128 x heads, ATTC_HEADS per SM at least)
    // fills the SMs, or when the batch has at least 256 tokens in rows of 128 on average (long
    // single requests: one row of 256 / 512 / 1000 / 2000 tokens measured 1 / 2 / 10 / 14 % faster
    // per forward); below that (short requests) the mma.sync kernel's 64-row, one-head blocks
    // spread the work wider (one row of 128 tokens: 1.26 against 1.33 ms). The rule reads only
    // the batch's shape (tokens, rows with dummy rows, work-list lengths), so a bucket's graph
    // always holds the same kernel.
    const size_t tc_blocks = m.items_full_tc.size() * (size_t)((d / 64 + ATTC_HEADS - 1) / ATTC_HEADS);
    const bool long_rows = T >= 2 * ATTC_BQ && T >= ATTC_BQ * std::max(m.n, 1);
    const bool tc = B.attn_mode == s1c_backend::ATTN_TC ||
                    (B.attn_mode == s1c_backend::ATTN_AUTO && !rows && (tc_blocks >= (size_t)nsm || long_rows));
    const int4* items = tc ? (rows ? dm.items_rows_tc : dm.items_full_tc) : (rows ? dm.items_rows : dm.items_full);
    const int n_items = (int)(tc ? (rows ? m.items_rows_tc.size() : m.items_full_tc.size())
                                 : (rows ? m.items_rows.size() : m.items_full.size()));
    if (n_items == 0) return;
    if (tc) {
      AttnTcArgs a{dm.acu, items, o, os, q_col0, k_col0, v_col0, d / 64, window, scale_log2, B.d_status, n_items};
      launch(B, nl, name, 4.0 * d * pairs, 0, [&] {
        const dim3 grid((unsigned)attc_grid(n_items, d / 64, nsm));
        launch_k(attention_tc_kernel, grid, dim3(ATTC_THREADS), ATTC_SMEM, st, tq, tkv, a);
      });
    } else {
      AttnArgs a{q, k, v, o, qs, ks, vs, os, dm.acu, items, window, scale_log2, d / 64};
      launch(B, nl, name, 4.0 * d * pairs, 0, [&] {
        launch_k(attention_varlen_kernel, dim3((unsigned)n_items * (d / 64)), dim3(ATT_THREADS), 0, st, a);
      });
    }
  };
  auto gemm_args = [&](int M, int N, int K) {
    GemmArgs a{};
    a.M = M; a.N = N; a.K = K; a.status = B.d_status;
    return a;
  };
  auto ln = [&](const char* name, const auto* in, const int* gather, int rows, const float* w, const float* b,
                float eps, bf16* out) {
    launch(B, nl, name, 0, (double)rows * d * (sizeof(*in) + 2.0),
           [&] { launch_ln<D>(in, gather, rows, w, b, eps, out, st, nsm); });
  };
  const double fl = 2.0 * T;  // GEMM FLOPs per (output column x reduction element)
  // Split-K contexts: the output buffer and pitch the finalize step writes (for residual GEMMs the
  // stream it adds to).
  auto sk = [&](void* out, int ldo) { return SplitCtx{B.splitk_ws.as<float>(), B.splitk_ws.bytes, out, ldo}; };
  SplitCtx sk_tmp{};

  for (int i = 0; i < B.L; ++i) {
    const EncLayer& l = B.layers[i];
    if (B.trace_layers) CK(cudaEventRecord(B.layer_ev[i], st));
    nvtxRangePushA(l.local ? "s1c encoder layer (window)" : "s1c encoder layer (global)");
    struct Pop {
      ~Pop() { nvtxRangePop(); }
    } pop;
    if (i > 0) ln("ln_attn", h, nullptr, T, l.attn_norm, nullptr, B.eps, x);
    GemmArgs g = gemm_args(T, 3 * d, d);
    g.pos = pos;
    g.inv_freq = B.inv_freq[l.local ? 1 : 0];
    g.rope_tab = B.rope_tab[l.local ? 1 : 0];
    g.rope_cols = 2 * d;
    // Each encoder GEMM names the next one's weights: the cluster split-K kernel (small batches,
    // where every GEMM streams its weights from HBM) prefetches them into L2 while it runs.
    g.pf = l.wo;
    g.pf_bytes = (size_t)d * d * 2;
    launch(B, nl, "gemm_qkv_rope", fl * 3 * d * d, 0, [&] { launch_gemm<EPI_ROPE>(B.tm_x, l.tm_wqkv, B.to_qkv3, g, nsm, st, B.gemm_variant, &(sk_tmp = sk(qkv, 3 * d)), &nl); });
    attn(l.local ? "attn_local" : "attn_global", B.tm_qkv_att, B.tm_qkv_kv, 0, d, 2 * d, qkv, qkv + d,
         qkv + 2 * d, att, 3 * d, 3 * d, 3 * d, d, false, l.local ? B.window : -1,
         l.local ? m.pairs_local : m.pairs_global);
    GemmArgs go = gemm_args(T, d, d);
    go.pf = l.wi;
    go.pf_bytes = (size_t)B.Ipad * d * 2;
    launch(B, nl, "gemm_wo_resid", fl * d * d, 0, [&] { launch_gemm<EPI_RESID16>(B.tm_att, l.tm_wo, B.to_h, go, nsm, st, B.gemm_variant, &(sk_tmp = sk(h, d)), &nl); });
    ln("ln_mlp", h, nullptr, T, l.mlp_norm, nullptr, B.eps, x);
    GemmArgs gi = gemm_args(T, B.Ipad, d);
    gi.out_cols = B.I;
    gi.pf = l.wo2;
    gi.pf_bytes = (size_t)d * B.I * 2;
    launch(B, nl, "gemm_wi_geglu", fl * 2 * B.I * d, 0, [&] { launch_gemm<EPI_GEGLU>(B.tm_x, l.tm_wi, B.to_act_i, gi, nsm, st, B.gemm_variant, &(sk_tmp = sk(act, B.I)), &nl); });
    GemmArgs g2 = gemm_args(T, d, B.I);
    g2.pf = i + 1 < B.L ? static_cast<const void*>(B.layers[i + 1].wqkv) : static_cast<const void*>(B.head[0].in_w);
    g2.pf_bytes = (size_t)3 * d * d * 2;
    launch(B, nl, "gemm_wo2_resid", fl * B.I * d, 0,
           [&] { launch_gemm<EPI_RESID16>(B.tm_act_i, l.tm_wo2, B.to_h, g2, nsm, st, B.gemm_variant, &(sk_tmp = sk(h, d)), &nl); });
  }

  if (B.trace_layers) CK(cudaEventRecord(B.layer_ev[B.L], st));
  // final_norm, + type embedding, head layer 0's norm1
  launch(B, nl, "final_to_head", 0, Td * (2 + 4 + 2 + (d_hidden ? 4 : 0)), [&] {
    launch_k(final_to_head_kernel<D>, dim3((T + 7) / 8), dim3(256), 0, st, h, T, B.final_norm, B.eps, d_hidden, m.hidden_rows, trow, dm.qtype,
                                                         B.type_emb, B.head[0].n1w, B.head[0].n1b, h2, x);
  });

  // full head layers (all but the last)
  for (int j = 0; j + 1 < B.n_head; ++j) {
    const HeadLayer& hl = B.head[j];
    GemmArgs g = gemm_args(T, 3 * d, d);
    g.bias = hl.in_b;
    launch(B, nl, "head_gemm_in", fl * 3 * d * d, 0, [&] { launch_gemm<EPI_STORE>(B.tm_x, hl.tm_in, B.to_qkv3, g, nsm, st, B.gemm_variant, &(sk_tmp = sk(qkv, 3 * d)), &nl); });
    attn("head_attn", B.tm_qkv_att, B.tm_qkv_kv, 0, d, 2 * d, qkv, qkv + d, qkv + 2 * d, att, 3 * d, 3 * d,
         3 * d, d, false, -1, m.pairs_global);
    GemmArgs go = gemm_args(T, d, d);
    go.bias = hl.out_b;
    launch(B, nl, "head_gemm_out", fl * d * d, 0, [&] { launch_gemm<EPI_RESID>(B.tm_att, hl.tm_out, B.to_h2, go, nsm, st, B.gemm_variant, &(sk_tmp = sk(h2, d)), &nl); });
    ln("head_ln", h2, nullptr, T, hl.n2w, hl.n2b, 1e-5f, x);
    GemmArgs g1 = gemm_args(T, B.F, d);
    g1.bias = hl.l1_b;
    g1.act = ACT_RELU;
    launch(B, nl, "head_gemm_l1", fl * B.F * d, 0, [&] { launch_gemm<EPI_STORE>(B.tm_x, hl.tm_l1, B.to_act_f, g1, nsm, st, B.gemm_variant, &(sk_tmp = sk(act, B.F)), &nl); });
    GemmArgs g2 = gemm_args(T, d, B.F);
    g2.bias = hl.l2_b;
    launch(B, nl, "head_gemm_l2", fl * B.F * d, 0,
           [&] { launch_gemm<EPI_RESID>(B.tm_act_f, hl.tm_l2, B.to_h2, g2, nsm, st, B.gemm_variant, &(sk_tmp = sk(h2, d)), &nl); });
    const HeadLayer& nx = B.head[j + 1];
    ln("head_ln", h2, nullptr, T, nx.n1w, nx.n1b, 1e-5f, x);
  }

  // last head layer, pruned to the scorer's rows: keys/values from every token, the rest at
  // position 0 and the marker slots only (lib.rs:1728-1748)
  {
    const HeadLayer& hl = B.head[B.n_head - 1];
    const int R = m.R;
    const double flr = 2.0 * R;
    bf16* kv = qkv;  // [T, 2d]
    GemmArgs gkv = gemm_args(T, 2 * d, d);
    gkv.bias = hl.in_b + d;
    launch(B, nl, "head_gemm_kv", fl * 2 * d * d, 0,
           [&] { launch_gemm<EPI_STORE>(B.tm_x, hl.tm_in_kv, B.to_kv2, gkv, nsm, st, B.gemm_variant, &(sk_tmp = sk(qkv, 2 * d)), &nl); });
    launch(B, nl, "gather_rows", 0, (double)R * d * 4, [&] {
      launch_k(gather_rows_bf16_kernel, dim3(R), dim3(128), 0, st, x, dm.srows, R, d, B.xs.as<bf16>());
    });
    launch(B, nl, "gather_rows", 0, (double)R * d * 8, [&] {
      launch_k(gather_rows_f32_kernel, dim3(R), dim3(256), 0, st, h2, dm.srows, R, d, B.hs.as<float>());
    });
    GemmArgs gq = gemm_args(R, d, d);
    gq.bias = hl.in_b;
    launch(B, nl, "head_rows_gemm", flr * d * d, 0, [&] { launch_gemm<EPI_STORE>(B.tm_xs, hl.tm_in_q, B.to_qs, gq, nsm, st, B.gemm_variant, &(sk_tmp = sk(B.qs.p, d)), &nl); });
    attn("head_rows_attn", B.tm_qs_att, B.tm_kv_att, 0, 0, d, B.qs.as<bf16>(), kv, kv + d, B.atts.as<bf16>(), d,
         2 * d, 2 * d, d, true, -1, m.pairs_rows);
    GemmArgs go = gemm_args(R, d, d);
    go.bias = hl.out_b;
    launch(B, nl, "head_rows_gemm", flr * d * d, 0,
           [&] { launch_gemm<EPI_RESID>(B.tm_atts, hl.tm_out, B.to_hs, go, nsm, st, B.gemm_variant, &(sk_tmp = sk(B.hs.p, d)), &nl); });
    ln("head_ln", B.hs.as<float>(), nullptr, R, hl.n2w, hl.n2b, 1e-5f, B.xs.as<bf16>());
    GemmArgs g1 = gemm_args(R, B.F, d);
    g1.bias = hl.l1_b;
    g1.act = ACT_RELU;
    launch(B, nl, "head_rows_gemm", flr * B.F * d, 0,
           [&] { launch_gemm<EPI_STORE>(B.tm_xs, hl.tm_l1, B.to_fs, g1, nsm, st, B.gemm_variant, &(sk_tmp = sk(B.fs.p, B.F)), &nl); });
    GemmArgs g2 = gemm_args(R, d, B.F);
    g2.bias = hl.l2_b;
    launch(B, nl, "head_rows_gemm", flr * B.F * d, 0,
           [&] { launch_gemm<EPI_RESID>(B.tm_fs, hl.tm_l2, B.to_hs, g2, nsm, st, B.gemm_variant, &(sk_tmp = sk(B.hs.p, d)), &nl); });
  }

  // scorer at the marker slots, pooled at position 0
  if (m.M > 0) {
    ln("scorer_ln", B.hs.as<float>(), dm.mrows, m.M, B.sc_nw, B.sc_nb, 1e-5f, B.xm.as<bf16>());
    GemmArgs gs = gemm_args(m.M, B.S, d);
    gs.bias = B.sc_b1;
    gs.act = ACT_GELU;
    gs.out_f32 = 1;
    launch(B, nl, "scorer_gemm", 2.0 * m.M * B.S * d, 0,
           [&] { launch_gemm<EPI_STORE>(B.tm_xm, B.tm_sc1, B.to_sh, gs, nsm, st, B.gemm_variant, &(sk_tmp = sk(B.sh.p, B.S)), &nl); });
    launch(B, nl, "scorer_logits", 2.0 * m.M * B.S, 0, [&] {
      launch_k(scorer_logits_kernel, dim3((m.M + 7) / 8), dim3(256), 0, st, B.sh.as<float>(), m.M, B.S, B.sc_w3, B.sc_b3, dm.mcount,
                                                          m.kmax, d_logits);
    });
  }
  if (m.n > 0) {
    launch(B, nl, "gather_rows", 0, (double)m.n * d * 8, [&] {
      launch_k(gather_rows_f32_kernel, dim3(m.n), dim3(256), 0, st, B.hs.as<float>(), dm.prows, m.n, d, d_pooled);
    });
  }
  B.launches = nl;
}

void forward_enqueue(s1c_backend& B, const HostMeta& m, const DevMeta& dm, const uint32_t* d_ids, float* d_logits,
                     float* d_pooled, float* d_hidden) {
  t_pdl = B.pdl;
  t_gemm_off = B.gemm_off;
  struct Reset {
    ~Reset() { t_gemm_off = 0; }
  } reset;
  switch (B.d) {
    case 256: run_forward<256>(B, m, dm, d_ids, d_logits, d_pooled, d_hidden); break;
    case 768: run_forward<768>(B, m, dm, d_ids, d_logits, d_pooled, d_hidden); break;
    case 1024: run_forward<1024>(B, m, dm, d_ids, d_logits, d_pooled, d_hidden); break;
    default: throw S1cError(S1C_ERR_CONFIG, "unsupported hidden size");
  }
}

// The trace lines of the last traced forward (after its stream has drained).
void trace_report(s1c_backend& B, const std::map<std::string, ProfStat>& ops_before) {
  if (!B.tr_pending) return;
  B.tr_pending = false;
  float dev_ms = 0.f;
  CK(cudaEventElapsedTime(&dev_ms, B.tr_ev[0], B.tr_ev[1]));
  if (B.trace)
    std::fprintf(stderr, "s1c trace: %s enqueue %.1f us device %.3f ms\n", B.tr_desc.c_str(), B.tr_enqueue_us, dev_ms);
  if (B.trace_layers && (int)B.layer_ev.size() == B.L + 1) {
    std::string line = "s1c layers (ms):";
    char buf[32];
    for (int i = 0; i < B.L; ++i) {
      float ms = 0.f;
      CK(cudaEventElapsedTime(&ms, B.layer_ev[i], B.layer_ev[i + 1]));
      std::snprintf(buf, sizeof buf, " %d:%.3f", i, ms);
      line += buf;
    }
    std::fprintf(stderr, "%s\n", line.c_str());
  }
  if (B.trace_ops) {
    for (const auto& kv : B.prof_stats) {
      auto it = ops_before.find(kv.first);
      const double ms = kv.second.ms - (it == ops_before.end() ? 0.0 : it->second.ms);
      const int64_t n = kv.second.launches - (it == ops_before.end() ? 0 : it->second.launches);
      if (n > 0) std::fprintf(stderr, "s1c ops: %-16s %4lld launches %8.3f ms\n", kv.first.c_str(), (long long)n, ms);
    }
    if (!B.prof_user) B.prof_stats.clear();
  }
}

void check_status(s1c_backend& B) {
  CK(cudaMemcpyAsync(B.h_status, B.d_status, sizeof(int), cudaMemcpyDeviceToHost, B.stream));
  CK(cudaStreamSynchronize(B.stream));
  const std::map<std::string, ProfStat> ops_before = B.trace_ops && B.prof_user ? B.prof_stats
                                                                                 : std::map<std::string, ProfStat>{};
  if (!B.prof_pending.empty()) prof_collect(B);
  trace_report(B, ops_before);
  if (*B.h_status != 0) {
    const int code = *B.h_status;
    CK(cudaMemsetAsync(B.d_status, 0, sizeof(int), B.stream));
    CK(cudaStreamSynchronize(B.stream));
    if (code == DEV_BAD_INDEX) throw S1cError(S1C_ERR_ARG, "a token id is outside the vocabulary");
    throw S1cError(S1C_ERR_DEVICE_TIMEOUT, "device-side wait ran out (code " + std::to_string(code) + ")");
  }
}

// Shape buckets (settings `buckets=`, `warm=`; the reference's length buckets and load-time
// warm-up, laya-mlx/src/lib.rs:89-94, :1152-1173, :1826-1831). A batch whose packed tokens fit a
// bucket runs as the bucket's shape: its rows first, then `nb - n` dummy rows (token id 0, no
// markers) that hold the bucket's remaining tokens (none when the tokens fill the bucket exactly),
// markers padded to `kb` slots per row. Dummy
// rows get no attention work items: their tokens' attention outputs are never written, so
// whatever those rows compute stays in their own rows (every kernel but attention is row-local,
// and attention only reads keys of a query's own row) and is dropped with them. The work lists
// are filled with empty items to lengths fixed by (T, nb, kb), so one captured graph per bucket
// shape replays every batch of that shape. Row counts are bucketed to powers of two up to 64 (at
// least one dummy row whenever there are tokens to hold), marker slots to 4, or to a multiple of
// 16 past 4 (the pruned head rows are one 128-row tile either way for a few rows).
constexpr int BUCKET_MAX_ROWS = 64;
struct BucketShape {
  int T = 0, n = 0, kmax = 0;
};
bool pick_bucket(const s1c_backend& B, const s1c_varlen& in, BucketShape& out) {
  if (B.buckets.empty() || in.n == 0) return false;
  const int T = in.cu_seqlens[in.n];
  if (in.n > BUCKET_MAX_ROWS) return false;
  int nb = 2;  // with padding tokens: room for at least one dummy row
  while (nb < in.n + 1) nb *= 2;
  for (int t : B.buckets) {
    const int pad = t - T;
    if (pad < 0) continue;
    int rows = in.n;  // the tokens fill the bucket: no dummy rows
    if (pad > 0) {
      if (nb > BUCKET_MAX_ROWS || pad < nb - in.n) continue;  // every dummy row holds at least one token
      if ((int64_t)pad > (int64_t)(nb - in.n) * B.max_pos) return false;  // dummy rows within max_position
      rows = nb;
    }
    out.T = t;
    out.n = rows;
    out.kmax = in.kmax <= 4 ? 4 : (in.kmax + 15) / 16 * 16;
    return true;
  }
  return false;
}
ItemPad bucket_item_pad(const BucketShape& bs) {
  // sum over rows of ceil(len / tile) <= ceil(T / tile) + rows
  ItemPad p;
  p.on = true;
  p.full = (bs.T + ATT_BQ - 1) / ATT_BQ + bs.n;
  p.full_tc = (bs.T + ATTC_BQ - 1) / ATTC_BQ + bs.n;
  p.rows = bs.n * ((1 + bs.kmax + ATT_BQ - 1) / ATT_BQ);
  p.rows_tc = bs.n * ((1 + bs.kmax + ATTC_BQ - 1) / ATTC_BQ);
  return p;
}
// The batch `in` laid out as bucket shape `bs` (ids only when they come from the host).
struct BucketBatch {
  std::vector<uint32_t> ids, mpos, qtype;
  std::vector<int32_t> cu, mcount;
  s1c_varlen v{};
};
void make_bucket_batch(const s1c_varlen& in, const uint32_t* host_ids, const BucketShape& bs, BucketBatch& o) {
  const int T = in.cu_seqlens[in.n], nd = bs.n - in.n, pad = bs.T - T;
  o.cu.assign(in.cu_seqlens, in.cu_seqlens + in.n + 1);
  for (int r = 0; r < nd; ++r) o.cu.push_back(T + (int)((int64_t)pad * (r + 1) / nd));  // pad tokens spread evenly
  o.mcount.assign(bs.n, 0);
  o.qtype.assign(bs.n, 0);
  o.mpos.assign((size_t)bs.n * bs.kmax, 0);
  for (int r = 0; r < in.n; ++r) {
    o.mcount[r] = in.marker_count[r];
    o.qtype[r] = in.qtype[r];
    for (int k = 0; k < in.kmax; ++k) o.mpos[(size_t)r * bs.kmax + k] = in.marker_pos[(size_t)r * in.kmax + k];
  }
  if (host_ids) {
    o.ids.assign(bs.T, 0u);
    std::memcpy(o.ids.data(), host_ids, (size_t)T * 4);
  }
  o.v = s1c_varlen{bs.n, bs.kmax, host_ids ? o.ids.data() : nullptr, o.cu.data(), o.mpos.data(), o.mcount.data(),
                   o.qtype.data()};
}

// Enqueue one forward. Token ids come from the host (`host_ids`, staged with the metadata) or
// from device memory (`dev_ids`, copied into the arena); logits and pooled land in `out_stage`;
// `d_hidden` (nullable) receives the encoder's final hidden state of the batch's own tokens.
// With graphs on, a bucket shape replays its graph from its first sighting on (captured then),
// any other shape from its third (captured at the second).
struct StageOut {
  float* logits;   // [n, kstride] (the batch's rows; slots past kmax belong to the bucket)
  float* pooled;   // [n, d]
  size_t n_logits, n_pooled;  // n * kstride, n * d
  int n = 0, kmax = 0, kstride = 0;
};
StageOut enqueue_forward_impl(s1c_backend& B, const s1c_varlen& in, const uint32_t* host_ids, const uint32_t* dev_ids,
                              float* d_hidden, const int* real_len, std::string& how);
StageOut enqueue_forward(s1c_backend& B, const s1c_varlen& in, const uint32_t* host_ids, const uint32_t* dev_ids,
                         float* d_hidden, const int* real_len = nullptr) {
  nvtxRangePushA("s1c forward");
  struct Pop {
    ~Pop() { nvtxRangePop(); }
  } pop;
  const bool tracing = B.trace || B.trace_layers || B.trace_ops;
  B.prof_on = B.prof_user || B.trace_ops;
  if (!tracing) {
    std::string how;
    return enqueue_forward_impl(B, in, host_ids, dev_ids, d_hidden, real_len, how);
  }
  for (cudaEvent_t& e : B.tr_ev)
    if (!e) CK(cudaEventCreate(&e));
  if (B.trace_layers && B.layer_ev.empty()) {
    B.layer_ev.resize(B.L + 1);
    for (cudaEvent_t& e : B.layer_ev) CK(cudaEventCreate(&e));
  }
  const auto t0 = std::chrono::steady_clock::now();
  CK(cudaEventRecord(B.tr_ev[0], B.stream));
  std::string how;
  const StageOut so = enqueue_forward_impl(B, in, host_ids, dev_ids, d_hidden, real_len, how);
  CK(cudaEventRecord(B.tr_ev[1], B.stream));
  B.tr_enqueue_us = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
  B.tr_pending = true;
  B.tr_desc = "rows " + std::to_string(in.n) + " tokens " + std::to_string(in.cu_seqlens[in.n]) + " kmax " +
              std::to_string(in.kmax) + " " + how + " launches " + std::to_string(B.launches);
  return so;
}
StageOut enqueue_forward_impl(s1c_backend& B, const s1c_varlen& in, const uint32_t* host_ids, const uint32_t* dev_ids,
                              float* d_hidden, const int* real_len, std::string& how) {
  BucketShape bs;
  BucketBatch bb;
  const bool bucketed = !real_len && pick_bucket(B, in, bs);
  if (bucketed) make_bucket_batch(in, host_ids, bs, bb);
  const s1c_varlen& run = bucketed ? bb.v : in;
  const int T_in = in.cu_seqlens[in.n];
  HostMeta m = make_meta(run, B.window, in.n, bucketed ? bucket_item_pad(bs) : ItemPad{}, real_len);
  m.hidden_rows = T_in;
  ensure_capacity(B, m.T, m.R);
  const size_t nl = (size_t)m.M, np = (size_t)m.n * B.d;
  const size_t need = ((nl + 63) / 64 * 64 + np) * 4;
  if (need > B.out_stage.bytes) {
    CK(cudaStreamSynchronize(B.stream));
    B.drop_graphs();
    B.out_stage.ensure(need * 2);
  }
  StageOut so{B.out_stage.as<float>(), B.out_stage.as<float>() + (nl + 63) / 64 * 64,
              in.kmax ? (size_t)in.n * run.kmax : 0, (size_t)in.n * B.d, in.n, in.kmax, run.kmax};
  DevMeta dm = upload_meta(B, m, host_ids ? run.ids : nullptr);
  if (dev_ids) {
    CK(cudaMemcpyAsync(const_cast<uint32_t*>(dm.ids), dev_ids, (size_t)T_in * 4, cudaMemcpyDeviceToDevice, B.stream));
    if (m.T > T_in)
      CK(cudaMemsetAsync(const_cast<uint32_t*>(dm.ids) + T_in, 0, (size_t)(m.T - T_in) * 4, B.stream));
  }
  how = bucketed ? "bucket " + std::to_string(m.T) + "x" + std::to_string(m.n) + "x" + std::to_string(m.kmax)
                 : std::string("exact shape");
  const bool graphable = B.use_graphs && !d_hidden && !B.prof_on && !B.trace_layers && B.stream != nullptr &&
                         B.stream != cudaStreamLegacy && B.stream != cudaStreamPerThread;
  if (!graphable) {
    how += ", direct";
    forward_enqueue(B, m, dm, dm.ids, so.logits, so.pooled, d_hidden);
    return so;
  }
  const std::vector<int> key = {m.T, m.n, m.kmax, (int)m.items_full.size(), (int)m.items_rows.size(),
                                (int)m.items_full_tc.size(), (int)m.items_rows_tc.size()};
  auto it = B.graphs.find(key);
  if (it == B.graphs.end()) {
    if (!bucketed) {
      if (B.seen.size() >= s1c_backend::MAX_SEEN) B.seen.clear();  // forget one-off shapes
      if (B.seen[key]++ < 1) {  // first sighting of an unbucketed shape: launch directly
        how += ", direct (first sighting)";
        forward_enqueue(B, m, dm, dm.ids, so.logits, so.pooled, nullptr);
        return so;
      }
    }
    B.evict_graphs(s1c_backend::MAX_GRAPHS - 1);
    cudaGraph_t g = nullptr;
    CK(cudaStreamBeginCapture(B.stream, cudaStreamCaptureModeThreadLocal));
    try {
      forward_enqueue(B, m, dm, dm.ids, so.logits, so.pooled, nullptr);
    } catch (...) {
      cudaStreamEndCapture(B.stream, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    CK(cudaStreamEndCapture(B.stream, &g));
    s1c_backend::Graph gr;
    const cudaError_t e = cudaGraphInstantiate(&gr.exec, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) throw S1cError(S1C_ERR_CUDA, std::string("cudaGraphInstantiate: ") + cudaGetErrorString(e));
    gr.launches = B.launches;
    B.seen.erase(key);
    it = B.graphs.emplace(key, gr).first;
    how += ", graph captured";
  } else {
    how += ", graph replayed";
  }
  it->second.last_used = ++B.graph_clock;
  CK(cudaGraphLaunch(it->second.exec, B.stream));
  B.launches = it->second.launches;
  return so;
}

// Host-buffer forward: ids and metadata copied in, logits / pooled / hidden copied out. With
// `real_len`, row r's first real_len[r] tokens are its real tokens and the rest padding tokens that
// attend them (never attended themselves).
void forward_host(s1c_backend& B, const s1c_varlen& in, float* logits, float* pooled, float* hidden,
                  const int* real_len = nullptr) {
  validate_varlen(B, in);
  if (in.n == 0) return;
  if (!in.ids) throw S1cError(S1C_ERR_ARG, "null batch array");
  const int T = in.cu_seqlens[in.n];
  for (int t = 0; t < T; ++t)
    if (in.ids[t] >= (uint32_t)B.V) throw S1cError(S1C_ERR_ARG, "token " + std::to_string(t) + ": id outside the vocabulary");
  const size_t nh = hidden ? (size_t)T * B.d : 0;
  DevBuf hid_dev;
  if (nh) hid_dev.ensure(nh * 4);
  const StageOut so = enqueue_forward(B, in, in.ids, nullptr, nh ? hid_dev.as<float>() : nullptr, real_len);
  const size_t out_bytes = (so.n_logits + so.n_pooled + nh) * 4;
  if (out_bytes > B.h_out_bytes) {
    CK(cudaStreamSynchronize(B.stream));
    if (B.h_out) cudaFreeHost(B.h_out);
    B.h_out = nullptr;
    B.h_out_bytes = 0;
    CK(cudaMallocHost(&B.h_out, out_bytes * 2 + 64));
    B.h_out_bytes = out_bytes * 2 + 64;
  }
  float* ho = B.h_out;
  if (so.n_logits) CK(cudaMemcpyAsync(ho, so.logits, so.n_logits * 4, cudaMemcpyDeviceToHost, B.stream));
  CK(cudaMemcpyAsync(ho + so.n_logits, so.pooled, so.n_pooled * 4, cudaMemcpyDeviceToHost, B.stream));
  if (nh) CK(cudaMemcpyAsync(ho + so.n_logits + so.n_pooled, hid_dev.p, nh * 4, cudaMemcpyDeviceToHost, B.stream));
  check_status(B);
  if (so.n_logits) {
    if (so.kstride == so.kmax) std::memcpy(logits, ho, so.n_logits * 4);
    else
      for (int r = 0; r < so.n; ++r) std::memcpy(logits + (size_t)r * so.kmax, ho + (size_t)r * so.kstride, (size_t)so.kmax * 4);
  }
  std::memcpy(pooled, ho + so.n_logits, so.n_pooled * 4);
  if (nh) std::memcpy(hidden, ho + so.n_logits + so.n_pooled, nh * 4);
}

// Device-buffer forward: ids already on the device, outputs copied device to device.
void forward_device(s1c_backend& B, const s1c_varlen& in, const uint32_t* d_ids, float* d_logits, float* d_pooled,
                    float* d_hidden) {
  validate_varlen(B, in);
  if (in.n == 0) return;
  if (!d_ids || !d_pooled || (in.kmax > 0 && !d_logits)) throw S1cError(S1C_ERR_ARG, "null device pointer");
  const StageOut so = enqueue_forward(B, in, nullptr, d_ids, d_hidden);
  if (so.n_logits && so.kmax) {
    if (so.kstride == so.kmax)
      CK(cudaMemcpyAsync(d_logits, so.logits, so.n_logits * 4, cudaMemcpyDeviceToDevice, B.stream));
    else
      CK(cudaMemcpy2DAsync(d_logits, (size_t)so.kmax * 4, so.logits, (size_t)so.kstride * 4, (size_t)so.kmax * 4,
                           (size_t)so.n, cudaMemcpyDeviceToDevice, B.stream));
  }
  CK(cudaMemcpyAsync(d_pooled, so.pooled, so.n_pooled * 4, cudaMemcpyDeviceToDevice, B.stream));
}

// Padded Batch -> varlen (Packing::new, lib.rs:906-930): real tokens row-major; positions are
// indices inside the row; markers keep their in-row positions.
struct PackedBatch {
  std::vector<uint32_t> ids;
  std::vector<int32_t> cu, mcount;
  std::vector<uint32_t> mpos, qtype;
  s1c_varlen v{};
};
void pack_batch(const s1c_batch& b, PackedBatch& p) {
  if (!b.input_ids || !b.attention_mask || !b.seq_lens || !b.marker_count || !b.qtype || (b.kmax && !b.marker_pos))
    throw S1cError(S1C_ERR_ARG, "null batch array");
  p.cu.assign(1, 0);
  for (size_t r = 0; r < b.n; ++r) {
    const size_t s = b.seq_lens[r];
    if (s < 1 || s > b.len) throw S1cError(S1C_ERR_ARG, "row " + std::to_string(r) + ": seq_len outside 1..len");
    for (size_t pos = 0; pos < b.len; ++pos) {
      const uint32_t mk = b.attention_mask[r * b.len + pos];
      if (mk != (pos < s ? 1u : 0u))
        throw S1cError(S1C_ERR_ARG, "row " + std::to_string(r) + ": attention mask does not match seq_len " +
                                        std::to_string(s));
      if (mk == 1) p.ids.push_back(b.input_ids[r * b.len + pos]);
    }
    p.cu.push_back((int32_t)p.ids.size());
    if (b.marker_count[r] > b.kmax) throw S1cError(S1C_ERR_ARG, "row " + std::to_string(r) + ": marker_count > kmax");
    p.mcount.push_back((int32_t)b.marker_count[r]);
    p.qtype.push_back(b.qtype[r]);
  }
  p.mpos.assign(b.marker_pos, b.marker_pos + b.n * b.kmax);
  p.v.n = (int32_t)b.n;
  p.v.kmax = (int32_t)b.kmax;
  p.v.ids = p.ids.data();
  p.v.cu_seqlens = p.cu.data();
  p.v.marker_pos = p.mpos.data();
  p.v.marker_count = p.mcount.data();
  p.v.qtype = p.qtype.data();
}

// Backend settings, a strict comma list like the reference's `Knobs` (laya-mlx/src/lib.rs:155-259):
// an unknown key or value is an error naming it. Keys: attn=auto|tc|mma,
// gemm=auto|1cta|2cta|splitk|csk, graphs=0|1, pdl=0|1, buckets=<t>:<t>... (packed-token buckets,
// 0 = none), warm=<rows>:... (row counts s1c_warmup runs at every bucket), check=0|1, check_fail=.
void apply_settings(s1c_backend& B, const char* spec) {
  if (!spec) return;
  std::string s(spec);
  size_t i = 0;
  while (i <= s.size()) {
    size_t j = s.find(',', i);
    if (j == std::string::npos) j = s.size();
    const std::string kv = s.substr(i, j - i);
    i = j + 1;
    if (kv.empty()) continue;
    const size_t eq = kv.find('=');
    const std::string k = kv.substr(0, eq), v = eq == std::string::npos ? "" : kv.substr(eq + 1);
    if (k == "pdl") {
      if (v == "1") B.pdl = true;
      else if (v == "0") B.pdl = false;
      else throw S1cError(S1C_ERR_CONFIG, "settings: `" + kv + "`: `" + v + "` is not 0 or 1");
    } else if (k == "graphs") {
      if (v == "1") B.use_graphs = true;
      else if (v == "0") B.use_graphs = false;
      else throw S1cError(S1C_ERR_CONFIG, "settings: `" + kv + "`: `" + v + "` is not 0 or 1");
    } else if (k == "gemm") {
      if (v == "auto") B.gemm_variant = 0;
      else if (v == "1cta") B.gemm_variant = 1;
      else if (v == "2cta") B.gemm_variant = 2;
      else if (v == "splitk") B.gemm_variant = 3;
      else if (v == "csk") B.gemm_variant = 4;
      else throw S1cError(S1C_ERR_CONFIG, "settings: `" + kv + "`: `" + v + "` is not one of auto, 1cta, 2cta, splitk, csk");
    } else if (k == "attn") {
      if (v == "auto") B.attn_mode = s1c_backend::ATTN_AUTO;
      else if (v == "tc") B.attn_mode = s1c_backend::ATTN_TC;
      else if (v == "mma") B.attn_mode = s1c_backend::ATTN_MMA;
      else throw S1cError(S1C_ERR_CONFIG, "settings: `" + kv + "`: `" + v + "` is not one of tc, mma");
    } else if (k == "buckets" || k == "warm") {
      // colon list of positive whole numbers; `buckets=0` turns the buckets off
      std::vector<int> vals;
      size_t a = 0;
      while (a <= v.size()) {
        size_t e = v.find(':', a);
        if (e == std::string::npos) e = v.size();
        const std::string t = v.substr(a, e - a);
        a = e + 1;
        char* end = nullptr;
        const long x = t.empty() ? -1 : std::strtol(t.c_str(), &end, 10);
        if (t.empty() || *end || x < 0 || x > (1 << 24))
          throw S1cError(S1C_ERR_CONFIG, "settings: `" + kv + "`: `" + t + "` is not a whole number");
        if (x > 0) vals.push_back((int)x);
      }
      std::sort(vals.begin(), vals.end());
      vals.erase(std::unique(vals.begin(), vals.end()), vals.end());
      if (k == "buckets") B.buckets = vals;
      else B.warm_rows = vals;
    } else if (k == "trace" || k == "layers" || k == "ops") {
      bool on;
      if (v.empty() || v == "1") on = true;
      else if (v == "0") on = false;
      else throw S1cError(S1C_ERR_CONFIG, "settings: `" + kv + "`: `" + v + "` is not 0 or 1");
      (k == "trace" ? B.trace : k == "layers" ? B.trace_layers : B.trace_ops) = on;
    } else if (k == "parallel_load") {
      // the runtime's own setting (BackendOptions::parallel_load, laya-core/src/backend.rs:44-66),
      // accepted here as the reference's backends accept it
      if (!v.empty() && v != "0" && v != "1")
        throw S1cError(S1C_ERR_CONFIG, "settings: `" + kv + "`: `" + v + "` is not 0 or 1");
    } else if (k == "check") {
      if (v == "1") B.check = true;
      else if (v == "0") B.check = false;
      else throw S1cError(S1C_ERR_CONFIG, "settings: `" + kv + "`: `" + v + "` is not 0 or 1");
    } else if (k == "check_fail") {
      size_t a = 0;
      while (a <= v.size()) {
        size_t e = v.find('+', a);
        if (e == std::string::npos) e = v.size();
        const std::string kern = v.substr(a, e - a);
        if (kern != "1cta" && kern != "2cta" && kern != "csk" && kern != "splitk" && kern != "tc" && kern != "mma")
          throw S1cError(S1C_ERR_CONFIG, "settings: `" + kv + "`: `" + kern + "` is not one of 1cta, 2cta, csk, splitk, tc, mma");
        a = e + 1;
      }
      B.check_fail = v;
    } else {
      throw S1cError(S1C_ERR_CONFIG, "settings: unknown setting `" + k + "`");
    }
  }
}

template <class F>
s1c_status guarded(s1c_backend* b, F&& f) {
  if (!b) return S1C_ERR_ARG;
  try {
    CK(cudaSetDevice(b->device));
    f();
    return S1C_OK;
  } catch (const S1cError& e) {
    b->last_error = e.what();
    return e.code;
  } catch (const std::exception& e) {
    b->last_error = e.what();
    return S1C_ERR_ARG;
  } catch (...) {
    b->last_error = "unknown error";
    return S1C_ERR_ARG;
  }
}

// ---------------------------------------------------------------------------------------------
// Load-time kernel self-check (setting `check=1`)
//
// The reference checks its fused kernels once at load against the op chains they replace and turns
// a kernel that does not reproduce them off for that load, with one line on stderr
// (laya-mlx/src/lib.rs:319-362, split_rope.rs:258-266). Here each kernel the forward can pick runs
// once on small seeded problems through the same launch code as the forward, and its output is
// compared with a plain computation on the host in double precision over the same bf16 inputs:
//   * GEMMs: the one-CTA, two-CTA and cluster split-K kernels (and the workspace split-K path when
//     `gemm=splitk` forces it), each with the bias + ReLU store, the bias + GELU fp32 store, the
//     fp32 and f16 residual adds, the RoPE and the GeGLU epilogues, at M = 300 (a partial last
//     tile);
//   * attention: the tcgen05 and mma.sync kernels, global and sliding window, over four ragged
//     sequences (200, 63, 129 and 1 tokens).
// An output passes when every element is within 1e-2 * (1 + |expected|) (bf16 output rounding is
// 2^-9 relative; a wrong tile, a missed mask or a lost accumulator is off by O(1)). A faster kernel
// that fails is turned off for this handle when a checked kernel can take its place (two-CTA or
// cluster split-K -> one-CTA GEMM; tcgen05 -> mma.sync attention), with one line on stderr and the
// change named in s1c_active_kernels. A failing one-CTA GEMM or mma.sync attention, or a failing
// kernel that the settings force, fails s1c_create with S1C_ERR_SELFCHECK.
//
// `check_fail=<kernel>[+<kernel>...]` (1cta, 2cta, csk, splitk, tc, mma) plants a wrong value in the
// host-side expected result of those kernels' checks: it lets tests drive the fallback rule (the
// reference's tests do the same by handing `rope_kernels` a failing build) without a faulty kernel.

constexpr double CHECK_TOL = 1e-2;

struct CheckRng {
  uint64_t s;
  float uniform() {  // [-1, 1), splitmix64
    s += 0x9E3779B97F4A7C15ull;
    uint64_t z = s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    z ^= z >> 31;
    return (float)((double)(z >> 40) * (1.0 / 8388608.0)) - 1.0f;
  }
};

// max over elements of |got - want| / (1 + |want|); NaN when any output is not finite
double scaled_err(const std::vector<float>& got, const std::vector<double>& want) {
  double e = 0;
  for (size_t i = 0; i < want.size(); ++i) {
    if (!std::isfinite(got[i])) return std::nan("");
    e = std::max(e, std::fabs((double)got[i] - want[i]) / (1.0 + std::fabs(want[i])));
  }
  return e;
}

// Output of a check as floats: fp32, bf16 or (f16) f16 elements.
std::vector<float> download(const void* d, size_t n, bool f32, bool f16 = false) {
  std::vector<float> out(n);
  if (f32) {
    CK(cudaMemcpy(out.data(), d, n * 4, cudaMemcpyDeviceToHost));
  } else {
    std::vector<uint16_t> raw(n);
    CK(cudaMemcpy(raw.data(), d, n * 2, cudaMemcpyDeviceToHost));
    for (size_t i = 0; i < n; ++i) out[i] = f16 ? f16_bits_to_f32(raw[i]) : bf16_bits_to_f32(raw[i]);
  }
  return out;
}

// Device buffers of one check. Uploads go through the check's stream and are waited for: the
// handle's stream does not synchronise with the legacy default stream, and a plain cudaMemcpy from
// pageable memory may return before its DMA has landed, so a kernel on the handle's stream could
// otherwise read an upload that is still in flight.
struct CheckBufs {
  cudaStream_t st;
  std::vector<void*> p;
  explicit CheckBufs(cudaStream_t s) : st(s) {}
  ~CheckBufs() {
    if (st) cudaStreamSynchronize(st);
    for (void* q : p) cudaFree(q);
  }
  template <class T>
  T* upload(const std::vector<T>& v) {
    void* q = nullptr;
    CK(cudaMalloc(&q, std::max<size_t>(v.size(), 1) * sizeof(T)));
    p.push_back(q);
    copy_in(q, v);
    return static_cast<T*>(q);
  }
  template <class T>
  void copy_in(void* q, const std::vector<T>& v) {
    CK(cudaMemcpyAsync(q, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice, st));
    CK(cudaStreamSynchronize(st));
  }
  void* alloc(size_t bytes) {
    void* q = nullptr;
    CK(cudaMalloc(&q, bytes));
    p.push_back(q);
    return q;
  }
};

double gelu_exact(double x) { return 0.5 * x * (1.0 + std::erf(x / std::sqrt(2.0))); }

// The GEMM problem of the check: A [300, 320] and B [768, 320] bf16 (unit-variance products), a
// bias, a residual, row positions, and A B^T over the bf16 inputs in double.
struct GemmCheck {
  static constexpr int M = 300, N = 768, K = 320, I = 384, ROPE_COLS = 512;
  static constexpr float THETA = 10000.0f;
  std::vector<uint16_t> a, b, resid16;
  std::vector<float> bias, resid;
  std::vector<int32_t> pos;
  std::vector<double> c;
  GemmCheck()
      : a((size_t)M * K), b((size_t)N * K), resid16((size_t)M * N), bias(N), resid((size_t)M * N), pos(M),
        c((size_t)M * N) {
    CheckRng rng{0x5e1fc4ec0001ull};
    const float sb = 3.0f / std::sqrt((float)K);
    for (auto& x : a) x = f32_to_bf16_bits(rng.uniform());
    for (auto& x : b) x = f32_to_bf16_bits(rng.uniform() * sb);
    for (auto& x : bias) x = 0.5f * rng.uniform();
    for (auto& x : resid) x = rng.uniform();
    for (size_t i = 0; i < resid.size(); ++i) resid16[i] = f32_to_f16_bits(resid[i]);
    for (int m = 0; m < M; ++m) pos[m] = (m * 37) % 1000;
    std::vector<double> af(a.size()), bfv(b.size());
    for (size_t i = 0; i < a.size(); ++i) af[i] = bf16_bits_to_f32(a[i]);
    for (size_t i = 0; i < b.size(); ++i) bfv[i] = bf16_bits_to_f32(b[i]);
    for (int m = 0; m < M; ++m)
      for (int n = 0; n < N; ++n) {
        const double* ar = &af[(size_t)m * K];
        const double* br = &bfv[(size_t)n * K];
        double s = 0;
        for (int k = 0; k < K; ++k) s += ar[k] * br[k];
        c[(size_t)m * N + n] = s;
      }
  }
  // Expected output of epilogue case `cs`: 0 bias + ReLU (bf16), 1 bias + GELU (fp32), 2 residual
  // + bias (fp32), 3 RoPE on the first ROPE_COLS columns (bf16), 4 GeGLU of the interleaved tiles
  // (bf16, I columns), 5 residual + bias on the f16 residual (f16).
  std::vector<double> want(int cs) const {
    std::vector<double> w(cs == 4 ? (size_t)M * I : (size_t)M * N);
    float inv_freq[32];
    const float lbase = std::log2(THETA);
    for (int i = 0; i < 32; ++i) inv_freq[i] = std::exp2(-((float)i / 32.0f) * lbase);
    for (int m = 0; m < M; ++m) {
      const double* row = &c[(size_t)m * N];
      if (cs == 4) {
        for (int j = 0; j < I; ++j) {
          const int t = j / 128, cc = j % 128;
          w[(size_t)m * I + j] = gelu_exact(row[256 * t + cc]) * row[256 * t + 128 + cc];
        }
        continue;
      }
      for (int n = 0; n < N; ++n) {
        double v = row[n];
        if (cs == 0) v = std::max(v + bias[n], 0.0);
        else if (cs == 1) v = gelu_exact(v + bias[n]);
        else if (cs == 2) v = (double)resid[(size_t)m * N + n] + v + bias[n];
        else if (cs == 5) v = (double)f16_bits_to_f32(resid16[(size_t)m * N + n]) + v + bias[n];
        else if (n < ROPE_COLS) {
          const int h0 = n / 64 * 64, i = n % 64, j = i % 32;
          const float ang = (float)pos[m] * inv_freq[j];  // the kernel's fp32 angle
          const double cs_ = std::cos((double)ang), sn = std::sin((double)ang);
          const double lo = row[h0 + j], hi = row[h0 + 32 + j];
          v = i < 32 ? lo * cs_ - hi * sn : lo * sn + hi * cs_;
        }
        w[(size_t)m * N + n] = v;
      }
    }
    return w;
  }
};

// One GEMM kernel (s1c_gemm variant: 1 one-CTA, 2 two-CTA, 3 workspace split-K, 4 cluster split-K)
// through the six epilogue cases; returns the largest scaled error (NaN for a non-finite output).
double check_gemm_kernel(const GemmCheck& g, const std::vector<std::vector<double>>& want, cudaStream_t st,
                         int variant, bool plant) {
  using G = GemmCheck;
  CheckBufs bufs(st);
  const uint16_t* dA = bufs.upload(g.a);
  const uint16_t* dB = bufs.upload(g.b);
  const float* dBias = bufs.upload(g.bias);
  const int32_t* dPos = bufs.upload(g.pos);
  void* dOut = bufs.alloc((size_t)G::M * G::N * 4);
  double worst = 0;
  for (int cs = 0; cs < 6; ++cs) {
    static const int epi_of[6] = {EPI_STORE, EPI_STORE, EPI_RESID, EPI_ROPE, EPI_GEGLU, EPI_RESID16};
    const int epi = epi_of[cs], f32 = (cs == 1 || cs == 2) ? 1 : 0;
    const int act = cs == 0 ? ACT_RELU : cs == 1 ? ACT_GELU : ACT_NONE;
    const float* bp = (cs <= 2 || cs == 5) ? dBias : nullptr;
    if (cs == 2) bufs.copy_in(dOut, g.resid);
    if (cs == 5) bufs.copy_in(dOut, g.resid16);
    const s1c_status rc = s1c_gemm(epi, dA, dB, dOut, G::M, G::N, G::K, bp, act, f32, dPos, G::THETA, G::ROPE_COLS,
                                   G::I, variant, st);
    if (rc != S1C_OK) throw S1cError(rc, "load check: GEMM launch: " + g_create_error);
    CK(cudaStreamSynchronize(st));
    std::vector<double> w = want[cs];
    if (plant) w[w.size() / 2] += 1.0;
    const double e = scaled_err(download(dOut, w.size(), f32 != 0, cs == 5), w);
    if (std::isnan(e)) return e;
    worst = std::max(worst, e);
  }
  return worst;
}

// The attention problem of the check: four ragged sequences (200, 63, 129, 1 tokens) of 4 heads in
// the forward's qkv layout [T, 3 x 256] (q scaled by 2 for sharper rows), and softmax(q k^T / 8) v
// in double over each query's key set: the whole sequence (window < 0) or |i - j| <= window.
struct AttnCheck {
  static constexpr int H = 4, D = H * 64, W = 3 * D;
  std::vector<int32_t> cu = {0, 200, 263, 392, 393};
  std::vector<uint16_t> qkv;
  AttnCheck() {
    const int T = cu.back();
    qkv.resize((size_t)T * W);
    CheckRng rng{0xa77e0001ull};
    for (int t = 0; t < T; ++t)
      for (int c = 0; c < W; ++c) qkv[(size_t)t * W + c] = f32_to_bf16_bits((c < D ? 2.0f : 1.0f) * rng.uniform());
  }
  std::vector<double> want(int window) const {
    const int n = (int)cu.size() - 1, T = cu[n];
    std::vector<double> f(qkv.size()), w((size_t)T * D), p;
    for (size_t i = 0; i < qkv.size(); ++i) f[i] = bf16_bits_to_f32(qkv[i]);
    for (int r = 0; r < n; ++r)
      for (int i = cu[r]; i < cu[r + 1]; ++i)
        for (int h = 0; h < H; ++h) {
          const int j0 = window < 0 ? cu[r] : std::max(cu[r], i - window);
          const int j1 = window < 0 ? cu[r + 1] : std::min(cu[r + 1], i + window + 1);
          p.assign((size_t)(j1 - j0), 0.0);
          double mx = -1e300;
          for (int j = j0; j < j1; ++j) {
            double s = 0;
            for (int e = 0; e < 64; ++e) s += f[(size_t)i * W + h * 64 + e] * f[(size_t)j * W + D + h * 64 + e];
            p[j - j0] = s * 0.125;
            mx = std::max(mx, p[j - j0]);
          }
          double sum = 0;
          for (double& x : p) sum += (x = std::exp(x - mx));
          for (int e = 0; e < 64; ++e) {
            double o = 0;
            for (int j = j0; j < j1; ++j) o += p[j - j0] * f[(size_t)j * W + 2 * D + h * 64 + e];
            w[(size_t)i * D + h * 64 + e] = o / sum;
          }
        }
    return w;
  }
};

// One attention kernel (impl 0 tcgen05, 1 mma.sync), global (want[0]) then sliding window with
// the model's half-width (want[1]); the largest scaled error.
double check_attention_kernel(const AttnCheck& a, const std::vector<double> (&want)[2], int window,
                              cudaStream_t st, int impl, bool plant) {
  using A = AttnCheck;
  const int n = (int)a.cu.size() - 1, T = a.cu[n];
  CheckBufs bufs(st);
  const uint16_t* q = bufs.upload(a.qkv);
  void* d_o = bufs.alloc((size_t)T * A::D * 2);
  double worst = 0;
  for (int pass = 0; pass < 2; ++pass) {
    const s1c_status rc = s1c_attention(q, q + A::D, q + 2 * A::D, d_o, A::W, A::W, A::W, A::D, A::H, a.cu.data(), n,
                                        pass == 0 ? -1 : window, 0.125f, impl, st);
    if (rc != S1C_OK) throw S1cError(rc, "load check: attention launch: " + g_create_error);
    std::vector<double> w = want[pass];
    if (plant) w[w.size() / 3] += 1.0;
    const double e = scaled_err(download(d_o, w.size(), false), w);
    if (std::isnan(e)) return e;
    worst = std::max(worst, e);
  }
  return worst;
}

std::string fmt_err(double e) {
  char buf[64];
  std::snprintf(buf, sizeof buf, "%.3g", e);
  return buf;
}

void selfcheck(s1c_backend& B) {
  auto planted = [&](const char* k) {
    const std::string& s = B.check_fail;
    size_t i = 0;
    while (i <= s.size()) {
      size_t j = s.find('+', i);
      if (j == std::string::npos) j = s.size();
      if (s.compare(i, j - i, k) == 0) return true;
      i = j + 1;
    }
    return false;
  };
  const bool pdl = t_pdl;
  t_pdl = false;  // plain stream order between the check's launches and its copies
  struct Restore {
    bool v;
    ~Restore() { t_pdl = v; }
  } restore{pdl};
  cudaStream_t st = B.stream;
  B.check_report.clear();
  auto refuse = [&](const std::string& what, double e) {
    throw S1cError(S1C_ERR_SELFCHECK, "load check: " + what + " differs from the plain computation (max scaled error " +
                                          fmt_err(e) + ", limit " + fmt_err(CHECK_TOL) + ")");
  };
  auto note = [&](const std::string& what, const char* key, const std::string& instead, double e) {
    std::fprintf(stderr, "s1c: %s is off for this load, %s runs instead: max scaled error %s (limit %s)\n",
                 what.c_str(), instead.c_str(), fmt_err(e).c_str(), fmt_err(CHECK_TOL).c_str());
    if (!B.check_report.empty()) B.check_report += "+";
    B.check_report += key;
  };
  const GemmCheck g;
  std::vector<std::vector<double>> gw;
  for (int cs = 0; cs < 6; ++cs) gw.push_back(g.want(cs));
  const AttnCheck ac;
  const std::vector<double> aw[2] = {ac.want(-1), ac.want(B.window)};
  auto gemm = [&](int variant, const char* k) { return check_gemm_kernel(g, gw, st, variant, planted(k)); };
  auto attn = [&](int impl, const char* k) { return check_attention_kernel(ac, aw, B.window, st, impl, planted(k)); };

  const double e1 = gemm(1, "1cta");
  if (!(e1 <= CHECK_TOL)) refuse("the one-CTA GEMM", e1);
  const double am = attn(1, "mma");
  if (!(am <= CHECK_TOL)) refuse("the mma.sync attention", am);
  if (B.gemm_variant == 3) {
    const double es = gemm(3, "splitk");
    if (!(es <= CHECK_TOL)) refuse("the workspace split-K GEMM (forced by gemm=splitk)", es);
  }
  if (B.gemm_variant == 0 || B.gemm_variant == 2) {
    const double e2 = gemm(2, "2cta");
    if (!(e2 <= CHECK_TOL)) {
      if (B.gemm_variant == 2) refuse("the two-CTA GEMM (forced by gemm=2cta)", e2);
      B.gemm_off |= GEMM_OFF_2CTA;
      note("the two-CTA GEMM", "2cta", "the one-CTA GEMM", e2);
    }
  }
  if (B.gemm_variant == 0 || B.gemm_variant == 4) {
    const double ek = gemm(4, "csk");
    if (!(ek <= CHECK_TOL)) {
      if (B.gemm_variant == 4) refuse("the cluster split-K GEMM (forced by gemm=csk)", ek);
      B.gemm_off |= GEMM_OFF_CSK;
      note("the cluster split-K GEMM", "csk", "the one-CTA GEMM", ek);
    }
  }
  if (B.attn_mode != s1c_backend::ATTN_MMA) {
    const double at = attn(0, "tc");
    if (!(at <= CHECK_TOL)) {
      if (B.attn_mode == s1c_backend::ATTN_TC) refuse("the tcgen05 attention (forced by attn=tc)", at);
      B.attn_mode = s1c_backend::ATTN_MMA;
      note("the tcgen05 attention", "tc", "the mma.sync attention", at);
    }
  }
  B.checked = true;
}

// `Backend::active_kernels`: the kernels this handle's forward can launch under its settings and
// load check, and the check's outcome.
void describe_kernels(s1c_backend& B) {
  std::string g;
  switch (B.gemm_variant) {
    case 1: g = "gemm_tcgen05_1cta"; break;
    case 2: g = "gemm_tcgen05_2cta"; break;
    case 3: g = "gemm_tcgen05_1cta_splitk,splitk_finalize"; break;
    case 4: g = "gemm_tcgen05_cluster_splitk"; break;
    default:
      g = "gemm_tcgen05_1cta";
      if (!(B.gemm_off & GEMM_OFF_2CTA)) g += ",gemm_tcgen05_2cta";
      if (!(B.gemm_off & GEMM_OFF_CSK)) g += ",gemm_tcgen05_cluster_splitk";
  }
  std::string s = "epilogues(rope,geglu,residual,bias_act)," + g;
  if (B.attn_mode != s1c_backend::ATTN_MMA) s += ",attention_varlen_tcgen05";
  if (B.attn_mode != s1c_backend::ATTN_TC) s += ",attention_varlen_mma";
  s += ",embed_ln,layernorm,final_to_head,scorer_logits";
  if (B.checked) s += B.check_report.empty() ? ",load_check(passed)" : ",load_check(off:" + B.check_report + ")";
  B.kernels = s;
}

}  // namespace

// =============================================================================================
// Allocation-free split-K GEMM (s1c_gemm_splitk_noalloc)
//
// For callers that must not allocate device memory: the split-K partial sums, the RoPE inverse
// frequencies and the device status word live in file-scope __device__ arrays of fixed size, held
// by every GPU that loads this library until the process exits. Host code cannot use these names
// as device addresses; `noalloc_device` looks the addresses up once per device (cudaGetSymbolAddress,
// with that device current) on the entry point's first call there. All calls share the arrays:
// each call overwrites them, and calls whose work overlaps on the GPU race on them.

constexpr size_t NOALLOC_SCRATCH_FLOATS = (size_t)1 << 20;  // 4 MiB of fp32 partial sums

static __device__ __align__(256) float s1c_noalloc_scratch[NOALLOC_SCRATCH_FLOATS];
static __device__ __align__(256) float s1c_noalloc_inv_freq[32];
static __device__ __align__(256) int s1c_noalloc_status;

// RoPE frequencies of the allocation-free GEMM: the 32 values travel as a kernel argument (copied
// at launch), so no host buffer has to outlive the call.
struct InvFreq32 {
  float v[32];
};
__global__ void noalloc_set_inv_freq_kernel(float* dst, const InvFreq32 f) { dst[threadIdx.x] = f.v[threadIdx.x]; }

namespace {

struct NoAllocDevice {
  bool ready = false;
  float* scratch = nullptr;
  float* inv_freq = nullptr;
  int* status = nullptr;
  int n_sms = 0;
};

NoAllocDevice& noalloc_device(int dev) {
  static NoAllocDevice devs[64];
  static std::mutex mu;
  if (dev < 0 || dev >= 64) throw S1cError(S1C_ERR_ARG, "device ordinal out of range");
  std::lock_guard<std::mutex> g(mu);
  NoAllocDevice& d = devs[dev];
  if (!d.ready) {
    CK(cudaGetSymbolAddress(reinterpret_cast<void**>(&d.scratch), s1c_noalloc_scratch));
    CK(cudaGetSymbolAddress(reinterpret_cast<void**>(&d.inv_freq), s1c_noalloc_inv_freq));
    CK(cudaGetSymbolAddress(reinterpret_cast<void**>(&d.status), s1c_noalloc_status));
    CK(cudaDeviceGetAttribute(&d.n_sms, cudaDevAttrMultiProcessorCount, dev));
    set_all_gemm_smem();
    d.ready = true;
  }
  return d;
}

}  // namespace

// =============================================================================================
// C ABI

extern "C" {

s1c_status s1c_create(const s1c_model_desc* desc, const s1c_tensor* tensors, int32_t n_tensors, int32_t device,
                      s1c_backend** out) {
  return s1c_create_with_settings(desc, tensors, n_tensors, device, nullptr, out);
}

s1c_status s1c_create_with_settings(const s1c_model_desc* desc, const s1c_tensor* tensors, int32_t n_tensors,
                                    int32_t device, const char* settings, s1c_backend** out) {
  g_create_error.clear();
  if (!desc || !out || (n_tensors > 0 && !tensors)) {
    g_create_error = "null argument";
    return S1C_ERR_ARG;
  }
  *out = nullptr;
  std::unique_ptr<s1c_backend> b(new s1c_backend());
  try {
    int n_dev = 0;
    CK(cudaGetDeviceCount(&n_dev));
    if (device < 0 || device >= n_dev) throw S1cError(S1C_ERR_ARG, "no CUDA device " + std::to_string(device));
    CK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
      throw S1cError(S1C_ERR_UNSUPPORTED, std::string("the kernels are built for sm_100a; device is ") + prop.name);
    b->device = device;
    b->num_sms = prop.multiProcessorCount;
    CK(cudaStreamCreateWithFlags(&b->own_stream, cudaStreamNonBlocking));
    b->stream = b->own_stream;
    set_all_gemm_smem();
    CK(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATTC_SMEM));
    apply_settings(*b, settings ? settings : std::getenv("S1C_SETTINGS"));
    build(*b, *desc, tensors, n_tensors);
    CK(cudaDeviceSynchronize());
    if (b->check) selfcheck(*b);
    describe_kernels(*b);
  } catch (const S1cError& e) {
    g_create_error = e.what();
    return e.code;
  } catch (const std::exception& e) {
    g_create_error = e.what();
    return S1C_ERR_ARG;
  }
  *out = b.release();
  return S1C_OK;
}

void s1c_destroy(s1c_backend* b) {
  if (!b) return;
  cudaSetDevice(b->device);
  delete b;
}

const char* s1c_last_error(const s1c_backend* b) { return b ? b->last_error.c_str() : "null backend"; }
const char* s1c_create_error(void) { return g_create_error.c_str(); }
const char* s1c_name(const s1c_backend* b) { return b ? b->name.c_str() : ""; }
const char* s1c_active_kernels(const s1c_backend* b) { return b ? b->kernels.c_str() : ""; }
size_t s1c_padded_len(const s1c_backend*, size_t len, size_t) { return len; }
int64_t s1c_last_launch_count(const s1c_backend* b) { return b ? b->launches : 0; }

s1c_status s1c_set_stream(s1c_backend* b, void* stream) {
  return guarded(b, [&] {
    CK(cudaStreamSynchronize(b->stream));
    b->stream = stream ? static_cast<cudaStream_t>(stream) : b->own_stream;
  });
}

s1c_status s1c_profile(s1c_backend* b, int32_t on) {
  return guarded(b, [&] {
    b->prof_user = on != 0;
    b->prof_on = b->prof_user || b->trace_ops;
    b->prof_stats.clear();
    b->prof_pending.clear();
    b->ev_used = 0;
  });
}

size_t s1c_profile_report(const s1c_backend* b, char* buf, size_t cap) {
  if (!b) return 0;
  std::string out;
  char line[256];
  for (const auto& kv : b->prof_stats) {
    std::snprintf(line, sizeof line, "%s %lld %.6f %.6e %.6e\n", kv.first.c_str(), (long long)kv.second.launches,
                  kv.second.ms, kv.second.flops, kv.second.bytes);
    out += line;
  }
  if (buf && cap) {
    const size_t n = std::min(cap - 1, out.size());
    std::memcpy(buf, out.data(), n);
    buf[n] = 0;
  }
  return out.size() + 1;
}

s1c_status s1c_warmup(s1c_backend* b) {
  return guarded(b, [&] {
    // Forwards per (bucket, warm row count) as the reference's warm_buckets (lib.rs:1152-1173):
    // rows of equal length, once filling the bucket exactly and once leaving room for the dummy
    // rows, each with 2 and with 16 markers (the two marker-slot buckets of up to 16 markers), so
    // the bucket shapes a batch of that many rows can land in have their graphs captured. Without
    // buckets: one short row and one 4-row batch.
    std::vector<std::pair<int, int>> shapes;  // (rows, tokens per row)
    if (b->buckets.empty()) {
      shapes = {{1, 64}, {4, 64}};
    } else {
      for (int t : b->buckets)
        for (int n : b->warm_rows) {
          if (n > BUCKET_MAX_ROWS) continue;
          if (t % n == 0 && t / n >= 3 && t / n <= b->max_pos) shapes.push_back({n, t / n});
          int nb = 2;
          while (nb < n + 1) nb *= 2;
          const int per = (t - (nb - n)) / n;
          if (nb <= BUCKET_MAX_ROWS && per >= 3 && per <= b->max_pos) shapes.push_back({n, per});
        }
    }
    for (auto [n, len] : shapes)
      for (int k : {2, 16}) {
        if (k > len) continue;
        std::vector<int32_t> cu(n + 1);
        for (int r = 0; r <= n; ++r) cu[r] = r * len;
        std::vector<uint32_t> ids((size_t)n * len, 0), mpos((size_t)n * k), qt(n, 0);
        std::vector<int32_t> mc(n, k);
        for (int r = 0; r < n; ++r)
          for (int i = 0; i < k; ++i) mpos[(size_t)r * k + i] = (uint32_t)i;
        s1c_varlen v{n, k, ids.data(), cu.data(), mpos.data(), mc.data(), qt.data()};
        std::vector<float> lg((size_t)n * k), pl((size_t)n * b->d);
        forward_host(*b, v, lg.data(), pl.data(), nullptr);
        if (b->buckets.empty()) break;
      }
  });
}

s1c_status s1c_forward_varlen(s1c_backend* b, const s1c_varlen* in, float* logits, float* pooled, float* hidden) {
  return guarded(b, [&] {
    if (!in || !pooled || (in->n > 0 && in->kmax > 0 && !logits)) throw S1cError(S1C_ERR_ARG, "null argument");
    forward_host(*b, *in, logits, pooled, hidden);
  });
}

s1c_status s1c_forward_padded(s1c_backend* b, const s1c_batch* batch, float* logits, float* pooled) {
  return guarded(b, [&] {
    if (!batch || !pooled || (batch->n > 0 && batch->kmax > 0 && !logits)) throw S1cError(S1C_ERR_ARG, "null argument");
    PackedBatch p;
    pack_batch(*batch, p);
    forward_host(*b, p.v, logits, pooled, nullptr);
  });
}

s1c_status s1c_encoder_hidden(s1c_backend* b, const s1c_batch* batch, float* out) {
  return guarded(b, [&] {
    if (!batch || !out) throw S1cError(S1C_ERR_ARG, "null argument");
    PackedBatch p;
    pack_batch(*batch, p);  // checks the mask against seq_lens
    validate_varlen(*b, p.v);
    // The reference's hook runs the padded layout (lib.rs:1865-1878): a padding position is the
    // batch's padding id at its padded index, attending its row's real keys through the -1e4 key
    // mask; real positions never attend it. Here each row runs its real tokens and then padding
    // tokens as queries whose key range is the row's real tokens. A padding position farther than
    // the window from every real token sees only masked keys in the reference's sliding-window
    // layers (a softmax over -1e4 entries); those positions are not computed and stay 0.
    const bool any_local = std::find(b->local.begin(), b->local.end(), 1) != b->local.end();
    const size_t n = batch->n, len = batch->len, d = b->d;
    PackedBatch q;
    std::vector<int> real(n), keep(n);
    q.cu.assign(1, 0);
    for (size_t r = 0; r < n; ++r) {
      const size_t sl = batch->seq_lens[r];
      real[r] = (int)sl;
      keep[r] = (int)(any_local ? std::min(len, sl + (size_t)b->window) : len);
      q.ids.insert(q.ids.end(), batch->input_ids + r * len, batch->input_ids + r * len + keep[r]);
      q.cu.push_back((int32_t)q.ids.size());
    }
    q.mcount = p.mcount;
    q.qtype = p.qtype;
    q.mpos = p.mpos;
    q.v = s1c_varlen{(int32_t)n, (int32_t)batch->kmax, q.ids.data(), q.cu.data(), q.mpos.data(), q.mcount.data(),
                     q.qtype.data()};
    std::vector<float> lg(n * batch->kmax), pl(n * d), hid(q.ids.size() * d);
    if (n) forward_host(*b, q.v, lg.data(), pl.data(), hid.data(), real.data());
    std::memset(out, 0, n * len * d * sizeof(float));
    for (size_t r = 0; r < n; ++r)
      std::memcpy(out + r * len * d, hid.data() + (size_t)q.cu[r] * d, (size_t)keep[r] * d * sizeof(float));
  });
}

s1c_status s1c_forward_device_async(s1c_backend* b, const s1c_varlen* in, const uint32_t* d_ids, float* d_logits,
                                    float* d_pooled, float* d_hidden) {
  return guarded(b, [&] {
    if (!in || !d_ids || !d_pooled || (in->n > 0 && in->kmax > 0 && !d_logits))
      throw S1cError(S1C_ERR_ARG, "null argument");
    forward_device(*b, *in, d_ids, d_logits, d_pooled, d_hidden);
  });
}

s1c_status s1c_synchronize(s1c_backend* b) {
  return guarded(b, [&] { check_status(*b); });
}

s1c_status s1c_forward_device(s1c_backend* b, const s1c_varlen* in, const uint32_t* d_ids, float* d_logits,
                              float* d_pooled, float* d_hidden) {
  return guarded(b, [&] {
    if (!in || !d_ids || !d_pooled || (in->n > 0 && in->kmax > 0 && !d_logits))
      throw S1cError(S1C_ERR_ARG, "null argument");
    forward_device(*b, *in, d_ids, d_logits, d_pooled, d_hidden);
    check_status(*b);
  });
}

s1c_status s1c_gemm(int32_t epi, const void* d_A, const void* d_B, void* d_out, int32_t M, int32_t N, int32_t K,
                    const float* d_bias, int32_t act, int32_t out_f32, const int32_t* d_pos, float rope_theta,
                    int32_t rope_cols, int32_t out_cols, int32_t variant, void* stream) {
  static std::mutex mu;
  static std::map<std::pair<int, float>, float*> tables;  // (device, theta) -> inverse frequencies
  static int* d_status_dummy[64] = {nullptr};
  try {
    if (!d_A || !d_B || !d_out || M <= 0 || N <= 0 || K <= 0 || K % 8 || N % 32)
      throw S1cError(S1C_ERR_ARG, "bad GEMM arguments (K must be a multiple of 8, N of 32)");
    int dev = 0, n_sms = 0;
    CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw S1cError(S1C_ERR_ARG, "device index out of range");
    CK(cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, dev));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    GemmArgs a{};
    a.M = M; a.N = N; a.K = K; a.bias = d_bias; a.act = act; a.out_f32 = out_f32;
    a.pos = d_pos; a.rope_cols = rope_cols; a.out_cols = out_cols;
    {
      std::lock_guard<std::mutex> g(mu);
      static bool smem_set[64] = {false};
      if (!smem_set[dev]) { set_all_gemm_smem(); smem_set[dev] = true; }
      if (!d_status_dummy[dev]) {
        CK(cudaMalloc(&d_status_dummy[dev], sizeof(int)));
        CK(cudaMemset(d_status_dummy[dev], 0, sizeof(int)));
        CK(cudaDeviceSynchronize());  // zeroed before any kernel on the caller's stream writes it
      }
      a.status = d_status_dummy[dev];
      if (epi == EPI_ROPE) {
        auto key = std::make_pair(dev, rope_theta);
        if (!tables.count(key)) tables[key] = make_inv_freq_raw(rope_theta);
        a.inv_freq = tables[key];
        static std::map<std::pair<int, float>, float*> rtabs;  // cos | sin tables, positions < 8192
        if (!rtabs.count(key)) rtabs[key] = make_rope_table_raw(tables[key], 8192);
        a.rope_tab = rtabs[key];
        if (!d_pos) throw S1cError(S1C_ERR_ARG, "RoPE needs positions");
      }
    }
    const bool f32 = epi == EPI_RESID || (epi == EPI_STORE && out_f32);
    const int out_w = (epi == EPI_GEGLU) ? out_cols : N;
    const CUtensorMap ta = make_tmap(d_A, (uint64_t)M, K, K, GEMM_BM);
    if (variant < 0 || variant > 5) throw S1cError(S1C_ERR_ARG, "variant must be 0 to 5");
    if (variant == 5 && epi == EPI_GEGLU) throw S1cError(S1C_ERR_ARG, "GeGLU tiles are 256 wide (variant 5 does not apply)");
    const WeightMap tb = make_wmap(d_B, N, K, K);
    const CUtensorMap tc = epi == EPI_RESID16 ? make_out_tmap_f16(d_out, (uint64_t)M, out_w, out_w)
                                              : make_out_tmap(d_out, f32, (uint64_t)M, out_w, out_w);
    // Split-K workspace of this entry point: one 32 MB buffer per device, kept for the process.
    static float* ws_dev[64] = {nullptr};
    {
      std::lock_guard<std::mutex> g(mu);
      if (!ws_dev[dev]) CK(cudaMalloc(&ws_dev[dev], (size_t)32 << 20));
    }
    const SplitCtx sk{ws_dev[dev], (size_t)32 << 20, d_out, out_w};
    switch (epi) {
      case EPI_STORE: launch_gemm<EPI_STORE>(ta, tb, tc, a, n_sms, st, variant, &sk); break;
      case EPI_ROPE: launch_gemm<EPI_ROPE>(ta, tb, tc, a, n_sms, st, variant, &sk); break;
      case EPI_GEGLU: launch_gemm<EPI_GEGLU>(ta, tb, tc, a, n_sms, st, variant, &sk); break;
      case EPI_RESID: launch_gemm<EPI_RESID>(ta, tb, tc, a, n_sms, st, variant, &sk); break;
      case EPI_RESID16: launch_gemm<EPI_RESID16>(ta, tb, tc, a, n_sms, st, variant, &sk); break;
      default: throw S1cError(S1C_ERR_ARG, "unknown epilogue");
    }
    return S1C_OK;
  } catch (const S1cError& e) {
    g_create_error = e.what();
    return e.code;
  } catch (const std::exception& e) {
    g_create_error = e.what();
    return S1C_ERR_ARG;
  }
}

s1c_status s1c_attention(const void* d_q, const void* d_k, const void* d_v, void* d_o, int32_t q_stride,
                         int32_t k_stride, int32_t v_stride, int32_t o_stride, int32_t heads,
                         const int32_t* cu_seqlens, int32_t n, int32_t window, float scale, int32_t impl,
                         void* stream) {
  // Metadata buffers of this entry point: one per device, grown on demand and kept for the
  // process (calls are serialised by the lock; each call waits for its kernel before returning).
  struct AttnScratch {
    int* d_cu = nullptr;
    int4* d_items = nullptr;
    int* d_status = nullptr;
    size_t cu_cap = 0, items_cap = 0;
  };
  static std::mutex mu;
  static AttnScratch scratch[64];
  std::lock_guard<std::mutex> guard(mu);
  try {
    if (!d_q || !d_k || !d_v || !d_o || !cu_seqlens || n <= 0 || heads <= 0 || (impl != 0 && impl != 1))
      throw S1cError(S1C_ERR_ARG, "bad attention arguments");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int dev = 0;
    CK(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) throw S1cError(S1C_ERR_ARG, "device index out of range");
    AttnScratch& sc = scratch[dev];
    const int qtile = impl == 0 ? ATTC_BQ : ATT_BQ;
    std::vector<int4> items;
    for (int r = 0; r < n; ++r) {
      const int base = cu_seqlens[r], len = cu_seqlens[r + 1] - base;
      for (int q = 0; q < len; q += qtile) items.push_back(make_int4(r, base + q, std::min(qtile, len - q), 0));
    }
    longest_first(items, cu_seqlens);
    const int T = cu_seqlens[n];
    if (sc.cu_cap < (size_t)n + 1) {
      if (sc.d_cu) CK(cudaFree(sc.d_cu));
      sc.d_cu = nullptr;
      sc.cu_cap = 0;
      CK(cudaMalloc(&sc.d_cu, ((size_t)n + 1) * 4));
      sc.cu_cap = (size_t)n + 1;
    }
    if (sc.items_cap < items.size()) {
      if (sc.d_items) CK(cudaFree(sc.d_items));
      sc.d_items = nullptr;
      sc.items_cap = 0;
      CK(cudaMalloc(&sc.d_items, items.size() * 16));
      sc.items_cap = items.size();
    }
    if (!sc.d_status) CK(cudaMalloc(&sc.d_status, sizeof(int)));
    int* d_cu = sc.d_cu;
    int4* d_items = sc.d_items;
    CK(cudaMemcpyAsync(d_cu, cu_seqlens, ((size_t)n + 1) * 4, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(d_items, items.data(), items.size() * 16, cudaMemcpyHostToDevice, st));
    const float scale_log2 = scale * 1.4426950408889634f;
    if (impl == 0) {
      // one map for Q, one for K and V together: V must sit in K's rows at a 64-aligned column
      const ptrdiff_t dv = static_cast<const bf16*>(d_v) - static_cast<const bf16*>(d_k);
      if (v_stride != k_stride || dv < 0 || dv % 64 || dv + heads * 64 > k_stride)
        throw S1cError(S1C_ERR_ARG, "tcgen05 attention needs v in the rows of k (same pitch, 64-aligned column)");
      static bool attr_set[64] = {false};
      if (!attr_set[dev]) {
        CK(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ATTC_SMEM));
        attr_set[dev] = true;
      }
      int* d_status = sc.d_status;
      CK(cudaMemsetAsync(d_status, 0, sizeof(int), st));
      const CUtensorMap tq = make_tmap(d_q, T, heads * 64, q_stride, ATTC_BQ);
      const CUtensorMap tkv = make_tmap(d_k, T, dv + heads * 64, k_stride, ATTC_BK);
      AttnTcArgs a{d_cu, d_items, static_cast<bf16*>(d_o), o_stride, 0, 0, (int)dv, heads, window, scale_log2, d_status,
                   (int)items.size()};
      int n_sms = 0;
      CK(cudaDeviceGetAttribute(&n_sms, cudaDevAttrMultiProcessorCount, dev));
      const dim3 grid((unsigned)attc_grid((int)items.size(), heads, n_sms));
      launch_k(attention_tc_kernel, grid, dim3(ATTC_THREADS), ATTC_SMEM, st, tq, tkv, a);
      cudaError_t e = cudaGetLastError();
      cudaError_t e2 = cudaStreamSynchronize(st);
      int hs = 0;
      if (e2 == cudaSuccess) cudaMemcpy(&hs, d_status, sizeof(int), cudaMemcpyDeviceToHost);
      if (e != cudaSuccess) throw S1cError(S1C_ERR_CUDA, cudaGetErrorString(e));
      if (e2 != cudaSuccess) throw S1cError(S1C_ERR_CUDA, cudaGetErrorString(e2));
      if (hs) throw S1cError(S1C_ERR_DEVICE_TIMEOUT, "device-side wait ran out (code " + std::to_string(hs) + ")");
    } else {
      AttnArgs a{static_cast<const bf16*>(d_q), static_cast<const bf16*>(d_k), static_cast<const bf16*>(d_v),
                 static_cast<bf16*>(d_o), q_stride, k_stride, v_stride, o_stride, d_cu, d_items, window, scale_log2,
                 heads};
      launch_k(attention_varlen_kernel, dim3((unsigned)items.size() * heads), dim3(ATT_THREADS), 0, st, a);
      cudaError_t e = cudaGetLastError();
      cudaError_t e2 = cudaStreamSynchronize(st);
      if (e != cudaSuccess) throw S1cError(S1C_ERR_CUDA, cudaGetErrorString(e));
      if (e2 != cudaSuccess) throw S1cError(S1C_ERR_CUDA, cudaGetErrorString(e2));
    }
    return S1C_OK;
  } catch (const S1cError& e) {
    g_create_error = e.what();
    return e.code;
  }
}

// Self-test of the bounded device waits: an mbarrier that nothing completes, waited on by one
// thread (mbar_wait, the producer / MMA form) and by one warp (mbar_wait_warp, the epilogue form)
// with a short budget. Each wait must give up, record its code in its status word and return, so
// the kernel ends and the context stays usable. Touches nothing but its four result words.
__global__ void wait_timeout_selftest_kernel(int* out, uint64_t budget_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool done = mbar_wait(&bar, 0, out + 0, DEV_TIMEOUT_PRODUCER, nullptr, budget_ns);
    out[2] = done ? 1 : 0;
  } else if (threadIdx.x >= 32) {
    const bool done = mbar_wait_warp(&bar, 0, out + 1, DEV_TIMEOUT_EPILOGUE, nullptr, budget_ns);
    if (threadIdx.x == 32) out[3] = done ? 1 : 0;
  }
}

s1c_status s1c_selftest_wait_timeout(int32_t device, int64_t budget_ns, int32_t* codes) {
  try {
    if (!codes || budget_ns < 1000000 || budget_ns > 2000000000)
      throw S1cError(S1C_ERR_ARG, "budget_ns must lie in [1e6, 2e9] and codes must not be null");
    CK(cudaSetDevice(device));
    int* d_out = nullptr;
    CK(cudaMalloc(&d_out, 4 * sizeof(int)));
    cudaError_t e = cudaMemset(d_out, 0, 4 * sizeof(int));
    if (e == cudaSuccess) {
      wait_timeout_selftest_kernel<<<1, 64>>>(d_out, (uint64_t)budget_ns);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(codes, d_out, 4 * sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(d_out);
    if (e != cudaSuccess) throw S1cError(S1C_ERR_CUDA, cudaGetErrorString(e));
    return S1C_OK;
  } catch (const S1cError& e) {
    g_create_error = e.what();
    return e.code;
  }
}

s1c_status s1c_gemm_splitk_noalloc(int32_t epi, const void* d_A, const void* d_B, void* d_out, int32_t M, int32_t N,
                                   int32_t K, const float* d_bias, int32_t act, int32_t out_f32, const int32_t* d_pos,
                                   float rope_theta, int32_t rope_cols, int32_t out_cols, void* stream) {
  try {
    if (!d_A || !d_B || !d_out || M <= 0 || N <= 0 || K <= 0 || K % 8 || N % 32 || epi < EPI_STORE || epi > EPI_RESID)
      throw S1cError(S1C_ERR_ARG, "bad GEMM arguments (K must be a multiple of 8, N of 32)");
    if (epi == EPI_ROPE && !d_pos) throw S1cError(S1C_ERR_ARG, "RoPE needs positions");
    if ((K + GEMM_BK - 1) / GEMM_BK < 2) throw S1cError(S1C_ERR_ARG, "split-K needs K > 64");
    const size_t rows = (size_t)(M + GEMM_BM - 1) / GEMM_BM * GEMM_BM;
    const size_t scratch_bytes = NOALLOC_SCRATCH_FLOATS * sizeof(float);
    if (2 * rows * (size_t)N * 4 > scratch_bytes)
      throw S1cError(S1C_ERR_ARG, "s1c_gemm_splitk_noalloc: two split slices of " + std::to_string(rows) + " x " +
                                      std::to_string(N) + " fp32 exceed the " + std::to_string(scratch_bytes >> 20) +
                                      " MiB static scratch (rows rounded up to 128; need 2 * rows * N * 4 bytes)");
    int dev = 0;
    CK(cudaGetDevice(&dev));
    NoAllocDevice& nd = noalloc_device(dev);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    CK(cudaMemsetAsync(nd.status, 0, sizeof(int), st));
    GemmArgs a{};
    a.M = M; a.N = N; a.K = K; a.bias = d_bias; a.act = act; a.out_f32 = out_f32;
    a.pos = d_pos; a.rope_cols = rope_cols; a.out_cols = out_cols; a.status = nd.status;
    if (epi == EPI_ROPE) {
      InvFreq32 inv;
      const float lbase = std::log2(rope_theta);
      for (int i = 0; i < 32; ++i) inv.v[i] = std::exp2(-((float)i / 32.0f) * lbase);
      noalloc_set_inv_freq_kernel<<<1, 32, 0, st>>>(nd.inv_freq, inv);
      CK(cudaGetLastError());
      a.inv_freq = nd.inv_freq;
    }
    const bool f32 = epi == EPI_RESID || (epi == EPI_STORE && out_f32);
    const int out_w = (epi == EPI_GEGLU) ? out_cols : N;
    const CUtensorMap ta = make_tmap(d_A, (uint64_t)M, K, K, GEMM_BM);
    const WeightMap tb = make_wmap(d_B, N, K, K);
    const CUtensorMap tc = make_out_tmap(d_out, f32, (uint64_t)M, out_w, out_w);
    const SplitCtx sk{nd.scratch, scratch_bytes, d_out, out_w};
    t_pdl = false;
    switch (epi) {
      case EPI_STORE: launch_gemm<EPI_STORE>(ta, tb, tc, a, nd.n_sms, st, 3, &sk); break;
      case EPI_ROPE: launch_gemm<EPI_ROPE>(ta, tb, tc, a, nd.n_sms, st, 3, &sk); break;
      case EPI_GEGLU: launch_gemm<EPI_GEGLU>(ta, tb, tc, a, nd.n_sms, st, 3, &sk); break;
      case EPI_RESID: launch_gemm<EPI_RESID>(ta, tb, tc, a, nd.n_sms, st, 3, &sk); break;
    }
    return S1C_OK;
  } catch (const S1cError& e) {
    g_create_error = e.what();
    return e.code;
  } catch (const std::exception& e) {
    g_create_error = e.what();
    return S1C_ERR_ARG;
  }
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Checkpoint files

struct s1c_weights {
  s1c::st::File file;
  std::string dir;
};

extern "C" {

s1c_status s1c_weights_open(const char* model_dir, s1c_weights** out) {
  g_create_error.clear();
  if (!model_dir || !out) {
    g_create_error = "null argument";
    return S1C_ERR_ARG;
  }
  *out = nullptr;
  const std::string dir(model_dir);
  const std::string path = dir + ((dir.empty() || dir.back() == '/') ? "" : "/") + "model.safetensors";
  struct stat sb;
  if (stat(path.c_str(), &sb) != 0 || !S_ISREG(sb.st_mode)) {
    g_create_error = "'model.safetensors' not found in " + dir;
    return S1C_ERR_WEIGHTS;
  }
  std::unique_ptr<s1c_weights> w(new s1c_weights());
  w->dir = dir;
  try {
    w->file.open(path);
  } catch (const std::exception& e) {
    g_create_error = path + " (" + std::to_string((unsigned long long)sb.st_size) +
                     " bytes) is truncated or not a safetensors file: " + e.what();
    return S1C_ERR_WEIGHTS;
  }
  *out = w.release();
  return S1C_OK;
}

void s1c_weights_close(s1c_weights* w) { delete w; }

int32_t s1c_weights_count(const s1c_weights* w) { return w ? (int32_t)w->file.tensors().size() : 0; }

int32_t s1c_weights_find(const s1c_weights* w, const char* name) {
  if (!w || !name) return -1;
  const auto& ts = w->file.tensors();
  for (size_t i = 0; i < ts.size(); ++i)
    if (ts[i].name == name) return (int32_t)i;
  return -1;
}

s1c_status s1c_weights_tensor(const s1c_weights* w, int32_t i, s1c_tensor* out) {
  g_create_error.clear();
  if (!w || !out || i < 0 || (size_t)i >= w->file.tensors().size()) {
    g_create_error = "tensor index out of range";
    return S1C_ERR_ARG;
  }
  const s1c::st::Tensor& t = w->file.tensors()[(size_t)i];
  int32_t dt;
  if (t.dtype == "F32") dt = S1C_DT_F32;
  else if (t.dtype == "F16") dt = S1C_DT_F16;
  else if (t.dtype == "BF16") dt = S1C_DT_BF16;
  else if (t.dtype == "F64") dt = S1C_DT_F64;
  else {
    g_create_error = t.name + ": unsupported dtype " + t.dtype;
    return S1C_ERR_WEIGHTS;
  }
  if (t.shape.size() > 4) {
    g_create_error = t.name + ": more than 4 dimensions";
    return S1C_ERR_WEIGHTS;
  }
  out->name = t.name.c_str();
  out->dtype = dt;
  out->ndim = (int32_t)t.shape.size();
  for (int d = 0; d < 4; ++d) out->shape[d] = d < out->ndim ? t.shape[(size_t)d] : 0;
  out->data = w->file.data(t);
  return S1C_OK;
}

s1c_status s1c_weights_verify(const s1c_weights* w) {
  g_create_error.clear();
  if (!w) {
    g_create_error = "null argument";
    return S1C_ERR_ARG;
  }
  for (const char* prefix : {"encoder.", "type_emb.", "scorer.", "act_head."}) {
    bool found = false;
    for (const auto& t : w->file.tensors())
      if (t.name.compare(0, std::strlen(prefix), prefix) == 0) {
        found = true;
        break;
      }
    if (!found) {
      g_create_error = std::string("checkpoint is missing '") + prefix +
                       "' parameters; expected an RL Agent decision model";
      return S1C_ERR_WEIGHTS;
    }
  }
  return S1C_OK;
}

s1c_status s1c_create_from_weights(const s1c_model_desc* desc, const s1c_weights* w, int32_t device,
                                   s1c_backend** out) {
  g_create_error.clear();
  if (!desc || !w || !out) {
    g_create_error = "null argument";
    return S1C_ERR_ARG;
  }
  std::vector<s1c_tensor> ts;
  for (int32_t i = 0; i < s1c_weights_count(w); ++i) {
    s1c_tensor t;
    if (s1c_weights_tensor(w, i, &t) == S1C_OK) ts.push_back(t);  // integer tensors are not weights
  }
  return s1c_create(desc, ts.data(), (int32_t)ts.size(), device, out);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Serving

struct s1c_server {
  s1c::srv::Server srv;
};

namespace {

s1c_status backend_forward(void* ctx, const s1c_varlen* v, float* logits, float* pooled, const char** err) {
  s1c_backend* b = static_cast<s1c_backend*>(ctx);
  const s1c_status st = s1c_forward_varlen(b, v, logits, pooled, nullptr);
  if (st != S1C_OK && err) *err = s1c_last_error(b);
  return st;
}

s1c_status server_start(s1c_server_forward_fn fn, void* const* ctx, int32_t n, int32_t hidden,
                        const s1c_server_opts* opts, s1c_server** out) {
  g_create_error.clear();
  if (!fn || !ctx || n <= 0 || hidden <= 0 || !out) {
    g_create_error = "bad server arguments";
    return S1C_ERR_ARG;
  }
  *out = nullptr;
  std::unique_ptr<s1c_server> s(new s1c_server());
  s1c::srv::Server& v = s->srv;
  v.fn = fn;
  v.ctx.assign(ctx, ctx + n);
  v.hidden = hidden;
  if (opts) v.opts = *opts;
  if (v.opts.max_concurrent <= 0) v.opts.max_concurrent = 16;
  if (v.opts.max_batch_tokens <= 0) v.opts.max_batch_tokens = 16384;
  if (v.opts.max_batch_rows <= 0) v.opts.max_batch_rows = 1024;
  if (v.opts.linger_us < 0) v.opts.linger_us = 0;
  try {
    for (int32_t w = 0; w < n; ++w) {
      ++v.alive;
      try {
        v.workers.emplace_back([&v, w] { v.run(w); });
      } catch (...) {
        --v.alive;
        throw;
      }
    }
  } catch (const std::exception& e) {
    {
      std::lock_guard<std::mutex> lk(v.mu);
      v.stopping = true;
    }
    v.cv_work.notify_all();
    for (auto& t : v.workers) t.join();
    g_create_error = std::string("cannot start the workers: ") + e.what();
    return S1C_ERR_ARG;
  }
  *out = s.release();
  return S1C_OK;
}

}  // namespace

extern "C" {

s1c_status s1c_server_create(s1c_backend* const* backends, int32_t n, const s1c_server_opts* opts, s1c_server** out) {
  if (!backends || n <= 0) {
    g_create_error = "no backends";
    return S1C_ERR_ARG;
  }
  int hidden = 0;
  for (int32_t i = 0; i < n; ++i) {
    if (!backends[i]) {
      g_create_error = "null backend";
      return S1C_ERR_ARG;
    }
    if (i > 0 && backends[i]->d != hidden) {
      g_create_error = "backends of different hidden sizes";
      return S1C_ERR_ARG;
    }
    hidden = backends[i]->d;
  }
  return server_start(backend_forward, reinterpret_cast<void* const*>(backends), n, hidden, opts, out);
}

s1c_status s1c_server_create_with(s1c_server_forward_fn fn, void* const* ctx, int32_t n_workers, int32_t hidden,
                                  const s1c_server_opts* opts, s1c_server** out) {
  return server_start(fn, ctx, n_workers, hidden, opts, out);
}

s1c_status s1c_server_submit(s1c_server* s, const s1c_request* req, uint64_t* ticket) {
  g_create_error.clear();
  if (!s || !req || !ticket) {
    g_create_error = "null argument";
    return S1C_ERR_ARG;
  }
  s1c::srv::Server& v = s->srv;
  std::unique_lock<std::mutex> lk(v.mu);
  if ((int32_t)v.jobs.size() >= v.opts.max_concurrent) {
    ++v.stats.busy_rejections;
    g_create_error = "server busy, try again later";
    return S1C_ERR_BUSY;
  }
  if (v.stopping || v.alive.load() == 0) {
    g_create_error = "inference worker is not running";
    return S1C_ERR_DEAD;
  }
  if (req->len <= 0 || !req->ids || (req->n_markers > 0 && !req->marker_pos) || req->n_markers < 0) {
    g_create_error = "malformed request: empty row or missing marker positions";
    return S1C_ERR_ARG;
  }
  for (int32_t k = 0; k < req->n_markers; ++k)
    if (req->marker_pos[k] >= (uint32_t)req->len) {
      g_create_error = "malformed request: marker position " + std::to_string(req->marker_pos[k]) +
                       " outside a row of " + std::to_string(req->len) + " tokens";
      return S1C_ERR_ARG;
    }
  auto j = std::make_shared<s1c::srv::Job>();
  j->id = v.next_id++;
  j->ids.assign(req->ids, req->ids + req->len);
  if (req->n_markers > 0) j->markers.assign(req->marker_pos, req->marker_pos + req->n_markers);
  j->qtype = req->qtype;
  v.jobs[j->id] = j;
  v.queue.push_back(j);
  *ticket = j->id;
  lk.unlock();
  v.cv_work.notify_one();
  return S1C_OK;
}

s1c_status s1c_server_wait(s1c_server* s, uint64_t ticket, int32_t timeout_ms, float* logits, float* pooled,
                           float* infer_ms) {
  g_create_error.clear();
  if (!s) {
    g_create_error = "null argument";
    return S1C_ERR_ARG;
  }
  s1c::srv::Server& v = s->srv;
  std::unique_lock<std::mutex> lk(v.mu);
  auto it = v.jobs.find(ticket);
  if (it == v.jobs.end()) {
    g_create_error = "unknown ticket " + std::to_string(ticket);
    return S1C_ERR_ARG;
  }
  std::shared_ptr<s1c::srv::Job> j = it->second;
  if (timeout_ms < 0) {
    v.cv_done.wait(lk, [&] { return j->done; });
  } else if (!v.cv_done.wait_for(lk, std::chrono::milliseconds(timeout_ms), [&] { return j->done; })) {
    g_create_error = "result not ready";
    return S1C_ERR_TIMEOUT;
  }
  v.jobs.erase(ticket);
  if (j->status != S1C_OK) {
    g_create_error = j->error;
    return j->status;
  }
  if (logits && !j->logits.empty()) std::memcpy(logits, j->logits.data(), j->logits.size() * sizeof(float));
  if (pooled) std::memcpy(pooled, j->pooled.data(), j->pooled.size() * sizeof(float));
  if (infer_ms) *infer_ms = (float)j->infer_ms;
  return S1C_OK;
}

s1c_status s1c_server_cancel(s1c_server* s, uint64_t ticket) {
  g_create_error.clear();
  if (!s) {
    g_create_error = "null argument";
    return S1C_ERR_ARG;
  }
  s1c::srv::Server& v = s->srv;
  std::lock_guard<std::mutex> lk(v.mu);
  auto it = v.jobs.find(ticket);
  if (it == v.jobs.end()) {
    g_create_error = "unknown ticket " + std::to_string(ticket);
    return S1C_ERR_ARG;
  }
  it->second->cancelled = true;
  v.jobs.erase(it);
  return S1C_OK;
}

s1c_status s1c_server_get_stats(s1c_server* s, s1c_server_stats* out) {
  if (!s || !out) return S1C_ERR_ARG;
  s1c::srv::Server& v = s->srv;
  std::lock_guard<std::mutex> lk(v.mu);
  *out = v.stats;
  out->in_flight = (int32_t)v.jobs.size();
  int32_t q = 0;
  for (auto& j : v.queue) q += j->cancelled ? 0 : 1;
  out->queued = q;
  out->workers_alive = v.alive.load();
  return S1C_OK;
}

void s1c_server_stop(s1c_server* s) {
  if (!s) return;
  s1c::srv::Server& v = s->srv;
  {
    std::lock_guard<std::mutex> lk(v.mu);
    if (v.stopping && v.workers.empty()) return;
    v.stopping = true;
    v.fail_queued_locked("inference worker is not running");
  }
  v.cv_work.notify_all();
  v.cv_done.notify_all();
  for (auto& t : v.workers)
    if (t.joinable()) t.join();
  v.workers.clear();
  v.cv_done.notify_all();
}

void s1c_server_destroy(s1c_server* s) {
  if (!s) return;
  s1c_server_stop(s);
  delete s;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Decode

extern "C" s1c_status s1c_decode(const float* logits, const float* pooled, int32_t n, int32_t kmax, int32_t hidden,
                                 const int32_t* marker_count, const uint32_t* qtype, const double* temperature,
                                 const s1c_act_head* head, double* probs, s1c_answer* out) {
  g_create_error.clear();
  if (n < 0 || kmax < 0 || hidden <= 0 || !head || !out || (n > 0 && (!logits || !pooled || !marker_count ||
                                                                      !qtype || !temperature))) {
    g_create_error = "bad decode arguments";
    return S1C_ERR_ARG;
  }
  const s1c_act_head& h = *head;
  if (h.d_in <= 4) {
    g_create_error = "act_head.0.weight has input width " + std::to_string(h.d_in) +
                     ", but the action head reads the pooled hidden state plus 4 scalar features, so it needs at least 5";
    return S1C_ERR_WEIGHTS;
  }
  if (h.d_in - 4 != hidden) {
    g_create_error = "act_head.0.weight has input width " + std::to_string(h.d_in) +
                     ", which is not the encoder hidden size " + std::to_string(hidden) + " plus 4 scalar features";
    return S1C_ERR_WEIGHTS;
  }
  if (h.hidden <= 0 || h.n_act <= 0 || !h.w0 || !h.b0 || !h.w2 || !h.b2) {
    g_create_error = "act_head has an empty layer";
    return S1C_ERR_WEIGHTS;
  }
  for (int32_t r = 0; r < n; ++r) {
    const int k = marker_count[r];
    if (k < 0 || k > kmax || qtype[r] > 2 || !(temperature[r] > 0.0) || !std::isfinite(temperature[r])) {
      g_create_error = "row " + std::to_string(r) + ": marker_count, qtype or temperature out of range";
      return S1C_ERR_ARG;
    }
    const float* row = logits + (size_t)r * kmax;
    std::vector<double> z((size_t)k);
    for (int i = 0; i < k; ++i) z[(size_t)i] = (double)row[i] / temperature[r];
    const std::vector<double> p = s1c::dec::softmax_f64(z);
    s1c_answer a{};
    a.qtype = (int32_t)qtype[r];
    a.k = k;
    int am = 0;
    for (int i = 1; i < k; ++i)
      if (p[(size_t)i] > p[(size_t)am]) am = i;
    a.argmax = am;
    const double conf = s1c::dec::confidence_from_probs(p, k);
    if (qtype[r] == 0) {
      a.confidence = conf;
      a.answer_confidence = k > 0 ? p[(size_t)am] : 0.0;
    } else if (qtype[r] == 1) {
      double es = 0.0, top = 0.0;
      for (int i = 0; i < k; ++i) {
        es += (double)i * p[(size_t)i];
        top = std::max(top, p[(size_t)i]);
      }
      a.score = es;
      a.confidence = conf;
      a.answer_confidence = top;
    } else {
      const double p1 = k > 1 ? p[1] : 0.0;
      a.noul = p1;
      a.confidence = a.answer_confidence = std::max(p1, 1.0 - p1);
    }
    float feats[4];
    s1c::dec::act_features(row, kmax, k, feats);
    a.act_probability = s1c::dec::act_probs(h, pooled + (size_t)r * hidden, feats)[0];
    out[r] = a;
    if (probs)
      for (int i = 0; i < kmax; ++i) probs[(size_t)r * kmax + i] = i < k ? p[(size_t)i] : 0.0;
  }
  return S1C_OK;
}
