// Shared device helpers for the sm_100a kernels of libs1c: bf16 packing, mbarriers with
// bounded waits, TMA tile loads (no cluster forms), and the tcgen05 (5th-gen tensor core)
// instructions with their shared-memory / instruction descriptors.
//
// Every spin-wait here is bounded by wall time (%globaltimer). A wait that runs out writes an
// error code into the device status word the host reads after each forward and returns
// false; callers then stop issuing work and fall through to their teardown, so a logic error
// surfaces as S1C_ERR_DEVICE_TIMEOUT instead of a hung GPU.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define S1C_DEV __device__ __forceinline__

namespace s1c {

// Device status codes (first error wins; 0 = ok). The host maps any non-zero value to
// S1C_ERR_DEVICE_TIMEOUT with the code in the error text.
enum DevStatus : int {
  DEV_OK = 0,
  DEV_TIMEOUT_PRODUCER = 1,
  DEV_TIMEOUT_MMA_FULL = 2,
  DEV_TIMEOUT_MMA_TEMPTY = 3,
  DEV_TIMEOUT_EPILOGUE = 4,
  DEV_TIMEOUT_DRAIN = 5,
  DEV_BAD_INDEX = 6,
};

// Wall-clock budget of one wait, in ns. A tile of the largest GEMM takes microseconds.
#ifndef S1C_WAIT_BUDGET_NS
#define S1C_WAIT_BUDGET_NS 2000000000ull
#endif

S1C_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

S1C_DEV void report(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialisation may start
// while its predecessor on the stream finishes. `pdl_trigger` lets this kernel's own successor be
// scheduled early; `pdl_wait` blocks until every predecessor has completed and its memory is
// visible. Each kernel calls `pdl_wait` before its first access to global memory that an earlier
// kernel of the forward reads or writes. Both are no-ops for a kernel launched without the attribute.
S1C_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
S1C_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

S1C_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------
// bf16 helpers
S1C_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
S1C_DEV float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
S1C_DEV float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// f16 helpers (the encoder's residual stream)
S1C_DEV uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
S1C_DEV float2 unpack_f16x2(uint32_t v) { return __half22float2(*reinterpret_cast<__half2*>(&v)); }

// ---------------------------------------------------------------------------------------
// mbarrier
S1C_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
S1C_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
S1C_DEV void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
S1C_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
S1C_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
S1C_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase with the given parity to complete; false when the wait budget ran out
// (the status word then holds `code`) or another role already gave up (`abort` set).
S1C_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code, volatile int* abort,
                       uint64_t budget_ns = S1C_WAIT_BUDGET_NS) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(a, parity)) return true;
    if ((it & 63u) == 0) {
      if (abort && *abort) return false;
      if (globaltimer() - t0 > budget_ns) {
        report(status, code);
        if (abort) *abort = 1;
        return false;
      }
    }
  }
}

// Warp-collective bounded wait: every lane polls, the warp leaves together.
S1C_DEV bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* status, int code, volatile int* abort,
                            uint64_t budget_ns = S1C_WAIT_BUDGET_NS) {
  const uint32_t a = smem_u32(bar);
  const int lane = threadIdx.x & 31;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    const bool done = mbar_try_wait(a, parity);
    if (__all_sync(0xffffffffu, done)) return true;
    if ((it & 63u) == 63u) {
      int give_up = 0;
      if (lane == 0) {
        const uint64_t now = globaltimer();
        if (t0 == 0) t0 = now;
        if ((abort && *abort) || now - t0 > budget_ns) give_up = 1;
      }
      give_up = __shfl_sync(0xffffffffu, give_up, 0);
      if (give_up) {
        if (lane == 0) {
          if (!(abort && *abort)) report(status, code);
          if (abort) *abort = 1;
        }
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------------------
// TMA: 2D tiled bulk tensor load into this CTA's shared memory, completing on an mbarrier.
// (No cluster or multi-destination forms are used anywhere in this library.)
S1C_DEV void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::
          "r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
S1C_DEV void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
// Bring [p, p + bytes) of global memory into L2 (bulk prefetch; nothing to wait for). p and bytes
// are multiples of 16.
S1C_DEV void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
// This CTA's share of an L2 prefetch of `bytes` at `p` spread over the grid: a 16-byte-aligned
// slice per CTA, issued in pieces of at most 32 KB.
S1C_DEV void prefetch_l2_share(const void* p, size_t bytes) {
  const size_t chunk = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~(size_t)15;
  const size_t b0 = (size_t)blockIdx.x * chunk, b1 = b0 + chunk < bytes ? b0 + chunk : bytes;
  for (size_t o = b0; o < b1; o += 32768)
    prefetch_l2_bulk(static_cast<const uint8_t*>(p) + o, (uint32_t)(b1 - o < 32768 ? b1 - o : 32768));
}

// ---------------------------------------------------------------------------------------
// tcgen05: tensor memory allocation, MMA, commit, loads.
S1C_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
S1C_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
S1C_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
S1C_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
S1C_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate), one CTA.
S1C_DEV void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05 op this thread issued so far has completed.
S1C_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 consecutive fp32 columns: lane i of the warp gets row (taddr.lane + i).
S1C_DEV void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  // The wait names every destination register as read-write so that no use of them can be
  // scheduled before the load has landed.
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 16 consecutive fp32 columns.
S1C_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Packed pairs of fp32 for Blackwell's f32x2 arithmetic (one FMA / MUL instruction per pair, each
// lane rounded exactly like the scalar instruction).
S1C_DEV uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
S1C_DEV uint64_t f2_splat(float v) { return f2_pack(v, v); }
S1C_DEV void f2_unpack(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
S1C_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
S1C_DEV uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// Shared-memory matrix descriptor for a K-major bf16 tile written by TMA with 128-byte
// swizzling: rows of 64 elements (128 B), 8-row swizzle atoms of 1024 B stacked along M/N
// (stride byte offset 1024). The tile base must be 1024-byte aligned; stepping K by 16
// elements inside the atom adds 32 B to the start address.
S1C_DEV uint64_t sdesc_kmajor_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);        // start address, bits [0,14)
  d |= (uint64_t)(16u >> 4) << 16;                 // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;               // stride byte offset, bits [32,46)
  d |= (uint64_t)1u << 46;                         // descriptor version for sm_100
  d |= (uint64_t)2u << 61;                         // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor, kind::f16: bf16 A and B (both K-major), fp32 D, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                      // D format f32
         | (1u << 7)                    // A format bf16
         | (1u << 10)                   // B format bf16
         | ((uint32_t)(N >> 3) << 17)   // N / 8
         | ((uint32_t)(M >> 4) << 24);  // M / 16
}

}  // namespace s1c
