// tcb_mv_ptx.cuh - PTX wrappers shared by the matvec kernels (mbarriers,
// TMA tensor copies, programmatic dependent launch, int8 mma.sync) and the
// host-side tensor-map encoder.  Internal to libtcb.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdint.h>

#include "tcb_common.cuh"

namespace tcb {
namespace mv {

// ----------------------------------------------------------------- PTX

__device__ __forceinline__ uint32_t sa(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(sa(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   sa(dst)),
               "l"(src), "r"(bytes), "r"(sa(bar))
               : "memory");
}

// 2-D tensor copy of one box into shared memory (no multicast)
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(sa(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(sa(bar))
      : "memory");
}
// the same box brought into L2 only (no shared memory, no completion)
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap *tm, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(tm)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// D += A(16x32 u8) * B(32x8 s8)
__device__ __forceinline__ void imma_u8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D += A(16x32 s8) * B(32x8 s8)
__device__ __forceinline__ void imma_s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
               : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
               : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// D += A(16x16 u8) * B(16x8 s8)
__device__ __forceinline__ void imma_u8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
               : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
               : "r"(a0), "r"(a1), "r"(b0));
}

__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ uint32_t lds16(const uint8_t *p) { return *reinterpret_cast<const uint16_t *>(p); }
// 4 bytes at a 2-byte aligned shared address
__device__ __forceinline__ uint32_t lds32_a2(const uint8_t *p) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if ((a & 2) == 0) return lds32(p);
  const uint8_t *q = p - 2;
  return __byte_perm(lds32(q), lds32(q + 4), 0x5432);
}

constexpr uint32_t M4 = 0x0F0F0F0Fu;

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(sa(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes (the copy engine's completion wakes it) or ~0.5 ms pass
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(sa(bar)), "r"(phase), "r"(500000u)
      : "memory");
  return ok != 0;
}

// a barrier completed by the copy engine (bounded: ~2 s at most)
__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t phase, int *err) {
  for (uint32_t i = 0; i < 4096u; i++)
    if (mbar_try_wait_hint(bar, phase)) return true;
  atomicExch(err, TCB_ERR_TIMEOUT);
  return false;
}

// Bring this CTA's share of [p, p + bytes) into L2 (bulk prefetches of at
// most 64 KB; a hint: no completion, no shared memory).  Used to stream the
// weights of the next kernel of a chain while this one runs.
__device__ __forceinline__ void prefetch_slice_l2(const void *p, size_t bytes) {
  if (!p || bytes < 16) return;
  const size_t per = ((bytes + gridDim.x - 1) / gridDim.x + 15) & ~(size_t)15;
  const size_t b0 = per * blockIdx.x;
  const size_t b1 = b0 + per < bytes ? b0 + per : bytes;
  const char *base = static_cast<const char *>(p);
  for (size_t o = b0; o + 16 <= b1; o += 65536) {
    const size_t n = (b1 - o < 65536 ? b1 - o : 65536) & ~(size_t)15;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(base + o)), "r"((uint32_t)n)
                 : "memory");
  }
}

// poll with a back-off of ns nanoseconds (bounded: about 2^24 polls)
__device__ __forceinline__ bool spin_bar_ns(uint64_t *bar, uint32_t phase, int *err, unsigned ns) {
  for (uint32_t i = 0; i < (1u << 24); i++) {
    if (mbar_test_wait(bar, phase)) return true;
    __nanosleep(ns);
  }
  atomicExch(err, TCB_ERR_TIMEOUT);
  return false;
}

// A barrier completed by other warps' arrives: a sleeping try_wait is not
// woken promptly by them, so poll with a short backoff (bounded: ~1 s).
__device__ __forceinline__ bool spin_bar(uint64_t *bar, uint32_t phase, int *err) {
  for (uint32_t i = 0; i < (1u << 24); i++) {
    if (mbar_test_wait(bar, phase)) return true;
    __nanosleep(32);
  }
  atomicExch(err, TCB_ERR_TIMEOUT);
  return false;
}

__device__ __forceinline__ float rcp_approx(float v) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

// small non-negative integer (< 2^16) in a 16-bit lane to float on the FMA
// pipe: place it under the exponent of 2^23 and subtract 2^23
__device__ __forceinline__ float lane16_f(uint32_t v, uint32_t sel) {
  return __int_as_float((int)__byte_perm(v, 0x4B000000u, sel)) - 8388608.0f;
}

}  // namespace mv

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda)
inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

}  // namespace tcb
