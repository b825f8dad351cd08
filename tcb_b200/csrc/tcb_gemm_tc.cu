// tcb_gemm_tc.cu - the many-row float product (prefill: M >= kTcMinM rows
// of activations) on the fifth-generation tensor cores.
//
// C (+)= X · dequant(W)ᵀ for weights W [N, K] in GGUF blocks (TR's
// Backend.Gemm quant branch, gpu/backend_quant.go:43-65; CPU semantics
// quantGemm, tensor/cpu_quant.go:47-147: the product of X with the opened
// weights).  Q4_K superblocks are dequantised inside the kernel; Q6_K, Q8_0
// and Q4_0 rows are first dequantised exactly (k_tc_wdeq) to row-scaled fp16
// in workspace, and the kernel loads them by TMA like X.
//
// Launches:
//  1. k_tc_prep: each activation row x[m] is scaled by a power of two
//     (row max brought into [2^14, 2^15)) and rounded once to fp16, stored
//     K-contiguous in workspace with the fixed 8-periodic order below; each
//     weight row n gets a power-of-two multiplier from its blocks' scales
//     (the largest magnitude a row can dequantise to is brought under 2^15),
//     so no dequantised fp16 weight overflows and small rows keep precision.
//  2. k_qgemm_tc2: clusters of two CTAs (one per SM) walk 256 x 256 tiles of
//     C persistently; the leader issues tcgen05.mma.cta_group::2 over both
//     CTAs' operand stages (warp roles at the kernel).  When the tiles are
//     fewer than the pairs, a tile's K range is split into whole-superblock
//     pieces (work units) and the epilogue writes f32 partials instead.
//  3. k_tc_reduce (split runs only): adds the partials in split order and
//     writes C.
// The epilogue divides out the two power-of-two multipliers (exact) and
// writes C with TR's one-rounding rule (accumulate: round(old + v)).
//
// Numerics: the weights are computed as fma(q, d·sc, -dmin·m) in fp16 with
// d·sc and dmin·m rounded once each, the activations are rounded once to
// fp16 (exact for bf16/f16 inputs), and the products accumulate in f32:
// about 2e-4 relative L2 against TR's f32 path.
//
// The K order inside every aligned group of 8 elements is (0 2 1 3 4 6 5 7):
// the order in which two 32-bit words of packed nibbles unpack into half2
// pairs with one mask each.  X is written in the same order, so the dot
// products are unchanged.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tcb.h"
#include "tcb_common.cuh"
#include "tcb_dequant.cuh"
#include "tcb_gemm_tc.h"
#include "tcb_mv_ptx.cuh"

namespace tcb {
namespace tc {

using mv::mbar_arrive;
using mv::mbar_expect_tx;
using mv::mbar_init;
using mv::mbar_test_wait;
using mv::sa;
using mv::tma_load_2d;

constexpr int kBK = 64;          // K elements per operand stage (one 128-byte swizzle row of fp16)
constexpr int kRawPitch = 144;  // one Q4_K superblock per staged row

// ----------------------------------------------------------------- PTX

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (SBO), descriptor version 1
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// 32 lanes x 32 consecutive 32-bit columns of tensor memory
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
      "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// 1024 + q for the two 4-bit fields of u under mask (lanes 0-15 / 16-31)
__device__ __forceinline__ __half2 nib2(uint32_t u, uint32_t mask) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(u), "r"(mask), "r"(0x64006400u));  // (u & mask) | magic
  return bits_h2(r);
}

// Q4_K 6-bit scale and min of sub-block j (0..7, a runtime index) from the
// three words y, z, w of the 12 packed scale bytes (TR tensor/quant.go:158-163)
__device__ __forceinline__ void q4k_scale_words(int j, uint32_t y, uint32_t z, uint32_t w, uint32_t &sc,
                                                uint32_t &m) {
  const uint32_t sh = 8u * (uint32_t)(j & 3);
  const uint32_t by = (y >> sh) & 0xFFu, bz = (z >> sh) & 0xFFu, bw = (w >> sh) & 0xFFu;
  if (j < 4) {
    sc = by & 63u;
    m = bz & 63u;
  } else {
    sc = (bw & 15u) | ((by >> 6) << 4);
    m = (bw >> 4) | ((bz >> 6) << 4);
  }
}

// 8 code bytes (w0 = bytes 0-3, w1 = bytes 4-7 of an 8-byte group) of a
// 64-element K step -> chunk c (their low nibbles) and chunk c + 4 (high
// nibbles) of a 128-byte swizzled row: fma(q, d·sc, -dmin·m) per half2
__device__ __forceinline__ void dq8(uint32_t w0, uint32_t w1, __half2 dlo, __half2 nlo, __half2 dhi, __half2 nhi,
                                    uint8_t *row, int c, uint32_t sw) {
  const __half2 magic = bits_h2(0x64006400u);
  const uint32_t u0 = w0 >> 8, u1 = w1 >> 8;
  uint4 lo, hi;
  lo.x = h2_bits(__hfma2(__hsub2(nib2(w0, 0x000F000Fu), magic), dlo, nlo));
  lo.y = h2_bits(__hfma2(__hsub2(nib2(u0, 0x000F000Fu), magic), dlo, nlo));
  lo.z = h2_bits(__hfma2(__hsub2(nib2(w1, 0x000F000Fu), magic), dlo, nlo));
  lo.w = h2_bits(__hfma2(__hsub2(nib2(u1, 0x000F000Fu), magic), dlo, nlo));
  hi.x = h2_bits(__hfma2(__hsub2(nib2(w0, 0x00F000F0u), magic), dhi, nhi));
  hi.y = h2_bits(__hfma2(__hsub2(nib2(u0, 0x00F000F0u), magic), dhi, nhi));
  hi.z = h2_bits(__hfma2(__hsub2(nib2(w1, 0x00F000F0u), magic), dhi, nhi));
  hi.w = h2_bits(__hfma2(__hsub2(nib2(u1, 0x00F000F0u), magic), dhi, nhi));
  *reinterpret_cast<uint4 *>(row + (((uint32_t)c ^ sw) << 4)) = lo;
  *reinterpret_cast<uint4 *>(row + (((uint32_t)(c + 4) ^ sw) << 4)) = hi;
}

// ----------------------------------------------------------------- kernels

// activation elements 8g .. 8g+7 of a row as f32 (16-byte loads when the
// row is 16-byte aligned)
__device__ __forceinline__ void load8(const char *row, int g, int xdt, bool vec, float (&v)[8]) {
  if (vec && xdt == TCB_F32) {
    const float4 *p = reinterpret_cast<const float4 *>(row) + 2 * g;
    const float4 a = p[0], b = p[1];
    v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
  } else if (vec) {
    const uint4 u = reinterpret_cast<const uint4 *>(row)[g];
    const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      if (xdt == TCB_BF16) {
        v[2 * i] = __uint_as_float(wd[i] << 16);
        v[2 * i + 1] = __uint_as_float(wd[i] & 0xFFFF0000u);
      } else {
        v[2 * i] = __half2float(__ushort_as_half((unsigned short)(wd[i] & 0xFFFFu)));
        v[2 * i + 1] = __half2float(__ushort_as_half((unsigned short)(wd[i] >> 16)));
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = load_act(row, 8 * g + i, xdt);
  }
}

// k_tc_prep: blocks [0, M) scale and convert activation rows; the rest scan
// weight rows (one warp per row).
__global__ void __launch_bounds__(256) k_tc_prep(const void *x, int xdt, long ldx, int M, int K, __half *xh,
                                                 float *ix, const uint8_t *w, int N, int nsb, float *mw,
                                                 float *iw, int perm) {
  __shared__ float red[8];
  __shared__ int bad_s;
  if ((int)blockIdx.x < M) {
    const int m = blockIdx.x;
    const char *row = static_cast<const char *>(x) + (size_t)m * ldx * (xdt == TCB_F32 ? 4 : 2);
    const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;  // 16-byte loads
    float amax = 0.f;
    int bad = 0;
    if (threadIdx.x == 0) bad_s = 0;
    for (int g = threadIdx.x; g < K / 8; g += blockDim.x) {
      float v[8];
      load8(row, g, xdt, vec, v);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float av = fabsf(v[i]);
        bad |= !(av <= 3.402823466e38f);
        amax = fmaxf(amax, av);
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (bad) bad_s = 1;
    __syncthreads();
    float a = red[0];
    for (int i = 1; i < 8; i++) a = fmaxf(a, red[i]);
    int e = 0;
    if (!bad_s && a > 0.f) e = min(max(ilogbf(a) - 14, -100), 100);
    const float mul = ldexpf(1.f, -e);
    if (threadIdx.x == 0) ix[m] = ldexpf(1.f, e);
    // 8 outputs per thread in the K order (0 2 1 3 4 6 5 7); the second pass
    // re-reads the row from L1
    uint4 *dst = reinterpret_cast<uint4 *>(xh + (size_t)m * K);
    for (int g = threadIdx.x; g < K / 8; g += blockDim.x) {
      float v[8];
      load8(row, g, xdt, vec, v);
#pragma unroll
      for (int i = 0; i < 8; i++) v[i] = __fmul_rn(v[i], mul);
      uint4 o;
      if (perm) {
        o.x = h2_bits(__floats2half2_rn(v[0], v[2]));
        o.y = h2_bits(__floats2half2_rn(v[1], v[3]));
        o.z = h2_bits(__floats2half2_rn(v[4], v[6]));
        o.w = h2_bits(__floats2half2_rn(v[5], v[7]));
      } else {
        o.x = h2_bits(__floats2half2_rn(v[0], v[1]));
        o.y = h2_bits(__floats2half2_rn(v[2], v[3]));
        o.z = h2_bits(__floats2half2_rn(v[4], v[5]));
        o.w = h2_bits(__floats2half2_rn(v[6], v[7]));
      }
      dst[g] = o;
    }
    return;
  }
  // weight row n: the largest |d·sc·q - dmin·m| any of its blocks can give is
  // below 945|d| + 63|dmin|
  const int n = ((int)blockIdx.x - M) * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (n >= N) return;
  const uint8_t *r = w + (size_t)n * nsb * kRawPitch;
  float bound = 0.f;
  int bad = 0;
  for (int b = lane; b < nsb; b += 32) {
    const uint32_t dm = *reinterpret_cast<const uint32_t *>(r + (size_t)b * kRawPitch);
    const float d = fabsf(__half2float(__ushort_as_half((unsigned short)(dm & 0xFFFFu))));
    const float dn = fabsf(__half2float(__ushort_as_half((unsigned short)(dm >> 16))));
    const float bb = fmaf(945.f, d, 63.f * dn);
    bad |= !(bb <= 3.402823466e38f);
    bound = fmaxf(bound, bb);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) bound = fmaxf(bound, __shfl_xor_sync(0xFFFFFFFFu, bound, o));
  bad = __any_sync(0xFFFFFFFFu, bad);
  int e = 0;
  if (!bad && bound > 0.f) e = min(max(ilogbf(bound) - 14, -100), 100);
  if (lane == 0) {
    mw[n] = ldexpf(1.f, -e);
    iw[n] = ldexpf(1.f, e);
  }
}

// elements j .. j+7 (j a multiple of 8) of the block at b, with TR's
// dequant operations; the 8 share their block scales
template <int W>
__device__ __forceinline__ void dequant8(const uint8_t *b, int j, float (&v)[8]) {
  if constexpr (W == TCB_Q6_K) {
    const int n = j >> 7, c = (j >> 5) & 3, l = j & 31;
    const float ds = mulx(half_exact(ld_u16(b + 208)), (float)(int8_t)b[192 + 8 * n + (l >> 4) + 2 * c]);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const uint32_t low = (b[64 * n + l + i + 32 * (c & 1)] >> (4 * (c >> 1))) & 0xFu;
      const uint32_t high = (b[128 + 32 * n + l + i] >> (2 * c)) & 3u;
      v[i] = mulx(ds, (float)((int)(low | (high << 4)) - 32));
    }
  } else if constexpr (W == TCB_Q8_0) {
    const float d = half_exact(ld_u16(b));
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = mulx((float)(int8_t)b[2 + j + i], d);
  } else {
    const float d = half_exact(ld_u16(b));
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const uint32_t q = b[2 + ((j + i) & 15)];
      v[i] = mulx((float)((int)(((j + i) < 16 ? q : q >> 4) & 0xFu) - 8), d);
    }
  }
}

// k_tc_wdeq: the weights of the other block types for the tensor-core
// kernel (rows of at most kWdeqMaxRowBytes): row n dequantised exactly (TR's dequant), scaled by a power of two
// and rounded once to fp16 (natural K order); iw[n] holds the inverse
// factor.  The factor brings the row's bound -- the largest magnitude its
// blocks' scales allow: 32|d|max|sc| (Q6_K), 128|d| (Q8_0), 8|d| (Q4_0) --
// into [2^14, 2^15), so no value overflows and the normal fp16 values keep
// their full precision; a non-finite scale leaves the row unscaled.  The
// row's blocks are first copied into shared memory with 16-byte loads (the
// whole row in flight at once) and dequantised from there in one pass; little
// register and shared-memory use per CTA keeps many rows in flight per SM.
// a weight row's blocks fit the default 48 KB of dynamic shared memory
constexpr size_t kWdeqMaxRowBytes = 48 * 1024;
// rows of a fused activation prologue (k_tc_prep_pro keeps a row in registers)
constexpr int kProMaxK = 16384;
template <int W>
__device__ __forceinline__ float block_bound(const uint8_t *b) {
  if constexpr (W == TCB_Q6_K) {
    int sm = 0;
#pragma unroll
    for (int i = 0; i < 16; i++) sm = max(sm, abs((int)(int8_t)b[192 + i]));
    return fabsf(half_exact(ld_u16(b + 208))) * (float)(32 * sm);
  } else if constexpr (W == TCB_Q8_0) {
    return fabsf(half_exact(ld_u16(b))) * 128.f;
  } else {
    return fabsf(half_exact(ld_u16(b))) * 8.f;
  }
}

template <int W>
__global__ void __launch_bounds__(256) k_tc_wdeq(const uint8_t *w, int N, int K, __half *wh, float *iw) {
  extern __shared__ __align__(16) uint8_t raw[];
  __shared__ float red[8];
  constexpr int E = Fmt<W>::E, B = Fmt<W>::B;
  const int n = blockIdx.x, tid = threadIdx.x;
  const int nb = K / E;
  const size_t rb = (size_t)nb * B;
  const uint8_t *row = w + (size_t)n * rb;
  if (((reinterpret_cast<uintptr_t>(row) | rb) & 15) == 0) {
    for (int i = tid; i < (int)(rb / 16); i += blockDim.x)
      reinterpret_cast<uint4 *>(raw)[i] = __ldcs(reinterpret_cast<const uint4 *>(row) + i);
  } else if (((reinterpret_cast<uintptr_t>(row) | rb) & 1) == 0) {
    for (int i = tid; i < (int)(rb / 2); i += blockDim.x)
      reinterpret_cast<uint16_t *>(raw)[i] = __ldcs(reinterpret_cast<const unsigned short *>(row) + i);
  } else {
    for (int i = tid; i < (int)rb; i += blockDim.x) raw[i] = row[i];
  }
  __syncthreads();
  float bound = 0.f;
  int bad = 0;
  for (int b = tid; b < nb; b += blockDim.x) {
    const float v = block_bound<W>(raw + (size_t)b * B);
    bad |= !(v <= 3.402823466e38f);
    bound = fmaxf(bound, v);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) bound = fmaxf(bound, __shfl_xor_sync(0xFFFFFFFFu, bound, o));
  if ((tid & 31) == 0) red[tid >> 5] = bound;
  const int any_bad = __syncthreads_or(bad);
  float a = red[0];
  for (int i = 1; i < 8; i++) a = fmaxf(a, red[i]);
  int e = 0;
  if (!any_bad && a > 0.f) e = min(max(ilogbf(a) - 14, -100), 100);
  const float mul = ldexpf(1.f, -e);
  if (tid == 0) iw[n] = ldexpf(1.f, e);
  uint4 *dst = reinterpret_cast<uint4 *>(wh + (size_t)n * K);
  for (int g = tid; 8 * g < K; g += blockDim.x) {
    float x[8];
    dequant8<W>(raw + (size_t)(8 * g / E) * B, (8 * g) % E, x);
    uint4 o;
    o.x = h2_bits(__floats2half2_rn(__fmul_rn(x[0], mul), __fmul_rn(x[1], mul)));
    o.y = h2_bits(__floats2half2_rn(__fmul_rn(x[2], mul), __fmul_rn(x[3], mul)));
    o.z = h2_bits(__floats2half2_rn(__fmul_rn(x[4], mul), __fmul_rn(x[5], mul)));
    o.w = h2_bits(__floats2half2_rn(__fmul_rn(x[6], mul), __fmul_rn(x[7], mul)));
    __stcs(dst + g, o);
  }
}

// k_tc_prep_pro: activation rows with a prologue applied before the scaling
// of k_tc_prep (same power-of-two rule, same K order):
//   kTcProRms:    x / sqrt(mean(x^2) + eps) * nw  (RMSNorm, TR lib/layers.tr 68-79)
//   kTcProSwiglu: silu(g) * u over merged rows [G | U] of 2K elements
//                 (TR's merged SwiGLU, lib/layers.tr 224-230)
// One CTA per row; a thread keeps its NG groups of 8 values in registers, so
// the row is read from memory once.  f32 rows only.
template <int NG>
__global__ void __launch_bounds__(256) k_tc_prep_pro(const float *x, long ldx, int K, int pro, const float *nw,
                                                     float eps, __half *xh, float *ix, int perm) {
  __shared__ float red[8], red2[8];
  const int m = blockIdx.x, tid = threadIdx.x;
  const float *row = x + (size_t)m * ldx;
  float v[NG][8];
#pragma unroll
  for (int gi = 0; gi < NG; gi++) {
    const int g = tid + gi * 256;
    if (8 * g < K) {
      const float4 a = __ldcs(reinterpret_cast<const float4 *>(row) + 2 * g);
      const float4 b = __ldcs(reinterpret_cast<const float4 *>(row) + 2 * g + 1);
      v[gi][0] = a.x, v[gi][1] = a.y, v[gi][2] = a.z, v[gi][3] = a.w;
      v[gi][4] = b.x, v[gi][5] = b.y, v[gi][6] = b.z, v[gi][7] = b.w;
      if (pro == kTcProSwiglu) {
        const float4 c = __ldcs(reinterpret_cast<const float4 *>(row + K) + 2 * g);
        const float4 d = __ldcs(reinterpret_cast<const float4 *>(row + K) + 2 * g + 1);
        const float u[8] = {c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float gg = v[gi][i];
          v[gi][i] = __fmul_rn(__fmul_rn(gg, __frcp_rn(__fadd_rn(1.0f, expf(-gg)))), u[i]);
        }
      }
    }
  }
  if (pro == kTcProRms) {
    float ss = 0.f;
#pragma unroll
    for (int gi = 0; gi < NG; gi++)
      if (8 * (tid + gi * 256) < K)
#pragma unroll
        for (int i = 0; i < 8; i++) ss = fmaf(v[gi][i], v[gi][i], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
    if ((tid & 31) == 0) red2[tid >> 5] = ss;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < 8; i++) t += red2[i];
    const float rs = sqrtf(__fdiv_rn(t, (float)K) + eps);
#pragma unroll
    for (int gi = 0; gi < NG; gi++) {
      const int g = tid + gi * 256;
      if (8 * g < K) {
        const float4 a = __ldg(reinterpret_cast<const float4 *>(nw) + 2 * g);
        const float4 b = __ldg(reinterpret_cast<const float4 *>(nw) + 2 * g + 1);
        const float ww[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; i++) v[gi][i] = __fmul_rn(__fdiv_rn(v[gi][i], rs), ww[i]);
      }
    }
  }
  float amax = 0.f;
  int bad = 0;
#pragma unroll
  for (int gi = 0; gi < NG; gi++)
    if (8 * (tid + gi * 256) < K)
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float av = fabsf(v[gi][i]);
        bad |= !(av <= 3.402823466e38f);
        amax = fmaxf(amax, av);
      }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  if ((tid & 31) == 0) red[tid >> 5] = amax;
  const int any_bad = __syncthreads_or(bad);
  float a = red[0];
  for (int i = 1; i < 8; i++) a = fmaxf(a, red[i]);
  int e = 0;
  if (!any_bad && a > 0.f) e = min(max(ilogbf(a) - 14, -100), 100);
  const float mul = ldexpf(1.f, -e);
  if (tid == 0) ix[m] = ldexpf(1.f, e);
  uint4 *dst = reinterpret_cast<uint4 *>(xh + (size_t)m * K);
#pragma unroll
  for (int gi = 0; gi < NG; gi++) {
    const int g = tid + gi * 256;
    if (8 * g < K) {
      float *q = v[gi];
#pragma unroll
      for (int i = 0; i < 8; i++) q[i] = __fmul_rn(q[i], mul);
      uint4 o;
      if (perm) {
        o.x = h2_bits(__floats2half2_rn(q[0], q[2]));
        o.y = h2_bits(__floats2half2_rn(q[1], q[3]));
        o.z = h2_bits(__floats2half2_rn(q[4], q[6]));
        o.w = h2_bits(__floats2half2_rn(q[5], q[7]));
      } else {
        o.x = h2_bits(__floats2half2_rn(q[0], q[1]));
        o.y = h2_bits(__floats2half2_rn(q[2], q[3]));
        o.z = h2_bits(__floats2half2_rn(q[4], q[5]));
        o.w = h2_bits(__floats2half2_rn(q[6], q[7]));
      }
      dst[g] = o;
    }
  }
}

struct TcArgs {
  CUtensorMap ta;  // fp16 X [M][K], box 64 x 128, 128-byte swizzle
  CUtensorMap tw;  // weight bytes [N][nsb * 144], box 144 x 128
  const float *mw, *iw, *ix;
  void *c;
  long ldc;
  int cdt, accumulate, M, N, nsb;
  int ksplit, sbper;  // K splits of a tile and superblocks per split
  float *part;        // [ksplit][M][N] f32 partials when ksplit > 1
  int *err;
};

// ----------------------------------------------------------------- 2-CTA kernel
//
// k_qgemm_tc2: a cluster of two CTAs (one per SM) owns a 256 x 256 tile of C
// and the pair walks the tiles persistently.  CTA r of the pair holds
// activation rows 128r.. and weight rows 128r.. of the tile; the leader
// (r = 0) issues tcgen05.mma.cta_group::2 (M 256, N 256, K 16), which reads
// both CTAs' operand stages and leaves rows 128r.. of the accumulator in CTA
// r's tensor memory.  Each SM therefore dequantises 128 weight rows per 256
// rows of X (half the work per flop of the one-CTA tile) and reads half the B
// operand from shared memory.
//   warp 0        TMA of the CTA's 128 x 64 fp16 activation tile (both
//                 CTAs complete_tx on the leader's full barrier of the stage,
//                 which the dequantising warps of both CTAs also arrive on)
//   warp 1        tensor-memory allocation (512 columns: two accumulators);
//                 in the leader, the MMA issue
//   warp 2        TMA of raw superblocks (128 weight rows x 144 B)
//   warps 3..10   dequantise into the swizzled fp16 stage, arrive on the
//                 leader: kGroups groups of warps take interleaved K steps
//                 of each superblock, so kGroups steps are in flight
//   warps 11..14  epilogue: tensor memory -> C while the next tile runs in
//                 the other accumulator
namespace tc2 {

constexpr int kRows = 128;  // activation rows and weight rows per CTA
constexpr int kBK = 64;
#ifndef TCB_TC2_STAGES
#define TCB_TC2_STAGES 5
#endif
#ifndef TCB_TC2_RAW_STAGES
#define TCB_TC2_RAW_STAGES 2
#endif
#ifndef TCB_TC2_DQ_SLEEP
#define TCB_TC2_DQ_SLEEP 0
#endif
constexpr int kS = TCB_TC2_STAGES;       // operand stages (A and B share the empty barrier)
constexpr int kSR = TCB_TC2_RAW_STAGES;  // raw superblock stages
constexpr unsigned kDqSleep = TCB_TC2_DQ_SLEEP;  // back-off of the dequantising warps' polls (ns)
constexpr int kABytes = kRows * kBK * 2;
constexpr int kBBytes = kRows * kBK * 2;
constexpr int kRawBytes = kRows * kRawPitch;
constexpr int kOffB = kS * kABytes;
constexpr int kOffR = kOffB + kS * kBBytes;
constexpr int kOffBar = kOffR + kSR * kRawBytes;
// F[kS] E[kS] rF[kSR] rE[kSR] accF[2] accE[2]
constexpr int kNumBars = 2 * kS + 2 * kSR + 4;
constexpr int kOffSlot = kOffBar + 8 * kNumBars;
constexpr int kSmem = kOffSlot + 16 + 1024;
constexpr int kWarpA = 0, kWarpMma = 1, kWarpRaw = 2, kWarpDq = 3, kDqWarps = 8, kWarpEp = 11, kEpWarps = 4;
constexpr int kThreads = 15 * 32;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(256 >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
#ifndef TCB_TC2_GROUPS
#define TCB_TC2_GROUPS 4
#endif
constexpr int kGroups = TCB_TC2_GROUPS;     // dequantising groups (K steps in flight)
constexpr int kGT = kDqWarps * 32 / kGroups;  // threads per group
constexpr int kRPT = kRows / kGT;             // weight rows per thread
static_assert((kGroups == 2 || kGroups == 4) && kRPT * kGT == kRows, "dequantising groups");
static_assert(kSmem <= 232448, "shared memory");

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// the same shared-memory location in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ void arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc2(uint32_t slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(cols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc2(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void mma2(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc)
      : "memory");
}
// arrive on the barrier at cluster address addr once this thread's MMAs are done
__device__ __forceinline__ void commit2(uint32_t addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(addr) : "memory");
}
// TMA into this CTA's shared memory, completing on a barrier of either CTA of the pair
__device__ __forceinline__ void tma_pair(void *dst, const CUtensorMap *tm, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(sa(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Bounded poll of a barrier phase by one thread (acquire at the default CTA
// scope, as for every barrier wait of this kernel, including phases that the
// peer CTA's copies, arrives and the leader's commits complete).  Gives up
// (false) when another role has aborted or after 2^26 polls (over a second),
// recording a timeout.  The bound is an iteration count: reading the clock
// inside the spin measured 8 % slower on the whole product.
__device__ __forceinline__ bool poll2(uint64_t *bar, uint32_t ph, volatile int *ab, int *err, unsigned ns) {
  for (uint32_t i = 0; i < (1u << 26); i++) {
    if (mbar_test_wait(bar, ph)) return true;
    if (*ab) return false;
    if (ns) __nanosleep(ns);
  }
  *ab = 1;
  atomicExch(err, TCB_ERR_TIMEOUT);
  return false;
}
__device__ __forceinline__ bool warp_poll2(uint64_t *bar, uint32_t ph, volatile int *ab, int *err, unsigned ns) {
  int ok = 0;
  if ((threadIdx.x & 31) == 0) ok = poll2(bar, ph, ab, err, ns);
  __syncwarp();
  return __shfl_sync(0xFFFFFFFFu, ok, 0) != 0;
}
// the same without the abort exit (draining copies still in flight)
__device__ __forceinline__ void drain2(uint64_t *bar, uint32_t ph, int *err) {
  for (uint32_t i = 0; i < (1u << 22); i++) {
    if (mbar_test_wait(bar, ph)) return;
    __nanosleep(64);
  }
  atomicExch(err, TCB_ERR_TIMEOUT);
}

// 32 outputs of row m starting at column n0 (all < N when full)
__device__ __forceinline__ void store32(const TcArgs &a, long m, int n0, const uint32_t (&v)[32], float sx,
                                        bool full) {
  float r[32];
#pragma unroll
  for (int i = 0; i < 32; i++) r[i] = __fmul_rn(__uint_as_float(v[i]), sx);
  const long base = m * a.ldc + n0;
  const size_t es = a.cdt == TCB_F32 ? 4 : 2;
  const bool vec = full && ((reinterpret_cast<uintptr_t>(a.c) + (size_t)base * es) & 15) == 0;
  if (vec) {
    const float4 *iw4 = reinterpret_cast<const float4 *>(a.iw + n0);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float4 f = iw4[i];
      r[4 * i] = __fmul_rn(r[4 * i], f.x);
      r[4 * i + 1] = __fmul_rn(r[4 * i + 1], f.y);
      r[4 * i + 2] = __fmul_rn(r[4 * i + 2], f.z);
      r[4 * i + 3] = __fmul_rn(r[4 * i + 3], f.w);
    }
    if (a.cdt == TCB_F32) {
      float4 *p = reinterpret_cast<float4 *>(static_cast<float *>(a.c) + base);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        float4 o = make_float4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
        if (a.accumulate) {
          const float4 old = p[i];
          o.x = __fadd_rn(old.x, o.x);
          o.y = __fadd_rn(old.y, o.y);
          o.z = __fadd_rn(old.z, o.z);
          o.w = __fadd_rn(old.w, o.w);
        }
        p[i] = o;
      }
    } else {
      uint4 *p = reinterpret_cast<uint4 *>(static_cast<uint16_t *>(a.c) + base);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        uint4 old = make_uint4(0, 0, 0, 0);
        if (a.accumulate) old = p[i];
        const uint32_t ow[4] = {old.x, old.y, old.z, old.w};
        uint32_t pk[4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
          uint32_t hh[2];
#pragma unroll
          for (int k = 0; k < 2; k++) {
            float v = r[8 * i + 2 * j + k];
            const uint16_t o = (uint16_t)(ow[j] >> (16 * k));
            if (a.accumulate) v = __fadd_rn(a.cdt == TCB_BF16 ? bf16_to_f32(o) : half_exact(o), v);
            hh[k] = a.cdt == TCB_BF16 ? f32_to_bf16(v) : f32_to_f16(v);
          }
          pk[j] = hh[0] | (hh[1] << 16);
        }
        p[i] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 32; i++)
    if (n0 + i < a.N) store_out(a.c, base + i, a.cdt, __fmul_rn(r[i], a.iw[n0 + i]), a.accumulate != 0);
}

// 32 scaled f32 partials of row m from column n0 into split `split`'s slice
__device__ __forceinline__ void store_part(const TcArgs &a, int split, long m, int n0, const uint32_t (&v)[32],
                                           float sx, bool full) {
  float *p = a.part + ((size_t)split * a.M + m) * a.N + n0;
  if (full && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
    const float4 *iw4 = reinterpret_cast<const float4 *>(a.iw + n0);
    float4 *p4 = reinterpret_cast<float4 *>(p);
#pragma unroll
    for (int i = 0; i < 8; i++) {
      const float4 f = iw4[i];
      p4[i] = make_float4(__fmul_rn(__fmul_rn(__uint_as_float(v[4 * i]), sx), f.x),
                          __fmul_rn(__fmul_rn(__uint_as_float(v[4 * i + 1]), sx), f.y),
                          __fmul_rn(__fmul_rn(__uint_as_float(v[4 * i + 2]), sx), f.z),
                          __fmul_rn(__fmul_rn(__uint_as_float(v[4 * i + 3]), sx), f.w));
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 32; i++)
    if (n0 + i < a.N) p[i] = __fmul_rn(__fmul_rn(__uint_as_float(v[i]), sx), a.iw[n0 + i]);
}

// DQ: Q4_K superblocks dequantised in the kernel; otherwise B is fp16
// weights (a.tw over them) loaded by TMA like A
template <bool DQ>
__global__ void __launch_bounds__(kThreads, 1) k_qgemm_tc2(const __grid_constant__ TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t *sA = sm, *sB = sm + kOffB, *sR = sm + kOffR;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kOffBar);
  uint64_t *F = bars, *E = bars + kS, *rF = bars + 2 * kS, *rE = rF + kSR, *accF = rE + kSR,
           *accE = accF + 2;
  uint32_t *slot = reinterpret_cast<uint32_t *>(sm + kOffSlot);
  volatile int *ab = reinterpret_cast<volatile int *>(sm + kOffSlot + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cta_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles_n = (a.N + 255) >> 8, tiles = ((a.M + 255) >> 8) * tiles_n;
  // work unit u: tile u / ksplit, superblocks [sb0, sb1) of split u % ksplit
  const int units = tiles * a.ksplit;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kS; i++) {
      // full: the leader's expect_tx arrive (both CTAs' activation bytes) and
      // the arrives of one dequantising group's warps in each CTA
      mbar_init(F + i, 1 + (DQ ? 2 * (kDqWarps / kGroups) : 0));
      mbar_init(E + i, 1);
    }
    for (int i = 0; i < kSR; i++) {
      mbar_init(rF + i, 1);
      mbar_init(rE + i, kDqWarps);
    }
    for (int i = 0; i < 2; i++) {
      mbar_init(accF + i, 1);
      mbar_init(accE + i, 2 * kEpWarps);
    }
    *ab = 0;
    mv::fence_barrier_init();
  }
  if (warp == kWarpMma) {
    tmem_alloc2(sa(slot), kTmemCols);
    tmem_relinquish2();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = *slot;
  mv::pdl_wait();

  if (warp == kWarpA) {
    if (lane == 0) {
      const uint32_t lF = mapa(sa(F), 0);
      int g = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs) {
        const int tile = u / a.ksplit, sb0 = (u % a.ksplit) * a.sbper, sb1 = min(a.nsb, sb0 + a.sbper);
        const int tm = tile / tiles_n;
        for (int ks = 4 * sb0; ks < 4 * sb1; ks++, g++) {
          const int s = g % kS;
          if (!poll2(E + s, ((g / kS) & 1) ^ 1, ab, a.err, 0)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(F + s, 2 * kABytes + (DQ ? 0 : 2 * kBBytes));
          tma_pair(sA + s * kABytes, &a.ta, ks * kBK, tm * 256 + (int)rank * kRows, lF + 8 * s);
        }
      }
      // loads still in flight complete before the MMA frees their stage
      for (int j = g - kS > 0 ? g - kS : 0; j < g; j++) drain2(E + j % kS, (j / kS) & 1, a.err);
    }
  } else if (warp == kWarpRaw) {
    if (lane == 0) {
      if constexpr (DQ) {
        int gr = 0;
        bool ok = true;
        for (int u = pair; u < units && ok; u += npairs) {
          const int tile = u / a.ksplit, sb0 = (u % a.ksplit) * a.sbper, sb1 = min(a.nsb, sb0 + a.sbper);
          const int tn = tile % tiles_n;
          for (int sb = sb0; sb < sb1; sb++, gr++) {
            const int r = gr % kSR;
            if (!poll2(rE + r, ((gr / kSR) & 1) ^ 1, ab, a.err, 0)) {
              ok = false;
              break;
            }
            mbar_expect_tx(rF + r, kRawBytes);
            tma_load_2d(sR + r * kRawBytes, &a.tw, sb * kRawPitch, tn * 256 + (int)rank * kRows, rF + r);
          }
        }
        for (int j = gr - kSR > 0 ? gr - kSR : 0; j < gr; j++) drain2(rF + j % kSR, (j / kSR) & 1, a.err);
      } else {
        // fp16 weight tiles of this CTA's 128 rows, on the leader's full barrier
        const uint32_t lF = mapa(sa(F), 0);
        int g = 0;
        bool ok = true;
        for (int u = pair; u < units && ok; u += npairs) {
          const int tile = u / a.ksplit, sb0 = (u % a.ksplit) * a.sbper, sb1 = min(a.nsb, sb0 + a.sbper);
          const int tn = tile % tiles_n;
          for (int ks = 4 * sb0; ks < 4 * sb1; ks++, g++) {
            const int s = g % kS;
            if (!poll2(E + s, ((g / kS) & 1) ^ 1, ab, a.err, 0)) {
              ok = false;
              break;
            }
            tma_pair(sB + s * kBBytes, &a.tw, ks * kBK, tn * 256 + (int)rank * kRows, lF + 8 * s);
          }
        }
        for (int j = g - kS > 0 ? g - kS : 0; j < g; j++) drain2(E + j % kS, (j / kS) & 1, a.err);
      }
    }
  } else if (warp == kWarpMma) {
    if (leader && lane == 0) {
      const uint64_t da0 = sw128_desc(sa(sA)), db0 = sw128_desc(sa(sB));
      const uint32_t eOwn = mapa(sa(E), 0), ePeer = mapa(sa(E), 1);
      const uint32_t fOwn = mapa(sa(accF), 0), fPeer = mapa(sa(accF), 1);
      int it = 0, s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int u = pair; u < units && ok; u += npairs, it++) {
        const int sb0 = (u % a.ksplit) * a.sbper, sb1 = min(a.nsb, sb0 + a.sbper);
        const int buf = it & 1;
        if (!poll2(accE + buf, ((it >> 1) & 1) ^ 1, ab, a.err, 0)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * 256);
        for (int ks = 4 * sb0; ks < 4 * sb1; ks++) {
          if (!poll2(F + s, ph, ab, a.err, 0)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // stage offsets in the descriptors' 16-byte address units
          const uint64_t da = da0 + (uint64_t)(s * (kABytes >> 4)), db = db0 + (uint64_t)(s * (kBBytes >> 4));
#pragma unroll
          for (int kk = 0; kk < kBK / 16; kk++) mma2(d, da + 2 * kk, db + 2 * kk, (ks != 4 * sb0) || kk != 0);
          commit2(eOwn + 8 * s);
          commit2(ePeer + 8 * s);
          if (++s == kS) {
            s = 0;
            ph ^= 1;
          }
        }
        commit2(fOwn + 8 * buf);
        commit2(fPeer + 8 * buf);
      }
    }
  } else if (warp < kWarpEp) {
    if constexpr (!DQ) {
      // B arrives by TMA: nothing to dequantise
    } else {
    // ---- dequantise: kGroups groups of warps take interleaved K steps of
    // each superblock (kGroups steps in flight); a thread owns kRPT rows
    const int tid = threadIdx.x - kWarpDq * 32, grp = tid / kGT, t = tid % kGT;
    const uint32_t lF = mapa(sa(F), 0);
    int gr = 0;
    bool ok = true;
    for (int u = pair; u < units && ok; u += npairs) {
      const int tile = u / a.ksplit, sb0 = (u % a.ksplit) * a.sbper, sb1 = min(a.nsb, sb0 + a.sbper);
      float mwr[kRPT];
#pragma unroll
      for (int i = 0; i < kRPT; i++) {
        const int n = (tile % tiles_n) * 256 + (int)rank * kRows + t + i * kGT;
        mwr[i] = n < a.N ? a.mw[n] : 0.f;
      }
      for (int sb = sb0; sb < sb1 && ok; sb++, gr++) {
        const int r = gr % kSR;
        if (!warp_poll2(rF + r, (gr / kSR) & 1, ab, a.err, kDqSleep)) {
          ok = false;
          break;
        }
        uint4 hdr[kRPT];
        float dd[kRPT], dm[kRPT];
#pragma unroll
        for (int i = 0; i < kRPT; i++) {
          hdr[i] = *reinterpret_cast<const uint4 *>(sR + r * kRawBytes + (t + i * kGT) * kRawPitch);
          dd[i] = __fmul_rn(__half2float(__ushort_as_half((unsigned short)(hdr[i].x & 0xFFFFu))), mwr[i]);
          dm[i] = __fmul_rn(__half2float(__ushort_as_half((unsigned short)(hdr[i].x >> 16))), mwr[i]);
        }
#pragma unroll
        for (int h2 = 0; h2 < 4 / kGroups; h2++) {
          const int g4 = grp + kGroups * h2;  // K step within the superblock
          const int g = gr * 4 + g4, s = g % kS;
          if (!warp_poll2(E + s, ((g / kS) & 1) ^ 1, ab, a.err, kDqSleep)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int i = 0; i < kRPT; i++) {
            const int row = t + i * kGT;
            const uint32_t sw = (uint32_t)(row & 7);
            uint32_t s0, m0, s1, m1;
            q4k_scale_words(2 * g4, hdr[i].y, hdr[i].z, hdr[i].w, s0, m0);
            q4k_scale_words(2 * g4 + 1, hdr[i].y, hdr[i].z, hdr[i].w, s1, m1);
            const __half2 dlo = __float2half2_rn(__fmul_rn(dd[i], (float)s0));
            const __half2 nlo = __float2half2_rn(-__fmul_rn(dm[i], (float)m0));
            const __half2 dhi = __float2half2_rn(__fmul_rn(dd[i], (float)s1 * 0.0625f));
            const __half2 nhi = __float2half2_rn(-__fmul_rn(dm[i], (float)m1));
            const uint4 *qs = reinterpret_cast<const uint4 *>(sR + r * kRawBytes + row * kRawPitch + 16 + 32 * g4);
            const uint4 q0 = qs[0], q1 = qs[1];
            uint8_t *dst = sB + s * kBBytes + row * 128;
            dq8(q0.x, q0.y, dlo, nlo, dhi, nhi, dst, 0, sw);
            dq8(q0.z, q0.w, dlo, nlo, dhi, nhi, dst, 1, sw);
            dq8(q1.x, q1.y, dlo, nlo, dhi, nhi, dst, 2, sw);
            dq8(q1.z, q1.w, dlo, nlo, dhi, nhi, dst, 3, sw);
          }
          mv::fence_proxy_async();
          __syncwarp();
          if (lane == 0) arrive_cluster(lF + 8 * s);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(rE + r);
      }
    }
    }
  } else {
    // ---- epilogue: TMEM lanes 32q.. are rows 128 rank + 32q.. of the tile
    const int q = warp & 3;
    const uint32_t laE = mapa(sa(accE), 0);
    int it = 0;
    for (int u = pair; u < units; u += npairs, it++) {
      const int tile = u / a.ksplit, split = u % a.ksplit;
      const int buf = it & 1;
      if (!warp_poll2(accF + buf, (it >> 1) & 1, ab, a.err, 64)) break;
      tc_fence_after();
      const int tm = tile / tiles_n, tn = tile % tiles_n;
      const long m = (long)tm * 256 + rank * kRows + q * 32 + lane;
      const bool live = m < a.M;
      const float sx = live ? a.ix[m] : 0.f;
#pragma unroll 1
      for (int j = 0; j < 8; j++) {
        uint32_t v[32];
        tmem_ld32(tmem + (uint32_t)(buf * 256 + j * 32) + ((uint32_t)(q * 32) << 16), v);
        if (j == 7) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) arrive_cluster(laE + 8 * buf);
        }
        const int n0 = tn * 256 + j * 32;
        if (!live || n0 >= a.N) continue;
        if (a.ksplit == 1) store32(a, m, n0, v, sx, n0 + 32 <= a.N);
        else store_part(a, split, m, n0, v, sx, n0 + 32 <= a.N);
      }
    }
  }
  tc_fence_before();
  __syncwarp();
  __syncthreads();
  cluster_sync();
  if (warp == kWarpMma) {
    tc_fence_after();
    tmem_dealloc2(tmem, kTmemCols);
  }
}

// C (+)= the sum of the K splits' partials, added in split order (deterministic)
__global__ void __launch_bounds__(256) k_tc_reduce(const float *part, int ksplit, int M, int N, void *c, int cdt,
                                                   long ldc, int accumulate) {
  const size_t total = (size_t)M * N, slice = total;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    float v = part[i];
    for (int k = 1; k < ksplit; k++) v = __fadd_rn(v, part[k * slice + i]);
    const long m = (long)(i / N), n = (long)(i % N);
    store_out(c, m * ldc + n, cdt, v, accumulate != 0);
  }
}

}  // namespace tc2

}  // namespace tc

// ----------------------------------------------------------------- host

namespace {

// clusters of the 2-CTA kernel that fit on the device at once (0 if the
// kernel cannot be configured)
int max_pairs() {
  static int n = [] {
    if (cudaFuncSetAttribute(tc::tc2::k_qgemm_tc2<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             tc::tc2::kSmem) != cudaSuccess ||
        cudaFuncSetAttribute(tc::tc2::k_qgemm_tc2<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             tc::tc2::kSmem) != cudaSuccess)
      return 0;
    cudaLaunchConfig_t q{};
    cudaLaunchAttribute ca[1];
    ca[0].id = cudaLaunchAttributeClusterDimension;
    ca[0].val.clusterDim.x = 2;
    ca[0].val.clusterDim.y = 1;
    ca[0].val.clusterDim.z = 1;
    q.gridDim = dim3(2 * 148);
    q.blockDim = dim3(tc::tc2::kThreads);
    q.dynamicSmemBytes = tc::tc2::kSmem;
    q.attrs = ca;
    q.numAttrs = 1;
    int r = 0;
    if (cudaOccupancyMaxActiveClusters(&r, tc::tc2::k_qgemm_tc2<true>, &q) != cudaSuccess) r = 0;
    return r;
  }();
  return n;
}

struct TcPlan {
  int tiles, ksplit, sbper, pairs;
  size_t xh, ix, w, part, wh;  // workspace pieces (bytes, 256-aligned)
};

size_t up256(size_t b) { return (b + 255) & ~(size_t)255; }

// K splits when the 256 x 256 tiles do not give every pair one: as many
// splits (whole superblocks each) as keep one round of work units
TcPlan tc_plan(int wtype, int M, int N, int K) {
  TcPlan p{};
  const int nsb = K / 256;
  p.pairs = max_pairs();
  p.tiles = ((M + 255) / 256) * ((N + 255) / 256);
  int ks = p.pairs > p.tiles ? p.pairs / p.tiles : 1;
  if (ks > nsb) ks = nsb;
  if (ks < 1) ks = 1;
  p.sbper = (nsb + ks - 1) / ks;
  p.ksplit = (nsb + p.sbper - 1) / p.sbper;
  p.xh = up256((size_t)M * K * 2);
  p.ix = up256((size_t)M * 4);
  p.w = up256((size_t)N * 4);
  p.part = p.ksplit > 1 ? up256((size_t)p.ksplit * M * N * 4) : 0;
  p.wh = wtype == TCB_Q4_K ? 0 : up256((size_t)N * K * 2);  // fp16 weights of the other types
  return p;
}

}  // namespace

bool tc_eligible_rows(int wtype, int N, int K, const void *w) {
  const bool typ = (wtype == TCB_Q4_K && (reinterpret_cast<uintptr_t>(w) & 15) == 0) || wtype == TCB_Q6_K ||
                   wtype == TCB_Q8_0 || wtype == TCB_Q4_0;
  return typ && N > 0 && K >= 256 && K % 256 == 0 &&
         (wtype == TCB_Q4_K ||
          (size_t)K / block_elems(wtype) * block_bytes(wtype) <= tc::kWdeqMaxRowBytes) &&
         tensor_map_encoder() != nullptr && max_pairs() > 0;
}

bool tc_eligible(int wtype, int M, int N, int K, const void *w) {
  const bool typ = (wtype == TCB_Q4_K && (reinterpret_cast<uintptr_t>(w) & 15) == 0) || wtype == TCB_Q6_K ||
                   wtype == TCB_Q8_0 || wtype == TCB_Q4_0;
  return typ && M >= kTcMinM && N > 0 && K >= 256 && K % 256 == 0 &&
         (wtype == TCB_Q4_K ||
          (size_t)K / block_elems(wtype) * block_bytes(wtype) <= tc::kWdeqMaxRowBytes) &&
         tensor_map_encoder() != nullptr && max_pairs() > 0;
}

size_t tc_workspace_bytes(int wtype, int M, int N, int K) {
  const TcPlan p = tc_plan(wtype, M, N, K);
  return p.xh + p.ix + 2 * p.w + p.part + p.wh;
}

bool tc_prologue_ok(const TcPrologue &pro, int K, const void *x, long ldx) {
  if (pro.kind == kTcProNone) return true;
  if (K > tc::kProMaxK || ldx % 4 || (reinterpret_cast<uintptr_t>(x) & 15)) return false;
  if (pro.kind == kTcProRms) return pro.w && (reinterpret_cast<uintptr_t>(pro.w) & 15) == 0 && ldx >= K;
  return pro.kind == kTcProSwiglu && ldx >= 2L * K;
}

cudaError_t launch_qgemm_tc(int wtype, const void *w, int M, int N, int K, const void *x, int xdt, long ldx, void *c,
                            int cdt, long ldc, int accumulate, void *ws, int *err, cudaStream_t s,
                            const TcPrologue *pro) {
  using namespace tc;
  const TcPlan pl = tc_plan(wtype, M, N, K);
  const bool dq = wtype == TCB_Q4_K;
  if (pl.pairs <= 0) return cudaErrorInvalidConfiguration;
  const int nsb = K / 256;
  uint8_t *p = static_cast<uint8_t *>(ws);
  __half *xh = reinterpret_cast<__half *>(p);
  float *ix = reinterpret_cast<float *>(p + pl.xh);
  float *mw = reinterpret_cast<float *>(p + pl.xh + pl.ix);
  float *iw = reinterpret_cast<float *>(p + pl.xh + pl.ix + pl.w);
  float *part = pl.ksplit > 1 ? reinterpret_cast<float *>(p + pl.xh + pl.ix + 2 * pl.w) : nullptr;
  __half *wh = dq ? nullptr : reinterpret_cast<__half *>(p + pl.xh + pl.ix + 2 * pl.w + pl.part);

  TcArgs a{};
  auto enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {kBK, (cuuint32_t)tc2::kRows}, es[2] = {1, 1};
    if (enc(&a.ta, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  if (dq) {
    const size_t rb = (size_t)nsb * kRawPitch;
    cuuint64_t dims[2] = {(cuuint64_t)rb, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)rb};
    cuuint32_t box[2] = {kRawPitch, (cuuint32_t)tc2::kRows}, es[2] = {1, 1};
    if (enc(&a.tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  } else {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {kBK, (cuuint32_t)tc2::kRows}, es[2] = {1, 1};
    if (enc(&a.tw, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, wh, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  a.mw = mw;
  a.iw = iw;
  a.ix = ix;
  a.c = c;
  a.ldc = ldc;
  a.cdt = cdt;
  a.accumulate = accumulate;
  a.M = M;
  a.N = N;
  a.nsb = nsb;
  a.ksplit = pl.ksplit;
  a.sbper = pl.sbper;
  a.part = part;
  a.err = err;

  const uint8_t *wb = static_cast<const uint8_t *>(w);
  const bool fused = pro && pro->kind != kTcProNone;
  if (fused && (xdt != TCB_F32 || !tc_prologue_ok(*pro, K, x, ldx))) return cudaErrorInvalidValue;
  if (dq) {
    // activation rows (unless the prologue kernel converts them) and the
    // weight rows' multipliers
    k_tc_prep<<<(fused ? 0 : M) + (N + 7) / 8, 256, 0, s>>>(x, xdt, ldx, fused ? 0 : M, K, xh, ix, wb, N, nsb, mw,
                                                             iw, 1);
  } else {
    const size_t rb = (size_t)nsb * 256 / block_elems(wtype) * block_bytes(wtype);
    switch (wtype) {
    case TCB_Q6_K: k_tc_wdeq<TCB_Q6_K><<<N, 256, rb, s>>>(wb, N, K, wh, iw); break;
    case TCB_Q8_0: k_tc_wdeq<TCB_Q8_0><<<N, 256, rb, s>>>(wb, N, K, wh, iw); break;
    default: k_tc_wdeq<TCB_Q4_0><<<N, 256, rb, s>>>(wb, N, K, wh, iw); break;
    }
    if (!fused) k_tc_prep<<<M, 256, 0, s>>>(x, xdt, ldx, M, K, xh, ix, nullptr, N, nsb, mw, iw, 0);
  }
  if (fused) {
    const float *xf = static_cast<const float *>(x);
    const int ng = (K / 8 + 255) / 256, perm = dq ? 1 : 0;
    if (ng <= 2)
      k_tc_prep_pro<2><<<M, 256, 0, s>>>(xf, ldx, K, pro->kind, pro->w, pro->eps, xh, ix, perm);
    else if (ng <= 4)
      k_tc_prep_pro<4><<<M, 256, 0, s>>>(xf, ldx, K, pro->kind, pro->w, pro->eps, xh, ix, perm);
    else
      k_tc_prep_pro<8><<<M, 256, 0, s>>>(xf, ldx, K, pro->kind, pro->w, pro->eps, xh, ix, perm);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  // persistent pairs: as many clusters as fit at once, at most one per work unit
  const int units = pl.tiles * pl.ksplit;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = 2;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  cfg.stream = s;
  cfg.gridDim = dim3(2 * (units < pl.pairs ? units : pl.pairs));
  cfg.blockDim = dim3(tc2::kThreads);
  cfg.dynamicSmemBytes = tc2::kSmem;
  e = dq ? cudaLaunchKernelEx(&cfg, tc2::k_qgemm_tc2<true>, a) : cudaLaunchKernelEx(&cfg, tc2::k_qgemm_tc2<false>, a);
  if (e != cudaSuccess || pl.ksplit == 1) return e;
  const size_t total = (size_t)M * N;
  const int blocks = (int)((total + 255) / 256 < 148 * 8 ? (total + 255) / 256 : 148 * 8);
  tc2::k_tc_reduce<<<blocks, 256, 0, s>>>(part, pl.ksplit, M, N, c, cdt, ldc, accumulate);
  return cudaGetLastError();
}

}  // namespace tcb
