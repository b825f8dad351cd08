// tcb_common.cuh - block layouts, exact element conversions and small
// helpers shared by the quantized-path kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tcb.h"

namespace tcb {

// GGUF block layouts (TR tensor/quant.go:23-29):
//   Q8_0: fp16 d, 32 x int8                       = 34 B / 32 elements
//   Q4_0: fp16 d, 16 B of nibbles                 = 18 B / 32 elements
//   Q4_K: fp16 d, fp16 dmin, 12 B scales, 128 B    = 144 B / 256 elements
//   Q6_K: ql 128 B, qh 64 B, int8 sc[16], fp16 d   = 210 B / 256 elements
template <int W> struct Fmt;
template <> struct Fmt<TCB_Q8_0> { static constexpr int E = 32, B = 34; };
template <> struct Fmt<TCB_Q4_0> { static constexpr int E = 32, B = 18; };
template <> struct Fmt<TCB_Q4_K> { static constexpr int E = 256, B = 144; };
template <> struct Fmt<TCB_Q6_K> { static constexpr int E = 256, B = 210; };

__host__ __device__ inline int block_elems(int w) {
  return (w == TCB_Q8_0 || w == TCB_Q4_0) ? 32 : (w == TCB_Q4_K || w == TCB_Q6_K) ? 256 : 0;
}
__host__ __device__ inline int block_bytes(int w) {
  return w == TCB_Q8_0 ? 34 : w == TCB_Q4_0 ? 18 : w == TCB_Q4_K ? 144 : w == TCB_Q6_K ? 210 : 0;
}

__device__ __forceinline__ float bits_f(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ uint32_t f_bits(float f) { return __float_as_uint(f); }

// little-endian u16 at a 2-byte aligned address
__device__ __forceinline__ uint32_t ld_u16(const uint8_t *p) {
  return *reinterpret_cast<const uint16_t *>(p);
}

// IEEE half -> float with the NaN payload kept (TR tensor/cpu_dtype.go:126-145).
// cvt.f32.f16 is exact for every finite value; NaN/Inf are rebuilt by hand
// because the hardware conversion canonicalises NaN.
__device__ __forceinline__ float half_exact(uint32_t h) {
  float v = __half2float(__ushort_as_half((unsigned short)h));
  if ((h & 0x7C00u) == 0x7C00u) v = bits_f(((h & 0x8000u) << 16) | 0x7F800000u | ((h & 0x3FFu) << 13));
  return v;
}

// x86 result for a NaN (TR gpu/kernel_quant.go:13-17): first NaN operand,
// quieted; with no NaN operand the default NaN 0xFFC00000.
__device__ __forceinline__ float nan_rule(float r, float a, float b) {
  if (r == r) return r;
  if (a != a) return bits_f(f_bits(a) | 0x00400000u);
  if (b != b) return bits_f(f_bits(b) | 0x00400000u);
  return bits_f(0xFFC00000u);
}
__device__ __forceinline__ float mulx(float a, float b) { return nan_rule(__fmul_rn(a, b), a, b); }
__device__ __forceinline__ float subx(float a, float b) { return nan_rule(__fsub_rn(a, b), a, b); }

// f32 -> bf16 / f16 exactly as TR's Cast (tensor/cpu_dtype.go:73-80, 87-126):
// round to nearest even; NaN keeps its sign and top payload, quieted.
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  uint32_t b = f_bits(f);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((b >> 16) | 0x0040u);
  b += 0x7FFFu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}
__device__ __forceinline__ uint16_t f32_to_f16(float f) {
  uint32_t b = f_bits(f);
  uint32_t sign = (b >> 16) & 0x8000u;
  int ex = (int)((b >> 23) & 0xFFu);
  uint32_t man = b & 0x7FFFFFu;
  if (ex == 0xFF) return (uint16_t)(man ? (sign | 0x7E00u | (man >> 13)) : (sign | 0x7C00u));
  int e = ex - 127 + 15;
  if (e >= 0x1F) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    uint32_t sh = (uint32_t)(14 - e);
    uint32_t m = man >> sh, rest = man & ((1u << sh) - 1u), half = 1u << (sh - 1u);
    if (rest > half || (rest == half && (m & 1u))) m++;
    return (uint16_t)(sign | m);
  }
  uint32_t m = man >> 13, rest = man & 0x1FFFu;
  uint32_t out = sign | ((uint32_t)e << 10) | m;
  if (rest > 0x1000u || (rest == 0x1000u && (m & 1u))) out++;  // may carry into Inf: correct
  return (uint16_t)out;
}

__device__ __forceinline__ float bf16_to_f32(uint16_t h) { return bits_f((uint32_t)h << 16); }

// activation element i of a row (dtype F32 / BF16 / F16) as f32
__device__ __forceinline__ float load_act(const void *row, long i, int dt) {
  if (dt == TCB_F32) return static_cast<const float *>(row)[i];
  uint16_t h = static_cast<const uint16_t *>(row)[i];
  return dt == TCB_BF16 ? bf16_to_f32(h) : half_exact(h);
}

// store one output: f32 math, one rounding into the destination type.
// accumulate: dst = round(f32(dst) + v)  (TR's temp-f32 write-back,
// gpu/backend_quant.go:41-47)
__device__ __forceinline__ void store_out(void *c, long i, int dt, float v, bool accumulate) {
  if (dt == TCB_F32) {
    float *p = static_cast<float *>(c) + i;
    *p = accumulate ? __fadd_rn(*p, v) : v;
    return;
  }
  uint16_t *p = static_cast<uint16_t *>(c) + i;
  if (dt == TCB_BF16) {
    float old = accumulate ? bf16_to_f32(*p) : 0.0f;
    *p = f32_to_bf16(accumulate ? __fadd_rn(old, v) : v);
  } else {
    float old = accumulate ? half_exact(*p) : 0.0f;
    *p = f32_to_f16(accumulate ? __fadd_rn(old, v) : v);
  }
}

// the old value of one output as f32 (for accumulation), read ahead of use
__device__ __forceinline__ float load_out(const void *c, long i, int dt) {
  if (dt == TCB_F32) return static_cast<const float *>(c)[i];
  const uint16_t h = static_cast<const uint16_t *>(c)[i];
  return dt == TCB_BF16 ? bf16_to_f32(h) : half_exact(h);
}

// store one output whose old value (if accumulating) was loaded earlier
__device__ __forceinline__ void store_out_old(void *c, long i, int dt, float v, bool accumulate, float old) {
  const float r = accumulate ? __fadd_rn(old, v) : v;
  if (dt == TCB_F32) static_cast<float *>(c)[i] = r;
  else if (dt == TCB_BF16) static_cast<uint16_t *>(c)[i] = f32_to_bf16(r);
  else static_cast<uint16_t *>(c)[i] = f32_to_f16(r);
}

// Q4_K packed 6-bit scale/min of sub-block j (TR tensor/quant.go:158-163)
__device__ __forceinline__ void q4k_scale(int j, const uint8_t *q, uint32_t &sc, uint32_t &m) {
  if (j < 4) {
    sc = q[j] & 63u;
    m = q[j + 4] & 63u;
  } else {
    sc = (q[j + 4] & 0xFu) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

}  // namespace tcb
