// tcb_dequant.cuh - exact dequantisation of one element of a GGUF block,
// with the same fp32 operations, in the same order, as TR's CPU dequant
// (tensor/quant.go:139-204) and its x86 NaN rule (gpu/kernel_quant.go:13-17).
// Internal to libtcb.
#pragma once

#include "tcb_common.cuh"

namespace tcb {

// element j of the block at b
template <int W>
__device__ __forceinline__ float dequant_elem(const uint8_t *b, int j);

template <>
__device__ __forceinline__ float dequant_elem<TCB_Q8_0>(const uint8_t *b, int j) {
  return mulx((float)(int8_t)b[2 + j], half_exact(ld_u16(b)));
}

template <>
__device__ __forceinline__ float dequant_elem<TCB_Q4_0>(const uint8_t *b, int j) {
  uint32_t q = b[2 + (j & 15)];
  int code = (int)((j < 16 ? q : q >> 4) & 0xFu) - 8;
  return mulx((float)code, half_exact(ld_u16(b)));
}

template <>
__device__ __forceinline__ float dequant_elem<TCB_Q4_K>(const uint8_t *b, int j) {
  int g = j >> 6, hi = (j >> 5) & 1, l = j & 31;
  uint32_t sc, m;
  q4k_scale(2 * g + hi, b + 4, sc, m);
  float d1 = mulx(half_exact(ld_u16(b)), (float)sc);
  float m1 = mulx(half_exact(ld_u16(b + 2)), (float)m);
  uint32_t q = b[16 + 32 * g + l];
  float code = (float)(hi ? (q >> 4) : (q & 0xFu));
  return subx(mulx(d1, code), m1);
}

template <>
__device__ __forceinline__ float dequant_elem<TCB_Q6_K>(const uint8_t *b, int j) {
  int n = j >> 7, c = (j >> 5) & 3, l = j & 31;
  uint32_t low = (b[64 * n + l + 32 * (c & 1)] >> (4 * (c >> 1))) & 0xFu;
  uint32_t high = (b[128 + 32 * n + l] >> (2 * c)) & 3u;
  int code = (int)(low | (high << 4)) - 32;
  float s = (float)(int8_t)b[192 + 8 * n + (l >> 4) + 2 * c];
  return mulx(mulx(half_exact(ld_u16(b + 208)), s), (float)code);
}

}  // namespace tcb
