// tcb_simt.cuh - per-lane SIMT pieces of the float path (portable
// kernel, and the non-finite fallback of the tensor-core kernel).
#pragma once

#include "tcb_common.cuh"

namespace tcb {

constexpr int kWarps = 8;  // rows in flight per CTA

// activation access: rows of x staged in shared memory as f32, or read
// (and converted) from global memory when they do not fit
struct XSmem {
  const float *xs;
  int K;
  __device__ __forceinline__ float operator()(int m, int k) const { return xs[m * K + k]; }
};
struct XGlobal {
  const void *x;
  long ldx;
  int dt;
  __device__ __forceinline__ float operator()(int m, int k) const {
    const char *row = static_cast<const char *>(x) + (long)m * ldx * (dt == TCB_F32 ? 4 : 2);
    return load_act(row, k, dt);
  }
};

// ---- float path: per-lane share of one weight row ----------------------
// Dequantised values are formed with one rounding (exact products), as in
// TR's dequant; the dot itself is a plain fp32 FMA chain (tolerance parity).

template <int W, int MC, class X>
__device__ __forceinline__ void lane_row_float(const uint8_t *row, int K, int lane, const X &xv, float *acc);

template <int MC, class X>
__device__ __forceinline__ void lane_row_float_q8_0(const uint8_t *row, int K, int lane, const X &xv, float *acc) {
  const int nb = K / 32, s = lane & 3;
  for (int b = lane >> 2; b < nb; b += 8) {
    const uint8_t *blk = row + (long)b * 34;
    float d = half_exact(ld_u16(blk));
#pragma unroll
    for (int i = 0; i < 8; i++) {
      float v = (float)(int8_t)blk[2 + 8 * s + i] * d;
      int e = 32 * b + 8 * s + i;
#pragma unroll
      for (int m = 0; m < MC; m++) acc[m] = fmaf(xv(m, e), v, acc[m]);
    }
  }
}

template <int MC, class X>
__device__ __forceinline__ void lane_row_float_q4_0(const uint8_t *row, int K, int lane, const X &xv, float *acc) {
  const int nb = K / 32, s = lane & 3;
  for (int b = lane >> 2; b < nb; b += 8) {
    const uint8_t *blk = row + (long)b * 18;
    float d = half_exact(ld_u16(blk));
#pragma unroll
    for (int i = 0; i < 4; i++) {
      uint32_t q = blk[2 + 4 * s + i];
      float lo = (float)((int)(q & 0xFu) - 8) * d, hi = (float)((int)(q >> 4) - 8) * d;
      int e = 32 * b + 4 * s + i;
#pragma unroll
      for (int m = 0; m < MC; m++) {
        acc[m] = fmaf(xv(m, e), lo, acc[m]);
        acc[m] = fmaf(xv(m, e + 16), hi, acc[m]);
      }
    }
  }
}

template <int MC, class X>
__device__ __forceinline__ void lane_row_float_q4_k(const uint8_t *row, int K, int lane, const X &xv, float *acc) {
  const int nb = K / 256, s = lane & 7, g = s >> 1, l0 = 16 * (s & 1);
  for (int b = lane >> 3; b < nb; b += 4) {
    const uint8_t *blk = row + (long)b * 144;
    float d = half_exact(ld_u16(blk)), dmin = half_exact(ld_u16(blk + 2));
    uint32_t sc1, m1, sc2, m2;
    q4k_scale(2 * g, blk + 4, sc1, m1);
    q4k_scale(2 * g + 1, blk + 4, sc2, m2);
    float d1 = d * (float)sc1, mm1 = dmin * (float)m1, d2 = d * (float)sc2, mm2 = dmin * (float)m2;
    const uint32_t *q32 = reinterpret_cast<const uint32_t *>(blk + 16 + 32 * g + l0);
#pragma unroll
    for (int wd = 0; wd < 4; wd++) {
      uint32_t qw = q32[wd];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        uint32_t q = (qw >> (8 * i)) & 0xFFu;
        float lo = fmaf(d1, (float)(q & 0xFu), -mm1), hi = fmaf(d2, (float)(q >> 4), -mm2);
        int e = 256 * b + 64 * g + l0 + 4 * wd + i;
#pragma unroll
        for (int m = 0; m < MC; m++) {
          acc[m] = fmaf(xv(m, e), lo, acc[m]);
          acc[m] = fmaf(xv(m, e + 32), hi, acc[m]);
        }
      }
    }
  }
}

template <int MC, class X>
__device__ __forceinline__ void lane_row_float_q6_k(const uint8_t *row, int K, int lane, const X &xv, float *acc) {
  const int nb = K / 256, s = lane & 7, n2 = s >> 2, l0 = 8 * (s & 3), is = l0 >> 4;
  for (int b = lane >> 3; b < nb; b += 4) {
    const uint8_t *blk = row + (long)b * 210;
    float d = half_exact(ld_u16(blk + 208));
    float ds[4];
#pragma unroll
    for (int c = 0; c < 4; c++) ds[c] = d * (float)(int8_t)blk[192 + 8 * n2 + is + 2 * c];
#pragma unroll
    for (int i = 0; i < 8; i++) {
      int l = l0 + i;
      uint32_t a = blk[64 * n2 + l], a2 = blk[64 * n2 + 32 + l], h = blk[128 + 32 * n2 + l];
      int q[4] = {(int)((a & 0xFu) | ((h & 3u) << 4)) - 32, (int)((a2 & 0xFu) | (((h >> 2) & 3u) << 4)) - 32,
                  (int)((a >> 4) | (((h >> 4) & 3u) << 4)) - 32, (int)((a2 >> 4) | (((h >> 6) & 3u) << 4)) - 32};
#pragma unroll
      for (int c = 0; c < 4; c++) {
        float v = __fmul_rn(ds[c], (float)q[c]);
        int e = 256 * b + 128 * n2 + l + 32 * c;
#pragma unroll
        for (int m = 0; m < MC; m++) acc[m] = fmaf(xv(m, e), v, acc[m]);
      }
    }
  }
}

template <int W, int MC, class X>
__device__ __forceinline__ void lane_row_float(const uint8_t *row, int K, int lane, const X &xv, float *acc) {
  if constexpr (W == TCB_Q8_0) lane_row_float_q8_0<MC>(row, K, lane, xv, acc);
  else if constexpr (W == TCB_Q4_0) lane_row_float_q4_0<MC>(row, K, lane, xv, acc);
  else if constexpr (W == TCB_Q4_K) lane_row_float_q4_k<MC>(row, K, lane, xv, acc);
  else lane_row_float_q6_k<MC>(row, K, lane, xv, acc);
}

}  // namespace tcb
