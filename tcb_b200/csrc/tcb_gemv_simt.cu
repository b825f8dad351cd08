// tcb_gemv_simt.cu - portable quantized matvec kernels (sm_100a SIMT):
//  * the float path for any shape whose rows are 2/4-byte aligned
//    (c (+)= x . dequant(w)^T, TR tensor/cpu_quant.go:47-160), and
//  * the int8-activation path (quantise x per weight block, integer block
//    dots, block-ordered fold; TR tensor/cpu_quant_q8.go), bit-exact with
//    TR's CPU kernels.
//
// One warp per weight row; lanes split the row's blocks, the activation
// rows (x) sit in shared memory as f32 when they fit.  Outputs are reduced
// in a fixed order (warp butterfly), no atomics: results are the same on
// every run and for every grid size.
#include "tcb_common.cuh"
#include "tcb_launch.h"
#include "tcb_simt.cuh"

namespace tcb {

template <int W, int MC, bool XSM>
__global__ void __launch_bounds__(kWarps * 32) k_qgemm_simt(const uint8_t *__restrict__ w, int N, int K,
                                                            const void *__restrict__ x, int xdt, long ldx, void *c,
                                                            int cdt, long ldc, int accumulate) {
  extern __shared__ float xs[];
  const long rowBytes = (long)K / Fmt<W>::E * Fmt<W>::B;
  if constexpr (XSM) {
    for (int i = threadIdx.x; i < MC * K; i += blockDim.x) {
      int m = i / K;
      const char *row = static_cast<const char *>(x) + (long)m * ldx * (xdt == TCB_F32 ? 4 : 2);
      xs[i] = load_act(row, i - m * K, xdt);
    }
    __syncthreads();
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int n = blockIdx.x * kWarps + warp; n < N; n += gridDim.x * kWarps) {
    float acc[MC];
#pragma unroll
    for (int m = 0; m < MC; m++) acc[m] = 0.0f;
    const uint8_t *row = w + (long)n * rowBytes;
    if constexpr (XSM) lane_row_float<W, MC>(row, K, lane, XSmem{xs, K}, acc);
    else lane_row_float<W, MC>(row, K, lane, XGlobal{x, ldx, xdt}, acc);
#pragma unroll
    for (int m = 0; m < MC; m++) {
      float v = warp_sum(acc[m]);
      if (lane == 0) store_out(c, (long)m * ldc + n, cdt, v, accumulate != 0);
    }
  }
}

template <int W, int MC>
static cudaError_t launch_simt_mc(const void *w, int N, int K, const void *x, int xdt, long ldx, void *c, int cdt,
                                  long ldc, int accumulate, int sms, cudaStream_t s) {
  const uint8_t *p = static_cast<const uint8_t *>(w);
  int rowsPerCta = kWarps;
  long ctas = (N + rowsPerCta - 1) / rowsPerCta;
  size_t smem = (size_t)MC * K * sizeof(float);
  if (smem <= 160 * 1024) {
    // enough CTAs to fill every SM twice; each stages x once
    long cap = (long)sms * (smem > 100 * 1024 ? 1 : 2);
    int g = (int)(ctas < cap ? ctas : cap);
    auto kern = k_qgemm_simt<W, MC, true>;
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
    }
    kern<<<g, kWarps * 32, smem, s>>>(p, N, K, x, xdt, ldx, c, cdt, ldc, accumulate);
  } else {
    long cap = (long)sms * 8;
    int g = (int)(ctas < cap ? ctas : cap);
    k_qgemm_simt<W, MC, false><<<g, kWarps * 32, 0, s>>>(p, N, K, x, xdt, ldx, c, cdt, ldc, accumulate);
  }
  return cudaGetLastError();
}

template <int W>
static cudaError_t launch_simt_w(const void *w, int M, int N, int K, const void *x, int xdt, long ldx, void *c,
                                 int cdt, long ldc, int accumulate, int sms, cudaStream_t s) {
  const size_t xel = xdt == TCB_F32 ? 4 : 2, cel = cdt == TCB_F32 ? 4 : 2;
  for (int m0 = 0; m0 < M; m0 += 8) {
    int mc = M - m0 < 8 ? M - m0 : 8;
    const void *xm = static_cast<const char *>(x) + (size_t)m0 * ldx * xel;
    void *cm = static_cast<char *>(c) + (size_t)m0 * ldc * cel;
    cudaError_t e;
    switch (mc) {
    case 1: e = launch_simt_mc<W, 1>(w, N, K, xm, xdt, ldx, cm, cdt, ldc, accumulate, sms, s); break;
    case 2: e = launch_simt_mc<W, 2>(w, N, K, xm, xdt, ldx, cm, cdt, ldc, accumulate, sms, s); break;
    case 3: e = launch_simt_mc<W, 3>(w, N, K, xm, xdt, ldx, cm, cdt, ldc, accumulate, sms, s); break;
    case 4: e = launch_simt_mc<W, 4>(w, N, K, xm, xdt, ldx, cm, cdt, ldc, accumulate, sms, s); break;
    case 5: e = launch_simt_mc<W, 5>(w, N, K, xm, xdt, ldx, cm, cdt, ldc, accumulate, sms, s); break;
    case 6: e = launch_simt_mc<W, 6>(w, N, K, xm, xdt, ldx, cm, cdt, ldc, accumulate, sms, s); break;
    case 7: e = launch_simt_mc<W, 7>(w, N, K, xm, xdt, ldx, cm, cdt, ldc, accumulate, sms, s); break;
    default: e = launch_simt_mc<W, 8>(w, N, K, xm, xdt, ldx, cm, cdt, ldc, accumulate, sms, s); break;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_qgemm_simt(int wtype, const void *w, int M, int N, int K, const void *x, int xdt, long ldx,
                              void *c, int cdt, long ldc, int accumulate, int sms, cudaStream_t s) {
  switch (wtype) {
  case TCB_Q8_0: return launch_simt_w<TCB_Q8_0>(w, M, N, K, x, xdt, ldx, c, cdt, ldc, accumulate, sms, s);
  case TCB_Q4_0: return launch_simt_w<TCB_Q4_0>(w, M, N, K, x, xdt, ldx, c, cdt, ldc, accumulate, sms, s);
  case TCB_Q4_K: return launch_simt_w<TCB_Q4_K>(w, M, N, K, x, xdt, ldx, c, cdt, ldc, accumulate, sms, s);
  case TCB_Q6_K: return launch_simt_w<TCB_Q6_K>(w, M, N, K, x, xdt, ldx, c, cdt, ldc, accumulate, sms, s);
  }
  return cudaErrorInvalidValue;
}

// ---- int8-activation path ----------------------------------------------

size_t act8_scratch_bytes(int M, int K, int blk) {
  size_t q = (size_t)M * K, nb = (size_t)M * (K / blk);
  auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
  return up(q) + up(nb * 4) + up((size_t)M * (K / 16) * 2) + up(nb);
}

Act8Scratch act8_scratch_carve(void *base, int M, int K, int blk) {
  auto up = [](size_t v) { return (v + 255) & ~(size_t)255; };
  char *p = static_cast<char *>(base);
  size_t q = (size_t)M * K, nb = (size_t)M * (K / blk);
  Act8Scratch s;
  s.q8 = reinterpret_cast<int8_t *>(p);
  p += up(q);
  s.d8 = reinterpret_cast<float *>(p);
  p += up(nb * 4);
  s.bs = reinterpret_cast<int16_t *>(p);
  p += up((size_t)M * (K / 16) * 2);
  s.flags = reinterpret_cast<uint8_t *>(p);
  return s;
}

// quantizeQ8 (TR tensor/cpu_quant_q8.go:39-68), one warp per activation
// block: amax; id = fp32(127/amax) (IEEE division); a zero or non-finite id
// zeroes the block; code = clamp(rint_even(fp32(v*id)), +-127);
// d = fp32(amax/127); bs = int16 sums of 16 codes.  flags = block finite.
template <int BLK>
__global__ void k_act8_quantize(int M, int K, const void *__restrict__ x, int xdt, long ldx, int8_t *q8, float *d8,
                                int16_t *bs, uint8_t *flags) {
  constexpr int PER = BLK / 32;  // elements per lane, contiguous
  const int lane = threadIdx.x & 31;
  const int nbk = K / BLK;
  const long warps = (long)gridDim.x * (blockDim.x >> 5);
  for (long t = blockIdx.x * (long)(blockDim.x >> 5) + (threadIdx.x >> 5); t < (long)M * nbk; t += warps) {
    const int m = (int)(t / nbk), bi = (int)(t - (long)m * nbk);
    const char *row = static_cast<const char *>(x) + (long)m * ldx * (xdt == TCB_F32 ? 4 : 2);
    float v[PER];
    float amax = 0.0f;
    bool fin = true;
#pragma unroll
    for (int i = 0; i < PER; i++) {
      v[i] = load_act(row, (long)bi * BLK + lane * PER + i, xdt);
      float a = fabsf(v[i]);
      amax = a > amax ? a : amax;
      fin = fin && (__fsub_rn(v[i], v[i]) == 0.0f);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float other = __shfl_xor_sync(0xFFFFFFFFu, amax, o);
      amax = other > amax ? other : amax;
    }
    fin = __all_sync(0xFFFFFFFFu, fin);
    const float id = __fdiv_rn(127.0f, amax);
    const bool zero = !(amax > 0.0f) || (__fsub_rn(id, id) != 0.0f);
    int codes[PER];
    int part = 0;
#pragma unroll
    for (int i = 0; i < PER; i++) {
      int q = 0;
      if (!zero) {
        q = __float2int_rn(__fmul_rn(v[i], id));
        q = q > 127 ? 127 : (q < -127 ? -127 : q);
      }
      codes[i] = q;
      part += q;
    }
    int8_t *qo = q8 + (long)m * K + (long)bi * BLK + lane * PER;
#pragma unroll
    for (int i = 0; i < PER; i++) qo[i] = (int8_t)codes[i];
    // sums of 16 consecutive codes
    if constexpr (PER == 8) {
      part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
      if ((lane & 1) == 0) bs[(long)m * (K / 16) + ((long)bi * BLK + lane * PER) / 16] = (int16_t)part;
    } else {
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) part += __shfl_xor_sync(0xFFFFFFFFu, part, o);
      if ((lane & 15) == 0) bs[(long)m * (K / 16) + ((long)bi * BLK + lane) / 16] = (int16_t)part;
    }
    if (lane == 0) {
      d8[(long)m * nbk + bi] = zero ? 0.0f : __fdiv_rn(amax, 127.0f);
      flags[(long)m * nbk + bi] = fin ? 1 : 0;
    }
  }
}

// one block's term of the int path (TR cpu_quant_q8.go:74-116, 378-407):
// integer sums, then each float step rounded on its own.
template <int W>
__device__ __forceinline__ float act8_term(const uint8_t *blk, const int8_t *x, float d8, const int16_t *bs);

template <>
__device__ __forceinline__ float act8_term<TCB_Q4_0>(const uint8_t *b, const int8_t *x, float d8, const int16_t *) {
  int isum = 0;
#pragma unroll
  for (int j = 0; j < 16; j++) {
    int q = b[2 + j];
    isum += ((q & 0xF) - 8) * x[j] + ((q >> 4) - 8) * x[j + 16];
  }
  float t = __fmul_rn(half_exact(ld_u16(b)), d8);
  return __fmul_rn(t, (float)isum);
}

template <>
__device__ __forceinline__ float act8_term<TCB_Q8_0>(const uint8_t *b, const int8_t *x, float d8, const int16_t *) {
  int isum = 0;
#pragma unroll
  for (int j = 0; j < 32; j++) isum += (int)(int8_t)b[2 + j] * x[j];
  float t = __fmul_rn(half_exact(ld_u16(b)), d8);
  return __fmul_rn(t, (float)isum);
}

template <>
__device__ __forceinline__ float act8_term<TCB_Q4_K>(const uint8_t *b, const int8_t *x, float d8, const int16_t *bs) {
  float d = half_exact(ld_u16(b)), dmin = half_exact(ld_u16(b + 2));
  int isum = 0, msum = 0;
#pragma unroll
  for (int g = 0; g < 4; g++) {
    uint32_t sc1, m1, sc2, m2;
    q4k_scale(2 * g, b + 4, sc1, m1);
    q4k_scale(2 * g + 1, b + 4, sc2, m2);
    int s1 = 0, s2 = 0;
    const uint8_t *q = b + 16 + 32 * g;
#pragma unroll 8
    for (int l = 0; l < 32; l++) {
      s1 += (int)(q[l] & 0xF) * x[64 * g + l];
      s2 += (int)(q[l] >> 4) * x[64 * g + 32 + l];
    }
    isum += (int)sc1 * s1 + (int)sc2 * s2;
    msum += (int)m1 * (int)(int16_t)(bs[4 * g] + bs[4 * g + 1]) + (int)m2 * (int)(int16_t)(bs[4 * g + 2] + bs[4 * g + 3]);
  }
  float u = __fmul_rn(d, (float)isum), v = __fmul_rn(dmin, (float)msum);
  return __fmul_rn(__fsub_rn(u, v), d8);
}

template <>
__device__ __forceinline__ float act8_term<TCB_Q6_K>(const uint8_t *b, const int8_t *x, float d8, const int16_t *bs) {
  float d = half_exact(ld_u16(b + 208));
  int isum = 0, msum = 0;
#pragma unroll
  for (int n = 0; n < 2; n++) {
#pragma unroll 8
    for (int l = 0; l < 32; l++) {
      uint32_t a = b[64 * n + l], a2 = b[64 * n + 32 + l], h = b[128 + 32 * n + l];
      int q1 = (int)((a & 0xFu) | ((h & 3u) << 4)), q2 = (int)((a2 & 0xFu) | (((h >> 2) & 3u) << 4));
      int q3 = (int)((a >> 4) | (((h >> 4) & 3u) << 4)), q4 = (int)((a2 >> 4) | (((h >> 6) & 3u) << 4));
      int is = l >> 4;
      const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192 + 8 * n);
      isum += sc[is] * q1 * x[128 * n + l] + sc[is + 2] * q2 * x[128 * n + l + 32] +
              sc[is + 4] * q3 * x[128 * n + l + 64] + sc[is + 6] * q4 * x[128 * n + l + 96];
    }
  }
  const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192);
#pragma unroll
  for (int j = 0; j < 16; j++) msum += (int)sc[j] * (int)bs[j];
  float t = __fmul_rn(d, (float)(isum - 32 * msum));
  return __fmul_rn(t, d8);
}

// Warp per weight row n, every activation row m: a row with a NaN/Inf
// takes the float path; otherwise lane i takes blocks i, i+32, ... and
// lane 0 folds the block terms in block order (acc = fp32(acc + term)).
template <int W>
__global__ void __launch_bounds__(kWarps * 32) k_act8_dot(const uint8_t *__restrict__ w, int M, int N, int K,
                                                          const int8_t *__restrict__ q8, const float *__restrict__ d8,
                                                          const int16_t *__restrict__ bs,
                                                          const uint8_t *__restrict__ flags, const void *x, int xdt,
                                                          long ldx, void *c, int cdt, long ldc, int accumulate) {
  constexpr int E = Fmt<W>::E, B = Fmt<W>::B;
  __shared__ float terms[kWarps][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nbk = K / E;
  const long rowBytes = (long)nbk * B;
  for (int n = blockIdx.x * kWarps + warp; n < N; n += gridDim.x * kWarps) {
    const uint8_t *row = w + (long)n * rowBytes;
    for (int m = 0; m < M; m++) {
      bool fin = true;
      for (int i = lane; i < nbk; i += 32) fin = fin && flags[(long)m * nbk + i];
      fin = __all_sync(0xFFFFFFFFu, fin);
      float r;
      if (!fin) {
        float acc[1] = {0.0f};
        const char *xm = static_cast<const char *>(x) + (long)m * ldx * (xdt == TCB_F32 ? 4 : 2);
        lane_row_float<W, 1>(row, K, lane, XGlobal{xm, 0, xdt}, acc);
        r = warp_sum(acc[0]);
      } else {
        float acc = 0.0f;
        for (int b0 = 0; b0 < nbk; b0 += 32) {
          const int b = b0 + lane;
          float t = 0.0f;
          if (b < nbk)
            t = act8_term<W>(row + (long)b * B, q8 + (long)m * K + (long)b * E, d8[(long)m * nbk + b],
                             bs + (long)m * (K / 16) + (long)b * (E / 16));
          terms[warp][lane] = t;
          __syncwarp();
          if (lane == 0) {
            const int cnt = nbk - b0 < 32 ? nbk - b0 : 32;
            for (int i = 0; i < cnt; i++) acc = __fadd_rn(acc, terms[warp][i]);
          }
          __syncwarp();
        }
        r = acc;
      }
      if (lane == 0) store_out(c, (long)m * ldc + n, cdt, r, accumulate != 0);
    }
  }
}

cudaError_t launch_act8_quantize(int blk, int M, int K, const void *x, int xdt, long ldx, const Act8Scratch &sc,
                                 int sms, cudaStream_t s) {
  long work = (long)M * (K / blk);
  long ctas = (work + 7) / 8;
  long cap = (long)sms * 8;
  int g = (int)(ctas < 1 ? 1 : ctas < cap ? ctas : cap);
  if (blk == 32) k_act8_quantize<32><<<g, 256, 0, s>>>(M, K, x, xdt, ldx, sc.q8, sc.d8, sc.bs, sc.flags);
  else k_act8_quantize<256><<<g, 256, 0, s>>>(M, K, x, xdt, ldx, sc.q8, sc.d8, sc.bs, sc.flags);
  return cudaGetLastError();
}

cudaError_t launch_act8_dot(int wtype, const void *w, int M, int N, int K, const Act8Scratch &sc, const void *x,
                            int xdt, long ldx, void *c, int cdt, long ldc, int accumulate, int sms,
                            cudaStream_t s) {
  long ctas = (N + kWarps - 1) / kWarps;
  long cap = (long)sms * 8;
  int g = (int)(ctas < cap ? ctas : cap);
  const uint8_t *p = static_cast<const uint8_t *>(w);
#define TCB_ACT8(WT) \
  k_act8_dot<WT><<<g, kWarps * 32, 0, s>>>(p, M, N, K, sc.q8, sc.d8, sc.bs, sc.flags, x, xdt, ldx, c, cdt, ldc, accumulate)
  switch (wtype) {
  case TCB_Q8_0: TCB_ACT8(TCB_Q8_0); break;
  case TCB_Q4_0: TCB_ACT8(TCB_Q4_0); break;
  case TCB_Q4_K: TCB_ACT8(TCB_Q4_K); break;
  case TCB_Q6_K: TCB_ACT8(TCB_Q6_K); break;
  default: return cudaErrorInvalidValue;
  }
#undef TCB_ACT8
  return cudaGetLastError();
}

}  // namespace tcb
