// tcb_matvec.cu - batch-1 quantized matvec on sm_100a tensor cores.
//
//   y[n] (+)= sum_k x[k] * dequant(W)[n, k]     W: [N, K] GGUF blocks
//
// Design (memory-bound at batch 1: every weight byte is read once):
//  * Weights stream from HBM into shared memory through 2-D TMA tensor
//    copies (cp.async.bulk.tensor, 8-byte elements, no multicast) issued by
//    a producer warp: a stage is 16 rows x 2-4 boxes of ~1.1-1.7 KB per row,
//    a few TMA instructions per ~40-70 KB, so DRAM sees long runs and the copy
//    engine few requests; the box width is padded so the staged rows fall on
//    different shared-memory banks; rows past N and bytes past the row end
//    arrive as zeros.  Sixteen consumer warps split each stage's blocks.
//  * Launched with programmatic stream serialization: the producer starts
//    streaming weights while the previous kernel of the stream drains; the
//    consumers wait for it (griddepcontrol.wait) before reading x or
//    writing c.  Weights are only read, never written, by these kernels.
//  * The dot products run on the int8 tensor-core path (mma.sync
//    m16n8k32 / m16n8k16, u8/s8 -> s32): the weight codes are exact small
//    integers, so the A fragment is the raw code bytes after one LOP3 per
//    four codes (no per-element dequantisation).  The 8 columns of the MMA
//    are not batch rows: column j carries scale group j (a Q4_K sub-block,
//    a Q6_K 16-element group, a whole Q8_0/Q4_0 block), so one MMA chain
//    leaves every (row, group) integer dot in its own accumulator and each
//    lane applies the scales of exactly four (row, group) pairs.
//  * Float path: x is split per 32-element group into int8 digits,
//    x ~= sigma * (h + l/254), |digits| <= 127, sigma = amax/127; the digit
//    products are exact int32 and recombine exactly (relative error of the
//    x representation <= 1/(2*127*254) of the group maximum, ~4e-5 rel-L2
//    on the outputs).  A row of x with
//    NaN/Inf takes an fp32 SIMT path instead (NaN/Inf propagate as in TR).
//  * Int8-activation path (TR_quantized_activations): x is quantised with
//    TR's quantizeQ8 and each block term is formed exactly as TR's CPU
//    kernels do, then folded in block order: bit-exact.
//  * Work split: a CTA owns whole 16-row tiles; warp w takes block (or
//    8-block round) w of every chunk, and the sixteen warp
//    partials of a row are added in warp order (float path) or every block
//    term is folded in block order (int8 path) in shared memory.  Results
//    do not depend on the SM count or on timing.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include "tcb_common.cuh"
#include "tcb_matvec.h"
#include "tcb_mv_ptx.cuh"
#include "tcb_simt.cuh"

namespace tcb {
namespace mv {


// ----------------------------------------------------------------- formats
// GRP: elements per scale group (one MMA k); GPB: groups per block; RB:
// blocks per warp work item (a Q8_0/Q4_0 round fills the 8 MMA columns
// with 8 blocks); BPB: blocks per TMA box (box starts 16-byte aligned, 8
// work items per box); BOX8: box width in 8-byte elements, the BPB blocks
// plus padding that makes the staged row pitch 32 or 96 mod 128 bytes;
// NDIG: digits of x on the float path (2 for Q6_K, whose k16 groups take
// twice the MMAs).  A stage is NBOX boxes: 16 work items, one per consumer
// warp.
template <int W> struct Pol;
template <> struct Pol<TCB_Q4_K> { static constexpr int E = 256, B = 144, GRP = 32, GPB = 8, RB = 1, BPB = 8, BOX8 = 148, NBOX = 2, NDIG = 2; };
template <> struct Pol<TCB_Q6_K> { static constexpr int E = 256, B = 210, GRP = 16, GPB = 16, RB = 1, BPB = 8, BOX8 = 212, NBOX = 2, NDIG = 2; };
template <> struct Pol<TCB_Q8_0> { static constexpr int E = 32, B = 34, GRP = 32, GPB = 1, RB = 8, BPB = 32, BOX8 = 140, NBOX = 4, NDIG = 2; };
template <> struct Pol<TCB_Q4_0> { static constexpr int E = 32, B = 18, GRP = 32, GPB = 1, RB = 8, BPB = 64, BOX8 = 148, NBOX = 2, NDIG = 2; };

constexpr int kConsumers = 16;         // compute warps; warp 16 produces, warp 17 finishes

struct Params {
  const uint8_t *w;
  long rowBytes;
  int N, K, nb;
  const void *x;
  int xdt;
  void *c;
  int cdt;
  int accumulate;
  int tiles, cbc, nch;    // 16-row tiles; blocks per chunk (NBOX boxes); chunks per row
  int *err;               // sticky error word (timeouts)
  int S;                  // stages
  int xoff, toff, soff;   // shared-memory offsets: x region, int8 terms, stages
  const void *pf;         // weights of the next kernel of a chain, prefetched into L2 (or nullptr)
  size_t pf_bytes;
  int M;                  // rows of x of this launch (float path: 1 .. MR of the kernel)
  long ldx, ldc;          // row strides of x and c, elements
  int xstride;            // bytes between the x regions of consecutive rows
};

// x region layout (float path): NDIG digit planes of K int8, then per group
// sg (sigma / 254^(NDIG-1)), S (sum of x), Sd (digit sum in recombined units).
// int8 path: q8 codes K int8, d8 per block, bs (int16 sums of 16 codes).
struct XF {
  const int8_t *dig;  // plane p at dig + p*K
  const float *sg, *sx, *sd;
};
struct XQ {
  const int8_t *q;
  const float *d8;
  const int16_t *bs;
};

template <int W, bool ACT8>
__host__ __device__ inline int x_region_bytes(int K) {
  using P = Pol<W>;
  auto up = [](int v) { return (v + 15) & ~15; };
  if (ACT8) return up(K) + up(K / P::E * 4) + up(K / 16 * 2) + 16;
  int ng = K / P::GRP;
  return up(P::NDIG * K) + 3 * up(ng * 4) + 16;
}

// ----------------------------------------------------------------- x prep

// float path: each thread takes 4 consecutive elements (8 threads per
// 32-element group, 4 per 16-element Q6_K group); loads are issued in
// batches of four so the L2 latency is paid once per batch.  Digits are
// rounded with the 1.5*2^23 trick (the integer lands in the low mantissa
// bits, ties to even) and packed with byte permutes.
template <int W>
__device__ void prep_float(const Params &a, uint8_t *xr, int *flag) {
  using P = Pol<W>;
  constexpr int ND = P::NDIG, G = P::GRP, LPG = G / 4, NB = 4;
  constexpr bool NEED_SX = W == TCB_Q4_K;                    // the min term uses sum(x)
  constexpr bool NEED_SD = W == TCB_Q4_0 || W == TCB_Q6_K;  // the code offset uses sum(digits)
  constexpr float MAGIC = 12582912.0f;
  const int K = a.K, ng = K / G;
  auto up = [](int v) { return (v + 15) & ~15; };
  int8_t *dig = reinterpret_cast<int8_t *>(xr);
  float *sg = reinterpret_cast<float *>(xr + up(ND * K));
  float *sx = sg + up(ng * 4) / 4;
  float *sd = sx + up(ng * 4) / 4;
  const int tid = threadIdx.x, nthr = 32 * kConsumers;
  const bool vec = a.xdt == TCB_F32 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0;
  bool fin_all = true;
  for (int base = 0; base < K; base += 4 * nthr * NB) {
    float4 v[NB];
#pragma unroll
    for (int i = 0; i < NB; i++) {
      const int e = base + 4 * (tid + i * nthr);
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < K) {
        if (vec) {
          v[i] = *reinterpret_cast<const float4 *>(static_cast<const float *>(a.x) + e);
        } else {
          v[i].x = load_act(a.x, e, a.xdt);
          v[i].y = load_act(a.x, e + 1, a.xdt);
          v[i].z = load_act(a.x, e + 2, a.xdt);
          v[i].w = load_act(a.x, e + 3, a.xdt);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < NB; i++) {
      const int e = base + 4 * (tid + i * nthr);
      float xv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
      float am = 0.f;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        if ((__float_as_uint(xv[q]) & 0x7F800000u) == 0x7F800000u) {
          fin_all = false;
          xv[q] = 0.f;
        }
        am = fmaxf(am, fabsf(xv[q]));
      }
#pragma unroll
      for (int o = LPG / 2; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xFFFFFFFFu, am, o));
      // y = x * 127/amax in [-127, 127]; tiny groups are lifted by 2^64 so
      // the reciprocal stays finite; sigma * id = 1 to a few ulp
      float id = 0.f, sigma = 0.f;
      if (am > 0.f) {
        const bool tiny = am < 1e-30f;
        const float sc = (tiny ? am * 18446744073709551616.0f : am) * (1.0f / 127.0f);
        id = __frcp_rn(sc) * (tiny ? 18446744073709551616.0f : 1.0f);
        sigma = tiny ? sc * 5.421010862427522e-20f : sc;
      }
      uint32_t bh[4], b1[4], b2[4];
      float fh = 0.f, f1 = 0.f, f2 = 0.f, s = 0.f;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const float y = __fmul_rn(xv[q], id);
        const float t0 = __fadd_rn(y, MAGIC), h = __fsub_rn(t0, MAGIC);
        const float r1 = __fmul_rn(__fsub_rn(y, h), 254.0f);
        const float t1 = __fadd_rn(r1, MAGIC), l1 = __fsub_rn(t1, MAGIC);
        bh[q] = __float_as_uint(t0);
        b1[q] = __float_as_uint(t1);
        if (ND > 2) {
          const float r2 = __fmul_rn(__fsub_rn(r1, l1), 254.0f);
          const float t2 = __fadd_rn(r2, MAGIC);
          b2[q] = __float_as_uint(t2);
          if (NEED_SD) f2 += __fsub_rn(t2, MAGIC);
        }
        if (NEED_SD) {
          fh += h;
          f1 += l1;
        }
        if (NEED_SX) s += xv[q];
      }
      const uint32_t ph = __byte_perm(__byte_perm(bh[0], bh[1], 0x0040), __byte_perm(bh[2], bh[3], 0x0040), 0x5410);
      const uint32_t p1 = __byte_perm(__byte_perm(b1[0], b1[1], 0x0040), __byte_perm(b1[2], b1[3], 0x0040), 0x5410);
      uint32_t p2 = 0;
      if (ND > 2) p2 = __byte_perm(__byte_perm(b2[0], b2[1], 0x0040), __byte_perm(b2[2], b2[3], 0x0040), 0x5410);
#pragma unroll
      for (int o = LPG / 2; o > 0; o >>= 1) {
        if (NEED_SX) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
        if (NEED_SD) {
          fh += __shfl_xor_sync(0xFFFFFFFFu, fh, o);
          f1 += __shfl_xor_sync(0xFFFFFFFFu, f1, o);
          if (ND > 2) f2 += __shfl_xor_sync(0xFFFFFFFFu, f2, o);
        }
      }
      if (e < K) {
        // Q4_0: within a 32-element block, the 4-byte words of elements 4t..
        // and 16+4t.. sit side by side (word 2t and 2t+1), so a lane reads its
        // low- and high-nibble digits with one conflict-free 8-byte load
        int pe = e;
        if constexpr (W == TCB_Q4_0) {
          const int w = (e & 31) >> 2;
          pe = (e & ~31) + 4 * (2 * (w & 3) + (w >> 2));
        }
        *reinterpret_cast<uint32_t *>(dig + pe) = ph;
        *reinterpret_cast<uint32_t *>(dig + K + pe) = p1;
        if (ND > 2) *reinterpret_cast<uint32_t *>(dig + 2 * K + pe) = p2;
        if ((tid & (LPG - 1)) == 0) {
          const int gi = e / G;
          sg[gi] = ND > 2 ? sigma * (1.0f / 64516.0f) : sigma * (1.0f / 254.0f);
          if (NEED_SX) sx[gi] = s;
          if (NEED_SD) sd[gi] = ND > 2 ? fmaf(fmaf(fh, 254.0f, f1), 254.0f, f2) : fmaf(fh, 254.0f, f1);
        }
      }
    }
  }
  if (!fin_all) *flag = 1;
}

// int8 path: TR's quantizeQ8 (tensor/cpu_quant_q8.go:39-68), one warp per
// activation block of E (= weight block) elements.
template <int W>
__device__ void prep_act8(const Params &a, uint8_t *xr, int *flag) {
  using P = Pol<W>;
  constexpr int E = P::E, PER = E / 32;
  const int K = a.K, nbk = K / E;
  auto up = [](int v) { return (v + 15) & ~15; };
  int8_t *q8 = reinterpret_cast<int8_t *>(xr);
  float *d8 = reinterpret_cast<float *>(xr + up(K));
  int16_t *bs = reinterpret_cast<int16_t *>(xr + up(K) + up(nbk * 4));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = kConsumers;
  // the loads of NB of the warp's blocks go out together (one memory round
  // trip per NB blocks, not per block); each block is then quantised as before
  constexpr int NB = PER == 1 ? 8 : 4;
  for (int b0 = warp; b0 < nbk; b0 += nw * NB) {
    float vb[NB][PER];
#pragma unroll
    for (int j = 0; j < NB; j++) {
      const int bj = b0 + j * nw;
#pragma unroll
      for (int i = 0; i < PER; i++) vb[j][i] = bj < nbk ? load_act(a.x, (long)bj * E + lane * PER + i, a.xdt) : 0.f;
    }
#pragma unroll
  for (int j = 0; j < NB; j++) {
    const int bi = b0 + j * nw;
    if (bi >= nbk) break;  // warp-uniform
    float v[PER];
    float amax = 0.0f;
    bool fin = true;
#pragma unroll
    for (int i = 0; i < PER; i++) {
      v[i] = vb[j][i];
      float t = fabsf(v[i]);
      amax = t > amax ? t : amax;
      fin = fin && (__fsub_rn(v[i], v[i]) == 0.0f);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float t = __shfl_xor_sync(0xFFFFFFFFu, amax, o);
      amax = t > amax ? t : amax;
    }
    if (!__all_sync(0xFFFFFFFFu, fin) && lane == 0) *flag = 1;
    const float id = __fdiv_rn(127.0f, amax);
    const bool zero = !(amax > 0.0f) || (__fsub_rn(id, id) != 0.0f);
    int part = 0;
#pragma unroll
    for (int i = 0; i < PER; i++) {
      int q = 0;
      if (!zero) q = max(-127, min(127, __float2int_rn(__fmul_rn(v[i], id))));
      q8[bi * E + lane * PER + i] = (int8_t)q;
      part += q;
    }
    if constexpr (PER == 8) {
      part += __shfl_xor_sync(0xFFFFFFFFu, part, 1);
      if ((lane & 1) == 0) bs[(bi * E + lane * PER) / 16] = (int16_t)part;
    } else {
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) part += __shfl_xor_sync(0xFFFFFFFFu, part, o);
      if ((lane & 15) == 0) bs[(bi * E + lane) / 16] = (int16_t)part;
    }
    if (lane == 0) d8[bi] = zero ? 0.0f : __fdiv_rn(amax, 127.0f);
  }
  }
}


// ----------------------------------------------------------------- format bodies
// A body consumes one work item of a staged chunk (a Q4_K/Q6_K block, or a
// Q8_0/Q4_0 round of 8 blocks) for the tile's 16 rows: rows g and g+8 of
// lane (g = lane/4, t = lane%4).  MMA column c carries scale group c: lane
// g supplies the B operand of column g only, so each lane loads the digits
// of its own group once and masks them with mk[c] = (g == c ? ~0 : 0).
// Float path: acc[4] accumulates (row g, column 2t), (g, 2t+1),
// (g+8, 2t), (g+8, 2t+1).  Int8 path: block terms go to
// tb[local block * 16 + row] (the epilogue's 16 lanes read a block's rows
// from consecutive words).

struct Lane {
  int g, t;
};

// Q4_K block: 8 sub-blocks of 32, two per 32-byte code group
template <bool ACT8>
__device__ __forceinline__ void body_q4k(const uint8_t *r0, const uint8_t *r1, int bg, int lb, const Lane &L,
                                         const uint32_t (&mk)[8], const uint8_t *xr, int K, float (&acc)[4],
                                         float *tb, int cbc) {
  constexpr int ND = ACT8 ? 1 : 2;
  auto up = [](int v) { return (v + 15) & ~15; };
  uint2 own[ND];
#pragma unroll
  for (int p = 0; p < ND; p++)
    own[p] = *reinterpret_cast<const uint2 *>(xr + p * K + (bg * 8 + L.g) * 32 + 8 * L.t);
  // four independent accumulator chains per digit (the MMA latency is long):
  // set (gq & 1) * 2 + h for code group gq, nibble half h.  Lane column 2t
  // (2t+1) is written only by group gq = t, low (high) half.
  int Ds[ND][4][4];
#pragma unroll
  for (int p = 0; p < ND; p++)
#pragma unroll
    for (int q = 0; q < 4; q++) Ds[p][q][0] = Ds[p][q][1] = Ds[p][q][2] = Ds[p][q][3] = 0;
#pragma unroll
  for (int gq = 0; gq < 4; gq++) {
    const uint2 q0 = *reinterpret_cast<const uint2 *>(r0 + 16 + 32 * gq + 8 * L.t);
    const uint2 q1 = *reinterpret_cast<const uint2 *>(r1 + 16 + 32 * gq + 8 * L.t);
    const uint32_t la0 = q0.x & M4, la1 = q1.x & M4, la2 = q0.y & M4, la3 = q1.y & M4;
    const uint32_t ha0 = (q0.x >> 4) & M4, ha1 = (q1.x >> 4) & M4, ha2 = (q0.y >> 4) & M4, ha3 = (q1.y >> 4) & M4;
#pragma unroll
    for (int p = 0; p < ND; p++) {
      imma_u8(Ds[p][(gq & 1) * 2], la0, la1, la2, la3, own[p].x & mk[2 * gq], own[p].y & mk[2 * gq]);
      imma_u8(Ds[p][(gq & 1) * 2 + 1], ha0, ha1, ha2, ha3, own[p].x & mk[2 * gq + 1], own[p].y & mk[2 * gq + 1]);
    }
  }
  const int odd = L.t & 1;
  int D[ND][4];
#pragma unroll
  for (int p = 0; p < ND; p++) {
    D[p][0] = odd ? Ds[p][2][0] : Ds[p][0][0];
    D[p][1] = odd ? Ds[p][3][1] : Ds[p][1][1];
    D[p][2] = odd ? Ds[p][2][2] : Ds[p][0][2];
    D[p][3] = odd ? Ds[p][3][3] : Ds[p][1][3];
  }
  // scales of sub-blocks j = 2t, 2t+1 for rows g, g+8 (get_scale_min_k4)
  const uint4 h0 = *reinterpret_cast<const uint4 *>(r0);
  const uint4 h1 = *reinterpret_cast<const uint4 *>(r1);
  const int sh = (L.t & 1) * 16;
  uint32_t sc2[2], mm2[2];
  float dd[2], dm[2];
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const uint4 h = r ? h1 : h0;
    const uint32_t A = h.y >> sh, Bq = h.z >> sh, C = h.w >> sh;
    const uint32_t lo_sc = A & 0x3F3Fu, lo_m = Bq & 0x3F3Fu;
    const uint32_t hi_sc = (C & 0x0F0Fu) | ((A >> 2) & 0x3030u);
    const uint32_t hi_m = ((C >> 4) & 0x0F0Fu) | ((Bq >> 2) & 0x3030u);
    sc2[r] = L.t < 2 ? lo_sc : hi_sc;
    mm2[r] = L.t < 2 ? lo_m : hi_m;
    dd[r] = half_exact(h.x & 0xFFFFu);
    dm[r] = half_exact(h.x >> 16);
  }
  if constexpr (!ACT8) {
    const float *sg = reinterpret_cast<const float *>(xr + up(2 * K));
    const float *sx = sg + up(K / 32 * 4) / 4;
    const int G0 = bg * 8 + 2 * L.t;
    const float sg0 = sg[G0], sg1 = sg[G0 + 1], sx0 = sx[G0], sx1 = sx[G0 + 1];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int r = i >> 1, j = i & 1;
      const float v = (float)(D[0][i] * 254 + D[1][i]);  // |.| < 2^24: exact
      const float sc = (float)((sc2[r] >> (8 * j)) & 0xFFu), m = (float)((mm2[r] >> (8 * j)) & 0xFFu);
      acc[i] = fmaf(dd[r] * sc * (j ? sg1 : sg0), v, acc[i]);
      acc[i] = fmaf(-(dm[r] * m), j ? sx1 : sx0, acc[i]);
    }
  } else {
    // TR dotQ4KQ8Go (cpu_quant_q8.go:91-116): isum = sum sc_j * dot_j,
    // msum = sum m_j * (bs pair); t = d*isum - dmin*msum; term = t * d8
    const int16_t *bs = reinterpret_cast<const int16_t *>(xr + up(K) + up(K / 256 * 4)) + bg * 16 + 4 * L.t;
    const float d8 = reinterpret_cast<const float *>(xr + up(K))[bg];
    const int p0 = (int)(int16_t)(bs[0] + bs[1]), p1 = (int)(int16_t)(bs[2] + bs[3]);
#pragma unroll
    for (int r = 0; r < 2; r++) {
      int is = (int)(sc2[r] & 0xFFu) * D[0][2 * r] + (int)((sc2[r] >> 8) & 0xFFu) * D[0][2 * r + 1];
      int ms = (int)(mm2[r] & 0xFFu) * p0 + (int)((mm2[r] >> 8) & 0xFFu) * p1;
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {
        is += __shfl_xor_sync(0xFFFFFFFFu, is, o);
        ms += __shfl_xor_sync(0xFFFFFFFFu, ms, o);
      }
      const float tt = __fsub_rn(__fmul_rn(dd[r], (float)is), __fmul_rn(dm[r], (float)ms));
      if (L.t == 0) tb[lb * 16 + L.g + 8 * r] = __fmul_rn(tt, d8);
    }
  }
}

// Q6_K block: 16 groups of 16 (k16 MMAs), two rounds (halves n = 0, 1);
// round n, column c = 2*cq + i holds group 8n + c
template <bool ACT8>
__device__ __forceinline__ void body_q6k(const uint8_t *r0, const uint8_t *r1, int bg, int lb, const Lane &L,
                                         const uint32_t (&mk)[8], const uint8_t *xr, int K, float (&acc)[4],
                                         float *tb, int cbc) {
  constexpr int ND = ACT8 ? 1 : 2;
  auto up = [](int v) { return (v + 15) & ~15; };
  int is[2] = {0, 0}, ms[2] = {0, 0};
  const float dd[2] = {half_exact(lds16(r0 + 208)), half_exact(lds16(r1 + 208))};
#pragma unroll
  for (int n = 0; n < 2; n++) {
    // own group 8n + g: elements 128n + 32*(g/2) + 16*(g%2) + [0, 16)
    uint32_t own[ND];
#pragma unroll
    for (int p = 0; p < ND; p++)
      own[p] = *reinterpret_cast<const uint32_t *>(xr + p * K + bg * 256 + 128 * n + 32 * (L.g >> 1) +
                                                    16 * (L.g & 1) + 4 * L.t);
    // four accumulator chains per digit: set col & 3 for MMA column col;
    // lane columns 2t, 2t+1 live in sets (2t) & 3, (2t+1) & 3
    int Ds[ND][4][4];
#pragma unroll
    for (int p = 0; p < ND; p++)
#pragma unroll
      for (int q = 0; q < 4; q++) Ds[p][q][0] = Ds[p][q][1] = Ds[p][q][2] = Ds[p][q][3] = 0;
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int off = 64 * n + 16 * i + 4 * L.t, offh = 128 + 32 * n + 16 * i + 4 * L.t;
      const uint32_t qa0 = lds32_a2(r0 + off), qb0 = lds32_a2(r0 + off + 32), qh0 = lds32_a2(r0 + offh);
      const uint32_t qa1 = lds32_a2(r1 + off), qb1 = lds32_a2(r1 + off + 32), qh1 = lds32_a2(r1 + offh);
      uint32_t A0[4], A1[4];
      A0[0] = (qa0 & M4) | ((qh0 << 4) & 0x30303030u);
      A0[1] = (qb0 & M4) | ((qh0 << 2) & 0x30303030u);
      A0[2] = ((qa0 >> 4) & M4) | (qh0 & 0x30303030u);
      A0[3] = ((qb0 >> 4) & M4) | ((qh0 >> 2) & 0x30303030u);
      A1[0] = (qa1 & M4) | ((qh1 << 4) & 0x30303030u);
      A1[1] = (qb1 & M4) | ((qh1 << 2) & 0x30303030u);
      A1[2] = ((qa1 >> 4) & M4) | (qh1 & 0x30303030u);
      A1[3] = ((qb1 >> 4) & M4) | ((qh1 >> 2) & 0x30303030u);
#pragma unroll
      for (int cq = 0; cq < 4; cq++)
#pragma unroll
        for (int p = 0; p < ND; p++) imma_u8_k16(Ds[p][(2 * cq + i) & 3], A0[cq], A1[cq], own[p] & mk[2 * cq + i]);
    }
    const int odd = L.t & 1;
    int D[ND][4];
#pragma unroll
    for (int p = 0; p < ND; p++) {
      D[p][0] = odd ? Ds[p][2][0] : Ds[p][0][0];
      D[p][1] = odd ? Ds[p][3][1] : Ds[p][1][1];
      D[p][2] = odd ? Ds[p][2][2] : Ds[p][0][2];
      D[p][3] = odd ? Ds[p][3][3] : Ds[p][1][3];
    }
    // lane groups: j = 8n + 2t + jj, sc index 8n + 2t + jj
    const uint32_t scw0 = lds16(r0 + 192 + 8 * n + 2 * L.t), scw1 = lds16(r1 + 192 + 8 * n + 2 * L.t);
    if constexpr (!ACT8) {
      const int ng = K / 16;
      const float *sg = reinterpret_cast<const float *>(xr + up(2 * K));
      const float *sd = sg + 2 * (up(ng * 4) / 4);
      const int G0 = bg * 16 + 8 * n + 2 * L.t;
#pragma unroll
      for (int ii = 0; ii < 4; ii++) {
        const int r = ii >> 1, jj = ii & 1;
        const uint32_t scw = r ? scw1 : scw0;
        const float sc = (float)(int8_t)((scw >> (8 * jj)) & 0xFFu);
        const float v = (float)(D[0][ii] * 254 + D[1][ii]);
        acc[ii] = fmaf(dd[r] * sc * sg[G0 + jj], fmaf(-32.0f, sd[G0 + jj], v), acc[ii]);
      }
    } else {
      const int16_t *bs = reinterpret_cast<const int16_t *>(xr + up(K) + up(K / 256 * 4)) + bg * 16 + 8 * n + 2 * L.t;
#pragma unroll
      for (int r = 0; r < 2; r++) {
        const uint32_t scw = r ? scw1 : scw0;
        const int s0 = (int)(int8_t)(scw & 0xFFu), s1 = (int)(int8_t)((scw >> 8) & 0xFFu);
        is[r] += s0 * D[0][2 * r] + s1 * D[0][2 * r + 1];
        ms[r] += s0 * (int)bs[0] + s1 * (int)bs[1];
      }
    }
  }
  if constexpr (ACT8) {
    // TR dotQ6KQ8Go (cpu_quant_q8.go:378-407): t = d*(isum - 32*msum); term = t*d8
    const float d8 = reinterpret_cast<const float *>(xr + up(K))[bg];
#pragma unroll
    for (int r = 0; r < 2; r++) {
#pragma unroll
      for (int o = 1; o < 4; o <<= 1) {
        is[r] += __shfl_xor_sync(0xFFFFFFFFu, is[r], o);
        ms[r] += __shfl_xor_sync(0xFFFFFFFFu, ms[r], o);
      }
      const float tt = __fmul_rn(dd[r], (float)(is[r] - 32 * ms[r]));
      if (L.t == 0) tb[lb * 16 + L.g + 8 * r] = __fmul_rn(tt, d8);
    }
  }
}

// Q8_0 / Q4_0 round: 8 consecutive blocks, block j of the round in MMA
// column j.  Rounds start 16-byte aligned (8 blocks = 272 / 144 bytes).
template <int W, bool ACT8>
__device__ __forceinline__ void body_q32(const uint8_t *s0, const uint8_t *s1, int bg0, int lb0, const Lane &L,
                                         const uint32_t (&mk)[8], const uint8_t *xr, int K, float (&acc)[4],
                                         float *tb, int cbc) {
  using P = Pol<W>;
  constexpr int ND = ACT8 ? 1 : 2;
  constexpr int B = P::B;
  auto up = [](int v) { return (v + 15) & ~15; };
  // own block bg0 + g: Q8_0 k-slots 4t.. <- codes 8t.., 4t+16.. <- 8t+4..;
  // Q4_0 k-slots 4t.. <- low nibbles 4t.., 4t+16.. <- high nibbles (16+4t..)
  uint2 own[ND];
#pragma unroll
  for (int p = 0; p < ND; p++) {
    const uint8_t *pl = xr + p * K + (bg0 + L.g) * 32;
    if constexpr (W == TCB_Q8_0 || !ACT8) own[p] = *reinterpret_cast<const uint2 *>(pl + 8 * L.t);  // float Q4_0: paired words
    else own[p] = make_uint2(*reinterpret_cast<const uint32_t *>(pl + 4 * L.t), *reinterpret_cast<const uint32_t *>(pl + 16 + 4 * L.t));
  }
  // four accumulator chains per digit: set j & 3 for block j of the round
  int Ds[ND][4][4];
#pragma unroll
  for (int p = 0; p < ND; p++)
#pragma unroll
    for (int q = 0; q < 4; q++) Ds[p][q][0] = Ds[p][q][1] = Ds[p][q][2] = Ds[p][q][3] = 0;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const uint8_t *b0 = s0 + j * B, *b1 = s1 + j * B;
    if constexpr (W == TCB_Q8_0) {
      const uint32_t w00 = lds32_a2(b0 + 2 + 8 * L.t), w01 = lds32_a2(b0 + 6 + 8 * L.t);
      const uint32_t w10 = lds32_a2(b1 + 2 + 8 * L.t), w11 = lds32_a2(b1 + 6 + 8 * L.t);
#pragma unroll
      for (int p = 0; p < ND; p++) imma_s8(Ds[p][j & 3], w00, w10, w01, w11, own[p].x & mk[j], own[p].y & mk[j]);
    } else {
      const uint32_t q0 = lds32_a2(b0 + 2 + 4 * L.t), q1 = lds32_a2(b1 + 2 + 4 * L.t);
      const uint32_t a0 = q0 & M4, a1 = q1 & M4, a2 = (q0 >> 4) & M4, a3 = (q1 >> 4) & M4;
#pragma unroll
      for (int p = 0; p < ND; p++) imma_u8(Ds[p][j & 3], a0, a1, a2, a3, own[p].x & mk[j], own[p].y & mk[j]);
    }
  }
  const int odd = L.t & 1;
  int D[ND][4];
#pragma unroll
  for (int p = 0; p < ND; p++) {
    D[p][0] = odd ? Ds[p][2][0] : Ds[p][0][0];
    D[p][1] = odd ? Ds[p][3][1] : Ds[p][1][1];
    D[p][2] = odd ? Ds[p][2][2] : Ds[p][0][2];
    D[p][3] = odd ? Ds[p][3][3] : Ds[p][1][3];
  }
  // lane blocks: 2t, 2t+1 of the round, rows g, g+8
  float dw[4];
#pragma unroll
  for (int i = 0; i < 4; i++) dw[i] = half_exact(lds16((i >> 1 ? s1 : s0) + (2 * L.t + (i & 1)) * B));
  const int G0 = bg0 + 2 * L.t;
  if constexpr (!ACT8) {
    const float *sg = reinterpret_cast<const float *>(xr + up(2 * K));
    const float *sd = sg + 2 * (up(K / 32 * 4) / 4);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int j = i & 1;
      float v = (float)(D[0][i] * 254 + D[1][i]);
      if (W == TCB_Q4_0) v = fmaf(-8.0f, sd[G0 + j], v);
      acc[i] = fmaf(dw[i] * sg[G0 + j], v, acc[i]);
    }
  } else {
    // TR dotQ4Q8Go (cpu_quant_q8.go:74-87), the same fold for Q8_0:
    // t = dw*d8; term = t*isum
    const float *d8 = reinterpret_cast<const float *>(xr + up(K));
    const int16_t *bs = reinterpret_cast<const int16_t *>(xr + up(K) + up(K / 32 * 4));
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int j = i & 1;
      int isum = D[0][i];
      if (W == TCB_Q4_0) isum -= 8 * ((int)bs[2 * (G0 + j)] + (int)bs[2 * (G0 + j) + 1]);
      tb[(lb0 + 2 * L.t + j) * 16 + L.g + 8 * (i >> 1)] = __fmul_rn(__fmul_rn(dw[i], d8[G0 + j]), (float)isum);
    }
  }
}

// ----------------------------------------------------------------- kernel
// Warps: 0..15 compute, 16 produces (TMA), 17 finishes outputs.  The
// compute warps run through the stages on their own (no CTA-wide barrier
// per stage); tile partials (float path) and block terms (int8 path) reach
// the epilogue warp through shared memory guarded by mbarriers.
// Shared memory: [barriers (1 KB) | flag | tile partials | x region |
// int8 terms | stages].  CTA b owns tiles b, b + grid, ...

constexpr int kEpi = kConsumers + 1;      // epilogue warp
constexpr int kWarpsAll = kConsumers + 2;
constexpr int kPartSlots = 8;             // tile partial slots in flight
constexpr int kBarBytes = 1024;

// MR: the most rows of x a launch takes.  Each row has its own x region and
// tile partials (float path) or block terms (int8 path, [S][MR][cbc][16],
// each row's folded in block order); every staged block is multiplied
// against all the rows before the stage is released.
template <int W, bool ACT8, int MR>
__global__ void __launch_bounds__(32 * kWarpsAll, 1) k_mv1(const __grid_constant__ CUtensorMap tmap, const Params a) {
  using P = Pol<W>;
  const int M = MR == 1 ? 1 : a.M;  // rows of x (a compile-time 1 for the batch-1 kernel)
  constexpr int pitch = P::BOX8 * 8, box_bytes = 16 * pitch, NBOX = P::NBOX;
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t *full = reinterpret_cast<uint64_t *>(sm);  // [S]     copy engine -> compute
  uint64_t *empty = full + 8;                         // [S]     compute -> producer
  uint64_t *sdone = full + 16;                        // [S]     int8 terms of a stage ready
  uint64_t *sfree = full + 24;                        // [S]     int8 terms folded
  uint64_t *tdone = full + 32;                        // [slots] tile partials ready
  uint64_t *tfree = full + 40;                        // [slots] tile partials summed
  int *flag = reinterpret_cast<int *>(sm + 512);   // the whole launch takes TR's float path
  int *rflag = flag + 1;                           // [MR] int8 path, MR > 1: row m is not finite
  float *part = reinterpret_cast<float *>(sm + kBarBytes);  // [slots][MR][kConsumers][16]
  uint8_t *xr = sm + a.xoff;                                // [MR] x regions, a.xstride apart
  float *terms = reinterpret_cast<float *>(sm + a.toff);  // [S][MR][cbc][16]
  uint8_t *stages = sm + a.soff;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int stage_bytes = NBOX * box_bytes;
  const int my_tiles = (a.tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int nstages = my_tiles * a.nch;

  if (threadIdx.x == 0) {
    *flag = 0;
    for (int m = 0; m < MR; m++) rflag[m] = 0;
    for (int s = 0; s < a.S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
      mbar_init(&sdone[s], kConsumers);
      mbar_init(&sfree[s], 1);
    }
    for (int s = 0; s < kPartSlots; s++) {
      mbar_init(&tdone[s], kConsumers);
      mbar_init(&tfree[s], 1);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == kConsumers) {
    // producer: a stage is NBOX boxes of 16 rows; rows past N and bytes
    // past the row end are zero-filled by the copy engine
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
      for (int it = 0; it < nstages; it++) {
        const int buf = it % a.S;
        if (!spin_bar(&empty[buf], (uint32_t)(((it / a.S) & 1) ^ 1), a.err)) return;
        const int tile = (int)blockIdx.x + (it / a.nch) * (int)gridDim.x, ch = it % a.nch;
        const int b0 = ch * a.cbc;
        const int nbox = min(NBOX, (a.nb - b0 + P::BPB - 1) / P::BPB);
        mbar_expect_tx(&full[buf], (uint32_t)(nbox * box_bytes));
        for (int k = 0; k < nbox; k++)
          tma_load_2d(stages + buf * stage_bytes + k * box_bytes, &tmap, (b0 + k * P::BPB) * P::B / 8, tile * 16,
                      &full[buf]);
        if (it == (nstages < a.S ? nstages : a.S) - 1) prefetch_slice_l2(a.pf, a.pf_bytes);
      }
    }
    return;
  }

  // compute and epilogue warps: x (and c) may be written by the previous
  // kernel of the stream
  pdl_wait();
  if (warp < kConsumers) {
    const size_t xel = a.xdt == TCB_F32 ? 4 : 2;
    for (int m = 0; m < M; m++) {
      Params ar = a;
      ar.x = static_cast<const char *>(a.x) + (size_t)m * a.ldx * xel;
      // int8 path with several rows: a row that is not finite takes TR's
      // float path alone (in the epilogue); the others stay integer-exact
      if constexpr (ACT8) prep_act8<W>(ar, xr + (size_t)m * a.xstride, MR == 1 ? flag : rflag + m);
      else prep_float<W>(ar, xr + (size_t)m * a.xstride, flag);
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(32 * (kConsumers + 1)) : "memory");
  const bool slow = *flag != 0;

  if (!slow && warp == kEpi) {
    // epilogue: sum the sixteen warp partials of each tile in warp order
    // (float path) or fold every block term in block order (int8 path)
    int it = 0;
    for (int ti = 0; ti < my_tiles; ti++) {
      const int tile = (int)blockIdx.x + ti * (int)gridDim.x;
      const int row = tile * 16 + lane;
      const bool mine = lane < 16 && row < a.N;
      if constexpr (!ACT8) {
        float cold[MR], vs[MR];
#pragma unroll
        for (int m = 0; m < MR; m++)
          cold[m] = (a.accumulate && mine && m < M) ? load_out(a.c, (long)m * a.ldc + row, a.cdt) : 0.f;
        const int slot = ti % kPartSlots;
        if (!spin_bar(&tdone[slot], (uint32_t)((ti / kPartSlots) & 1), a.err)) return;
#pragma unroll
        for (int m = 0; m < MR; m++) {
          vs[m] = 0.f;
          if (m >= M) continue;
          const float *pt = part + (slot * MR + m) * kConsumers * 16;
          if (lane < 16)
#pragma unroll
            for (int w2 = 0; w2 < kConsumers; w2++) vs[m] += pt[w2 * 16 + lane];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&tfree[slot]);
        it += a.nch;
        if (mine) {
#pragma unroll
          for (int m = 0; m < MR; m++)
            if (m < M) store_out_old(a.c, (long)m * a.ldc + row, a.cdt, vs[m], a.accumulate != 0, cold[m]);
        }
      } else {
      float cold[MR], v[MR];
#pragma unroll
      for (int m = 0; m < MR; m++) {
        cold[m] = (a.accumulate && mine && m < M) ? load_out(a.c, (long)m * a.ldc + row, a.cdt) : 0.f;
        v[m] = 0.f;
      }
      for (int ch = 0; ch < a.nch; ch++, it++) {
        const int buf = it % a.S;
        if (!spin_bar(&sdone[buf], (uint32_t)((it / a.S) & 1), a.err)) return;
        const int nblk = min(a.nb, (ch + 1) * a.cbc) - ch * a.cbc;
#pragma unroll
        for (int m = 0; m < MR; m++) {
          if (m >= M) break;
          const float *tb = terms + (buf * MR + m) * 16 * a.cbc;
          if (lane < 16)
            for (int lb = 0; lb < nblk; lb++) v[m] = __fadd_rn(v[m], tb[lb * 16 + lane]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfree[buf]);
      }
      if constexpr (MR > 1) {
        // rows of x that are not finite: TR's float path, one output row at
        // a time over the warp (their int8 terms are discarded)
        const size_t xel = a.xdt == TCB_F32 ? 4 : 2;
        for (int m = 0; m < M; m++) {
          if (!rflag[m]) continue;
          const void *xrow = static_cast<const char *>(a.x) + (size_t)m * a.ldx * xel;
          for (int r = 0; r < 16; r++) {
            const int n = tile * 16 + r;
            if (n >= a.N) break;
            float accs[1] = {0.0f};
            lane_row_float<W, 1>(a.w + (long)n * a.rowBytes, a.K, lane, XGlobal{xrow, 0, a.xdt}, accs);
            const float f = warp_sum(accs[0]);
#pragma unroll
            for (int mm = 0; mm < MR; mm++)
              if (mm == m && lane == r) v[mm] = f;
          }
        }
      }
      if (mine) {
#pragma unroll
        for (int m = 0; m < MR; m++)
          if (m < M) store_out_old(a.c, (long)m * a.ldc + row, a.cdt, v[m], a.accumulate != 0, cold[m]);
      }
      }
    }
    return;
  }

  if (warp < kConsumers) {
    const Lane L{lane >> 2, lane & 3};
    uint32_t mk[8];
#pragma unroll
    for (int c = 0; c < 8; c++) mk[c] = L.g == c ? 0xFFFFFFFFu : 0u;
    int it = 0;
    for (int ti = 0; ti < my_tiles; ti++) {
      float acc[MR][4] = {};
      for (int ch = 0; ch < a.nch; ch++, it++) {
        const int buf = it % a.S;
        const uint32_t ph = (uint32_t)((it / a.S) & 1);
        bool ok = true;
        if (lane == 0) ok = wait_bar(&full[buf], ph, a.err);
        if (ACT8 && !slow && lane == 0 && ok) ok = spin_bar(&sfree[buf], ph ^ 1, a.err);
        if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return;
        if (!slow) {
          const uint8_t *st = stages + buf * stage_bytes;
          const int b0 = ch * a.cbc, nblk = min(a.nb, b0 + a.cbc) - b0;
          for (int lb = warp * P::RB; lb < nblk; lb += kConsumers * P::RB) {
            const uint8_t *r0 = st + (lb / P::BPB) * box_bytes + L.g * pitch + (lb % P::BPB) * P::B;
            const uint8_t *r1 = r0 + 8 * pitch;
#pragma unroll
            for (int m = 0; m < MR; m++) {
              if (m >= M) break;  // uniform
              const uint8_t *xm = xr + (size_t)m * a.xstride;
              float *tb = terms + (buf * MR + m) * 16 * a.cbc;
              if constexpr (W == TCB_Q4_K) body_q4k<ACT8>(r0, r1, b0 + lb, lb, L, mk, xm, a.K, acc[m], tb, a.cbc);
              else if constexpr (W == TCB_Q6_K) body_q6k<ACT8>(r0, r1, b0 + lb, lb, L, mk, xm, a.K, acc[m], tb, a.cbc);
              else body_q32<W, ACT8>(r0, r1, b0 + lb, lb, L, mk, xm, a.K, acc[m], tb, a.cbc);
            }
          }
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&empty[buf]);
          if (ACT8 && !slow) mbar_arrive(&sdone[buf]);
        }
      }
      if (!ACT8 && !slow) {
        const int slot = ti % kPartSlots;
        bool ok = true;
        if (lane == 0) ok = spin_bar(&tfree[slot], (uint32_t)(((ti / kPartSlots) & 1) ^ 1), a.err);
        if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return;
#pragma unroll
        for (int m = 0; m < MR; m++) {
          if (m >= M) break;
          float s0 = acc[m][0] + acc[m][1], s1 = acc[m][2] + acc[m][3];
          s0 += __shfl_xor_sync(0xFFFFFFFFu, s0, 1);
          s1 += __shfl_xor_sync(0xFFFFFFFFu, s1, 1);
          s0 += __shfl_xor_sync(0xFFFFFFFFu, s0, 2);
          s1 += __shfl_xor_sync(0xFFFFFFFFu, s1, 2);
          float *pt = part + (slot * MR + m) * kConsumers * 16;
          if (L.t == 0) {
            pt[warp * 16 + L.g] = s0;
            pt[warp * 16 + L.g + 8] = s1;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&tdone[slot]);
      }
    }
  }
  if (slow) {
    // NaN/Inf in x: TR's float path (the int8 path also falls back to it,
    // cpu_quant_q8.go:157-163), one warp per row
    const int widx = warp == kEpi ? kConsumers : warp;  // 0..16 over the compute and epilogue warps
    const size_t xel = a.xdt == TCB_F32 ? 4 : 2;
    for (int n = (int)blockIdx.x * (kConsumers + 1) + widx; n < a.N; n += (int)gridDim.x * (kConsumers + 1))
      for (int m = 0; m < M; m++) {
        float accs[1] = {0.0f};
        const void *xrow = static_cast<const char *>(a.x) + (size_t)m * a.ldx * xel;
        lane_row_float<W, 1>(a.w + (long)n * a.rowBytes, a.K, lane, XGlobal{xrow, 0, a.xdt}, accs);
        const float v = warp_sum(accs[0]);
        if (lane == 0) store_out(a.c, (long)m * a.ldc + n, a.cdt, v, a.accumulate != 0);
      }
  }
}

}  // namespace mv

// ----------------------------------------------------------------- host

namespace {

constexpr int kSmemMax = 227 * 1024;

// [N rows, rowBytes/8 eight-byte elements] view of the block store, rows
// ldw bytes apart (a padded row's last element may hold up to 7 pad bytes,
// which no block reads)
template <int W, bool ACT8>
bool encode_weight_map(CUtensorMap *tm, const void *w, int N, long rowBytes, long ldw) {
  auto enc = tensor_map_encoder();
  if (!enc) return false;
  cuuint64_t gdim[2] = {(cuuint64_t)((rowBytes + 7) / 8), (cuuint64_t)N};
  cuuint64_t gstride[1] = {(cuuint64_t)ldw};
  cuuint32_t box[2] = {(cuuint32_t)mv::Pol<W>::BOX8, 16};
  cuuint32_t estr[2] = {1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), gdim, gstride, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int W, bool ACT8>
cudaError_t plan_launch(const MvPlan &pl, const void *w, int N, int K, const void *x, int xdt, void *c, int cdt,
                        int accumulate, int *err, cudaStream_t s, const void *pf, size_t pf_bytes, int M, long ldx,
                        long ldc) {
  if (M < 1 || M > pl.rows) return cudaErrorInvalidValue;
  mv::Params a{};
  a.w = static_cast<const uint8_t *>(w);
  a.nb = K / mv::Pol<W>::E;
  a.rowBytes = pl.ldw;
  a.N = N;
  a.K = K;
  a.x = x;
  a.xdt = xdt;
  a.c = c;
  a.cdt = cdt;
  a.accumulate = accumulate;
  a.tiles = pl.tiles;
  a.cbc = pl.cbc;
  a.nch = pl.nch;
  a.err = err;
  a.S = pl.stages;
  a.xoff = pl.xoff;
  a.toff = pl.toff;
  a.soff = pl.soff;
  a.pf = pf;
  a.pf_bytes = pf_bytes;
  a.M = M;
  a.ldx = ldx;
  a.ldc = ldc;
  a.xstride = pl.xstride;
  CUtensorMap tm;
  static_assert(sizeof(tm) == sizeof(pl.tmap), "CUtensorMap size");
  memcpy(&tm, pl.tmap, sizeof tm);
  void (*kern)(const CUtensorMap, const mv::Params) = mv::k_mv1<W, ACT8, 1>;
  if constexpr (ACT8 || W != TCB_Q4_K) {  // Q4_K float rows take k_mvq4k
    if (pl.rows == 8) kern = mv::k_mv1<W, ACT8, 8>;
    else if (pl.rows == 4) kern = mv::k_mv1<W, ACT8, 4>;
    else if (pl.rows == 2) kern = mv::k_mv1<W, ACT8, 2>;
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(32 * mv::kWarpsAll);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tm, a);
}

// mr (1, 2, 4, 8; 1 on the int8 path): the most rows of x a launch takes
template <int W, bool ACT8>
MvPlan plan_w(int N, int K, const void *w, int sms, int mr = 1, long ldw = 0) {
  using P = mv::Pol<W>;
  MvPlan pl{};
  if (mr != 1 && mr != 2 && mr != 4 && mr != 8) return pl;
  const int nb = K / P::E;
  const long rowBytes = (long)nb * P::B;
  if (ldw == 0) ldw = rowBytes;
  if (ldw % 16 || ldw < rowBytes || reinterpret_cast<uintptr_t>(w) % 16 || nb == 0) return pl;
  if (P::RB == 8 && nb % 8) return pl;  // Q8_0 / Q4_0 rounds are 8 blocks
  if (!tensor_map_encoder()) return pl;
  pl.cbc = P::NBOX * P::BPB;
  pl.nch = (nb + pl.cbc - 1) / pl.cbc;
  pl.ksplit = 1;
  pl.cpk = pl.nch;
  pl.pitch = mv::Pol<W>::BOX8 * 8;
  pl.xstride = (mv::x_region_bytes<W, ACT8>(K) + 127) & ~127;
  pl.xoff = mv::kBarBytes + mr * mv::kPartSlots * mv::kConsumers * 16 * 4;
  pl.toff = pl.xoff + mr * pl.xstride;
  const int tbytes_per_stage = ACT8 ? mr * 16 * pl.cbc * 4 : 0;
  const int stage_bytes = P::NBOX * 16 * pl.pitch;
  int S = (kSmemMax - pl.toff - 128) / (stage_bytes + tbytes_per_stage);
  if (S > 6) S = 6;
  pl.soff = (pl.toff + S * tbytes_per_stage + 127) & ~127;
  if (S < 2) return pl;
  pl.stages = S;
  pl.smem = pl.soff + S * stage_bytes;
  pl.tiles = (N + 15) / 16;
  pl.grid = pl.tiles < sms ? pl.tiles : sms;
  pl.rows = mr;
  pl.ldw = ldw;
  CUtensorMap tm;
  if (!encode_weight_map<W, ACT8>(&tm, w, N, rowBytes, ldw)) return pl;
  memcpy(pl.tmap, &tm, sizeof tm);
  pl.ok = true;
  return pl;
}

}  // namespace

MvPlan matvec_plan(int wtype, int act8, int M, int N, int K, const void *w, int sms, long ldw) {
  MvPlan none{};
  if (M != 1 || N <= 0 || K <= 0) return none;
  if (ldw) return wtype == TCB_Q6_K && !act8 ? plan_w<TCB_Q6_K, false>(N, K, w, sms, 1, ldw) : none;
  switch (wtype) {
  case TCB_Q4_K: return act8 ? plan_w<TCB_Q4_K, true>(N, K, w, sms) : q4k_plan(N, K, w, sms);
  case TCB_Q6_K:
    // the k-slot Q6_K kernel wins on wide products (the output head); inside
    // a decode chain of 4096-row products the generic kernel overlaps its
    // neighbours better (measured 436 vs 424 tok/s on the 8B step)
    if (act8) return plan_w<TCB_Q6_K, true>(N, K, w, sms);
    return N >= kQ6kMinRows ? q6k_plan(N, K, w, sms) : plan_w<TCB_Q6_K, false>(N, K, w, sms);
  case TCB_Q8_0: return act8 ? plan_w<TCB_Q8_0, true>(N, K, w, sms) : plan_w<TCB_Q8_0, false>(N, K, w, sms);
  case TCB_Q4_0: return act8 ? plan_w<TCB_Q4_0, true>(N, K, w, sms) : plan_w<TCB_Q4_0, false>(N, K, w, sms);
  }
  return none;
}

MvPlan matvec_plan_rows(int wtype, int act8, int N, int K, const void *w, int sms, int mr, long ldw) {
  MvPlan none{};
  if (N <= 0 || K <= 0) return none;
  if (ldw) return wtype == TCB_Q6_K && !act8 && K <= 8192 ? plan_w<TCB_Q6_K, false>(N, K, w, sms, mr, ldw) : none;
  if (act8) {
    switch (wtype) {
    case TCB_Q4_K: return plan_w<TCB_Q4_K, true>(N, K, w, sms, mr);
    case TCB_Q6_K: return plan_w<TCB_Q6_K, true>(N, K, w, sms, mr);
    case TCB_Q8_0: return plan_w<TCB_Q8_0, true>(N, K, w, sms, mr);
    case TCB_Q4_0: return plan_w<TCB_Q4_0, true>(N, K, w, sms, mr);
    }
    return none;
  }
  switch (wtype) {
  case TCB_Q4_K: return q4k_plan(N, K, w, sms, mr);
  // Q6_K rows of more than 8192 elements: one row per launch measured faster
  // (4096x14336: 37 vs 42 us at M = 2, the digit regions crowd out stages)
  case TCB_Q6_K: return N >= kQ6kMinRows || K > 8192 ? none : plan_w<TCB_Q6_K, false>(N, K, w, sms, mr);
  case TCB_Q8_0: return plan_w<TCB_Q8_0, false>(N, K, w, sms, mr);
  case TCB_Q4_0: return plan_w<TCB_Q4_0, false>(N, K, w, sms, mr);
  }
  return none;
}

cudaError_t matvec_launch(const MvPlan &pl, int wtype, int act8, int N, int K, const void *w, const void *x, int xdt,
                          void *c, int cdt, int accumulate, int *err, cudaStream_t s, const void *pf, size_t pf_bytes,
                          void *scratch, int M, long ldx, long ldc) {
#define TCB_MV(WT)                                                                                                \
  return act8 ? plan_launch<WT, true>(pl, w, N, K, x, xdt, c, cdt, accumulate, err, s, pf, pf_bytes, M, ldx, ldc) \
              : plan_launch<WT, false>(pl, w, N, K, x, xdt, c, cdt, accumulate, err, s, pf, pf_bytes, M, ldx, ldc)
  if (pl.kind == 1)
    return q4k_launch(pl, N, K, w, x, xdt, c, cdt, accumulate, err, scratch, s, nullptr, 0.f, pf, pf_bytes, M, ldx,
                      ldc);
  if (pl.kind == 3) return rows_launch(pl, N, K, w, x, xdt, ldx, c, cdt, ldc, accumulate, M, err, scratch, s);
  if (pl.kind == 2) {
    if (M != 1) return cudaErrorInvalidValue;
    return q6k_launch(pl, N, K, w, x, xdt, c, cdt, accumulate, err, s, pf, pf_bytes, scratch);
  }
  switch (wtype) {
  case TCB_Q4_K: TCB_MV(TCB_Q4_K);
  case TCB_Q6_K: TCB_MV(TCB_Q6_K);
  case TCB_Q8_0: TCB_MV(TCB_Q8_0);
  case TCB_Q4_0: TCB_MV(TCB_Q4_0);
  }
#undef TCB_MV
  return cudaErrorInvalidValue;
}

}  // namespace tcb
