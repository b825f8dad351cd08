// tcb_mv_rows.cu - Q4_K, Q6_K and Q4_0 float-path product of 2 to 16
// activation rows, the weights streamed once for all of them:
//
//   y[m][n] (+)= sum_k x[m][k] * dequant(W)[n, k]     W: [N, K] blocks
//
// This is TR's quantGemm with a few rows (tensor/cpu_quant.go:47-160, the
// float path: a batch of decode steps, or the rows of a small prefill).  At
// a handful of rows the product is still a weight stream; what limits it
// is the per-element work, so the design keeps that work per (weight row,
// sub-block, activation row) to one integer multiply-add:
//
//  * The activations are digitised once per call (k_xdig), not per CTA:
//    per row and 256-element superblock, x ~= sigma * (h + l/254) with
//    sigma = max|x| / 127 and int8 digits h, l (representation error at
//    most max|x| / 64516 per element).  The digits are written straight in
//    the B-operand layout of the MMAs below, four rows (eight digit columns)
//    per 256-byte panel of 32 elements, plus a ninth panel holding each
//    sub-block's digit sums (split into a high and a low byte).
//  * Dot products: int8 mma.sync with A = 16 weight rows x one sub-block of
//    codes (u8) and B = the sub-block's digits of four activation rows
//    (column 2r + digit): one MMA gives every (weight row, activation row,
//    digit) sum of the sub-block.  Q4_K: m16n8k32, lane t's k-slots are 8
//    consecutive elements (one 8-byte load per row pair); high-nibble codes
//    are read in place as 16*q, low-nibble sub-blocks take their scale times
//    16.  Q6_K: m16n8k16 per 16-element sub-block.
//  * The sub-block scale is applied in integers, sc_j * D_j added into a
//    per-superblock s32 accumulator (Q4_K: at most 8 * 63 * 16 * 32 * 15 *
//    127 < 2^31; Q6_K: 16 * 128 * 16 * 63 * 127 < 2^31).  The second term
//    of the block (Q4_K: dmin * sum_j m_j sum_i x_i; Q6_K: the -32 code
//    offset, 32 * sum_j sc_j sum_i x_i) is one k16 MMA per digit-sum byte
//    over the superblock's sub-blocks (A = m_j or sc_j, B = the digit sums).
//    Once per superblock the accumulators become f32:
//      Q4_K: acc += sigma * (d/16 * (H + L/254) - dmin/254 * (254*MH + ML))
//      Q6_K: acc += sigma * d * ((H - 32 OH) + (L - 32 OL) / 254).
//  * Staging: one CTA per SM; a stage is one TMA box of 32 weight rows x 8
//    superblocks.  16 compute warps: warp w owns the 16-row half w / 8 of
//    superblock w % 8 of every stage; it copies its operands to registers
//    and releases the stage before the math.  Thread 0 issues the first
//    stages before the dependency wait; after that the last warp to release
//    a buffer (a shared counter per buffer) issues its next stage at once,
//    so no warp waits on a producer.  The activation digits of the CTA's K
//    range stay resident in shared memory.
//  * Split K: when the digits of the whole row do not fit beside the stages
//    (or more CTAs balance the tiles better), the CTAs are split into ksplit
//    groups, each owning one K range for its lifetime; their partials go to
//    scratch and k_rows_red adds them in range order.
//  * Tile partials: each warp's sums go to shared memory; the warp that
//    finishes a tile last adds the partials of each row in superblock order
//    and stores them, so no warp waits for the others.  Results do not
//    depend on timing.
//  * A NaN or Inf anywhere in x sends the whole call down TR's fp32 path
//    (one warp per output, the CTAs of the first K range), so NaN and Inf
//    propagate as in TR.
#include <string.h>

#include "tcb_common.cuh"
#include "tcb_matvec.h"
#include "tcb_mv_ptx.cuh"
#include "tcb_simt.cuh"

namespace tcb {
namespace mvr {

using namespace mv;

constexpr int kC = 16;                     // compute warps (thread 0 also issues the copies)
constexpr int kWarps = kC;
constexpr int kRows = 32;                  // weight rows per tile
constexpr int kBlk = 8;                    // superblocks per stage
constexpr int kPanel = 256;                // digits of 32 elements of 4 rows: 8 columns x 32
constexpr int kGroupBytes = 9 * kPanel;    // one superblock of one 4-row group: 8 panels + digit sums
constexpr int kMaxS = 6;
constexpr int kBarOff = 0, kCntOff = 128, kPartOff = 256;
constexpr int kSmemMax = 227 * 1024;

// weight formats: superblock bytes, stage box width (8-byte elements) and
// staged row pitch
template <int W>
struct Fmt;
template <>
struct Fmt<TCB_Q4_K> {
  static constexpr int kBB = 144;
  static constexpr int kBox8 = 148;     // 8 superblocks + 32 bytes
  static constexpr int kPitch = 1184;   // 32 mod 128: a warp's 8-byte code loads are conflict-free
};
template <>
struct Fmt<TCB_Q4_0> {
  static constexpr int kBB = 144;       // eight 18-byte blocks: 256 elements
  static constexpr int kBox8 = 148;
  static constexpr int kPitch = 1184;
};
template <>
struct Fmt<TCB_Q6_K> {
  static constexpr int kBB = 210;
  static constexpr int kBox8 = 210;     // 8 superblocks
  static constexpr int kPitch = 1680;   // 16 mod 128: a warp's 4-byte code loads are conflict-free
};

// 4 bytes at a 2-byte aligned shared address (Q6_K superblocks sit 210
// bytes apart; the branch is uniform over a warp)
__device__ __forceinline__ uint32_t ld4(const uint8_t *p) {
  const uintptr_t v = reinterpret_cast<uintptr_t>(p);
  if ((v & 2) == 0) return *reinterpret_cast<const uint32_t *>(p);
  const uint32_t *q = reinterpret_cast<const uint32_t *>(p - 2);
  return __byte_perm(q[0], q[1], 0x5432);
}

// D += A(16x16 s8) * B(16x8 s8)
__device__ __forceinline__ void imma_s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// global scratch (after the shared counter region):
//   digits [nb][J][9 panels][8 columns][32]     nb * J * 2304 bytes
//   sigma  [nb][4 (row in group)][J] f32        nb * 16 * J bytes
//   bad    [nb][16] u8 (row has a NaN/Inf in the superblock)
//   part   [ksplit][4J][N] f32 (ksplit > 1)
struct Layout {
  size_t dig, sig, bad, part, end;
};
__host__ __device__ inline size_t al256(size_t v) { return (v + 255) & ~(size_t)255; }
__host__ __device__ inline Layout layout(int nb, int J, int ksplit, int N) {
  Layout L;
  L.dig = kScratchCntBytes;
  L.sig = al256(L.dig + (size_t)nb * J * kGroupBytes);
  L.bad = al256(L.sig + (size_t)nb * 16 * J);
  L.part = al256(L.bad + (size_t)nb * 16);
  L.end = ksplit > 1 ? al256(L.part + (size_t)ksplit * 4 * J * N * 4) : L.part;
  return L;
}

struct Params {
  const uint8_t *w;
  int N, K, nb, M;
  const void *x;
  int xdt;
  long ldx;
  void *c;
  int cdt;
  long ldc;
  int accumulate;
  int tiles, ksplit, nbr, nch, S, slots;
  int soff, xoff;  // shared memory: stages, digits (+ sigma after them)
  const uint8_t *dig;
  const float *sig;
  const uint8_t *bad;
  float *part;
  int *err;
};

// ---------------------------------------------------------------- digits

// One warp per (superblock, row); rows M..4J-1 get zero digits.  Q6_K and
// Q4_0 take the k-slot order that puts a lane's two 4-byte code groups side
// by side within a 32-element panel column (bytes 8t..8t+3 = elements
// 4t..4t+3, bytes 8t+4..8t+7 = elements 16+4t..16+4t+3); Q4_K element order.
// The ninth panel: Q4_K / Q6_K the sub-block digit sums (32 / 16 elements)
// for the second-term MMA, [high byte, low byte][column][16 k-slots], S = 64
// * high + low with low in 0..63; Q4_0 the combined sums 254 * Sh + Sl of
// each 32-element block, int32 [block][row in group].
template <int J, int W>
__global__ void __launch_bounds__(256) k_xdig(const void *x, int xdt, long ldx, int M, int nb, uint8_t *dig, float *sig,
                                             uint8_t *bad) {
  pdl_launch_dependents();
  pdl_wait();  // x may be written by the previous kernel of the stream
  const int lane = threadIdx.x & 31;
  const int wid = (int)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (wid >= nb * 4 * J) return;
  const int b = wid / (4 * J), m = wid % (4 * J);
  const int j = m >> 2, r = m & 3;
  float v[8];
  bool fin = true;
  float amax = 0.f;
  if (m < M) {
    const char *row = static_cast<const char *>(x) + (size_t)m * ldx * (xdt == TCB_F32 ? 4 : 2);
    const long k0 = (long)b * 256 + lane * 8;
#pragma unroll
    for (int i = 0; i < 8; i++) {
      v[i] = load_act(row, k0 + i, xdt);
      fin = fin && isfinite(v[i]);
      amax = fmaxf(amax, fabsf(v[i]));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = 0.f;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
  fin = __all_sync(0xFFFFFFFFu, fin);
  if (!fin) amax = 0.f;
  const float inv = amax > 0.f ? __fdiv_rn(127.f, amax) : 0.f;
  uint32_t h[2] = {0u, 0u}, l[2] = {0u, 0u};
  int sh = 0, sl = 0;  // digit sums of this lane's 8 elements
#pragma unroll
  for (int i = 0; i < 8; i++) {
    const float q = v[i] * inv;
    float hf = fminf(fmaxf(rintf(q), -127.f), 127.f);
    float lf = fminf(fmaxf(rintf((q - hf) * 254.f), -127.f), 127.f);
    sh += (int)hf;
    sl += (int)lf;
    h[i >> 2] |= ((uint32_t)(int)hf & 0xFFu) << (8 * (i & 3));
    l[i >> 2] |= ((uint32_t)(int)lf & 0xFFu) << (8 * (i & 3));
  }
  // lane: elements 8u .. 8u+7 (u = lane % 4) of 32-element panel lane / 4
  const int u = lane & 3;
  uint8_t *grp = dig + (size_t)(b * J + j) * kGroupBytes;
  uint8_t *p = grp + (lane >> 2) * kPanel;
  constexpr bool Q6 = W == TCB_Q6_K, NAT = W != TCB_Q4_K;
  if (NAT) {
    const int o = 16 * (u & 1) + 4 * (u >> 1);
    uint32_t *ph = reinterpret_cast<uint32_t *>(p + (2 * r) * 32 + o), *pl = reinterpret_cast<uint32_t *>(p + (2 * r + 1) * 32 + o);
    ph[0] = h[0];
    ph[2] = h[1];
    pl[0] = l[0];
    pl[2] = l[1];
  } else {
    *reinterpret_cast<uint2 *>(p + (2 * r) * 32 + 8 * u) = make_uint2(h[0], h[1]);
    *reinterpret_cast<uint2 *>(p + (2 * r + 1) * 32 + 8 * u) = make_uint2(l[0], l[1]);
  }
  // sub-block sums: 16 elements (lane pairs) for Q6_K, 32 (lane quads) for Q4_K
  sh += __shfl_xor_sync(0xFFFFFFFFu, sh, 1);
  sl += __shfl_xor_sync(0xFFFFFFFFu, sl, 1);
  if (!Q6) {
    sh += __shfl_xor_sync(0xFFFFFFFFu, sh, 2);
    sl += __shfl_xor_sync(0xFFFFFFFFu, sl, 2);
  }
  uint8_t *ps = grp + 8 * kPanel;
  const int kslot = Q6 ? 2 * (lane >> 2) + (u >> 1) : (lane >> 2);
  if (W == TCB_Q4_0) {
    if (u == 0) reinterpret_cast<int *>(ps)[kslot * 4 + r] = 254 * sh + sl;
  } else if (Q6 ? (u & 1) == 0 : u == 0) {
    ps[(2 * r) * 16 + kslot] = (uint8_t)(sh >> 6);
    ps[128 + (2 * r) * 16 + kslot] = (uint8_t)(sh & 63);
    ps[(2 * r + 1) * 16 + kslot] = (uint8_t)(sl >> 6);
    ps[128 + (2 * r + 1) * 16 + kslot] = (uint8_t)(sl & 63);
  }
  if (W == TCB_Q4_K && lane < 8) {
    // k-slots 8..15 of the Q4_K sums (eight sub-blocks only)
    ps[(2 * r + (lane >> 2)) * 16 + 8 + (lane & 3) * 2] = 0;
    ps[(2 * r + (lane >> 2)) * 16 + 9 + (lane & 3) * 2] = 0;
    ps[128 + (2 * r + (lane >> 2)) * 16 + 8 + (lane & 3) * 2] = 0;
    ps[128 + (2 * r + (lane >> 2)) * 16 + 9 + (lane & 3) * 2] = 0;
  }
  if (lane == 0) {
    sig[((size_t)b * 4 + r) * J + j] = amax * (1.f / 127.f);
    bad[(size_t)b * 16 + m] = fin ? 0 : 1;
    for (int mm = m + 4 * J; mm < 16; mm += 4 * J) bad[(size_t)b * 16 + mm] = 0;  // flags of rows past 4J
  }
}

// ---------------------------------------------------------------- product

// Q4_K superblock, the 16 rows g, g + 8 (+ 16h) of this warp: operands to
// registers, the stage released, then the MMAs and the integer scale math,
// folded into facc[q][j] (row g + 8q, x row 4j + t).
template <int J, class Rel>
__device__ __forceinline__ void block_q4k(const uint8_t *r0, const uint8_t *dg, const float *sg, int g, int t, bool has,
                                          const Rel &rel, int lane, float (&facc)[2][J]) {
  constexpr int P = Fmt<TCB_Q4_K>::kPitch;
  uint4 hd[2];
  uint2 qs[2][4];
  if (has) {
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const uint8_t *rp = r0 + 8 * q * P;
      hd[q] = *reinterpret_cast<const uint4 *>(rp);
#pragma unroll
      for (int c = 0; c < 4; c++) qs[q][c] = *reinterpret_cast<const uint2 *>(rp + 16 + 32 * c + 8 * t);
    }
  }
  __syncwarp();
  if (lane == 0) rel();
  if (!has) return;
  // scales and mins of sub-blocks 0-3 / 4-7, one byte each
  uint32_t sc[2][2], mn[2][2];
  float dd[2], dmn[2];
#pragma unroll
  for (int q = 0; q < 2; q++) {
    const uint4 v = hd[q];
    sc[q][0] = v.y & 0x3F3F3F3Fu;
    mn[q][0] = v.z & 0x3F3F3F3Fu;
    sc[q][1] = (v.w & 0x0F0F0F0Fu) | ((v.y >> 2) & 0x30303030u);
    mn[q][1] = ((v.w >> 4) & 0x0F0F0F0Fu) | ((v.z >> 2) & 0x30303030u);
    dd[q] = half_exact(v.x & 0xFFFFu) * 0.0625f;
    dmn[q] = half_exact(v.x >> 16) * (1.f / 254.f);
  }
  int ah[2][J], al[2][J];
#pragma unroll
  for (int j = 0; j < J; j++) ah[0][j] = ah[1][j] = al[0][j] = al[1][j] = 0;
#pragma unroll
  for (int sb = 0; sb < 8; sb++) {
    const int c = sb >> 1;
    const uint32_t msk = (sb & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
    const uint32_t sel = 0x4440u + (uint32_t)(sb & 3);
    int scp[2];
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const int s8 = (int)__byte_perm(sc[q][sb >> 2], 0u, sel);
      scp[q] = (sb & 1) ? s8 : s8 << 4;
    }
    const uint32_t a0 = qs[0][c].x & msk, a1 = qs[1][c].x & msk, a2 = qs[0][c].y & msk, a3 = qs[1][c].y & msk;
#pragma unroll
    for (int j = 0; j < J; j++) {
      const uint2 bf = *reinterpret_cast<const uint2 *>(dg + j * kGroupBytes + sb * kPanel + g * 32 + 8 * t);
      int D[4] = {0, 0, 0, 0};
      imma_u8(D, a0, a1, a2, a3, bf.x, bf.y);
      ah[0][j] += scp[0] * D[0];
      al[0][j] += scp[0] * D[1];
      ah[1][j] += scp[1] * D[2];
      al[1][j] += scp[1] * D[3];
    }
  }
  // mins term: sum_j m_j S_j, k-slots = the 8 sub-blocks (lanes t < 2)
  const uint32_t m0 = t == 0 ? mn[0][0] : t == 1 ? mn[0][1] : 0u;
  const uint32_t m1 = t == 0 ? mn[1][0] : t == 1 ? mn[1][1] : 0u;
#pragma unroll
  for (int j = 0; j < J; j++) {
    const uint8_t *ps = dg + j * kGroupBytes + 8 * kPanel + g * 16 + 4 * t;
    int Mh[4] = {0, 0, 0, 0}, Ml[4] = {0, 0, 0, 0};
    imma_u8_k16(Mh, m0, m1, *reinterpret_cast<const uint32_t *>(ps));
    imma_u8_k16(Ml, m0, m1, *reinterpret_cast<const uint32_t *>(ps + 128));
    const float s = sg[j];
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const float main = fmaf((float)al[q][j], 1.f / 254.f, (float)ah[q][j]);
      // 254 * MH + ML, MH / ML = 64 * high + low of each digit's sums
      const float mt = (float)(254 * (64 * Mh[2 * q] + Ml[2 * q]) + 64 * Mh[2 * q + 1] + Ml[2 * q + 1]);
      const float v = fmaf(-dmn[q], mt, dd[q] * main);
      facc[q][j] = fmaf(s, v, facc[q][j]);
    }
  }
}

// Q6_K superblock: value = d * sc_j * (q - 32), q 6-bit (4 low bits in ql,
// 2 high in qh), sixteen 16-element sub-blocks with int8 scales (TR
// tensor/quant.go Q6_K dequant).  Each sub-block is one k16 MMA (u8 codes x
// s8 digits; lane t's k-slots are elements 4t..4t+3 of the sub-block), its
// signed scale applied in integers; the -32 offset is sum_j sc_j S_j, one
// k16 MMA per digit-sum byte with A = the 16 scales.
template <int J, class Rel>
__device__ __forceinline__ void block_q6k(const uint8_t *r0, const uint8_t *dg, const float *sg, int g, int t, bool has,
                                          const Rel &rel, int lane, float (&facc)[2][J]) {
  constexpr int P = Fmt<TCB_Q6_K>::kPitch;
  uint32_t ql[2][2][4], qh[2][2][2], scw[2][4];
  float dd[2];
  if (has) {
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const uint8_t *rp = r0 + 8 * q * P;
#pragma unroll
      for (int n = 0; n < 2; n++) {
#pragma unroll
        for (int c = 0; c < 4; c++) ql[q][n][c] = ld4(rp + 64 * n + 16 * c + 4 * t);
#pragma unroll
        for (int c = 0; c < 2; c++) qh[q][n][c] = ld4(rp + 128 + 32 * n + 16 * c + 4 * t);
      }
#pragma unroll
      for (int c = 0; c < 4; c++) scw[q][c] = ld4(rp + 192 + 4 * c);
      dd[q] = half_exact(*reinterpret_cast<const uint16_t *>(rp + 208));
    }
  }
  __syncwarp();
  if (lane == 0) rel();
  if (!has) return;
  int ah[2][J], al[2][J];
#pragma unroll
  for (int j = 0; j < J; j++) ah[0][j] = ah[1][j] = al[0][j] = al[1][j] = 0;
#pragma unroll
  for (int n = 0; n < 2; n++)
#pragma unroll
    for (int k = 0; k < 4; k++) {
      // 32-element group 4n + k: sub-blocks 8n + 2k + s, s = 0, 1
#pragma unroll
      for (int s2 = 0; s2 < 2; s2++) {
        uint32_t qa[2];
        int scs[2];
#pragma unroll
        for (int q = 0; q < 2; q++) {
          const uint32_t lo = (ql[q][n][2 * (k & 1) + s2] >> (4 * (k >> 1))) & 0x0F0F0F0Fu;
          const uint32_t hi = ((qh[q][n][s2] >> (2 * k)) & 0x03030303u) << 4;
          qa[q] = lo | hi;
          const int si = 8 * n + 2 * k + s2;  // scale index 0..15
          scs[q] = (int)(signed char)(scw[q][si >> 2] >> (8 * (si & 3)));
        }
#pragma unroll
        for (int j = 0; j < J; j++) {
          const uint32_t bf = *reinterpret_cast<const uint32_t *>(dg + j * kGroupBytes + (4 * n + k) * kPanel + g * 32 +
                                                                  8 * t + 4 * s2);
          int D[4] = {0, 0, 0, 0};
          imma_u8_k16(D, qa[0], qa[1], bf);
          ah[0][j] += scs[0] * D[0];
          al[0][j] += scs[0] * D[1];
          ah[1][j] += scs[1] * D[2];
          al[1][j] += scs[1] * D[3];
        }
      }
    }
  // code offset: sum_j sc_j S_j, k-slots = the 16 sub-blocks (lane t: 4t..4t+3)
  const uint32_t sa0 = t == 0 ? scw[0][0] : t == 1 ? scw[0][1] : t == 2 ? scw[0][2] : scw[0][3];
  const uint32_t sa1 = t == 0 ? scw[1][0] : t == 1 ? scw[1][1] : t == 2 ? scw[1][2] : scw[1][3];
#pragma unroll
  for (int j = 0; j < J; j++) {
    const uint8_t *ps = dg + j * kGroupBytes + 8 * kPanel + g * 16 + 4 * t;
    int Oh[4] = {0, 0, 0, 0}, Ol[4] = {0, 0, 0, 0};
    imma_s8_k16(Oh, sa0, sa1, *reinterpret_cast<const uint32_t *>(ps));
    imma_s8_k16(Ol, sa0, sa1, *reinterpret_cast<const uint32_t *>(ps + 128));
    const float s = sg[j];
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const int mh = ah[q][j] - 32 * (64 * Oh[2 * q] + Ol[2 * q]);
      const int ml = al[q][j] - 32 * (64 * Oh[2 * q + 1] + Ol[2 * q + 1]);
      const float main = fmaf((float)ml, 1.f / 254.f, (float)mh);
      facc[q][j] = fmaf(s, dd[q] * main, facc[q][j]);
    }
  }
}

// Q4_0: eight 18-byte blocks (d, then 16 bytes: element i in the low nibble
// of byte i, element 16 + i in the high nibble) make one 256-element unit;
// value = d * (q - 8) (TR tensor/quant.go Q4_0 dequant).  Each block is one
// k32 MMA (lane t: low nibbles of bytes 4t..4t+3 = elements 4t..4t+3, high
// nibbles = elements 16+4t..), then per (weight row, x row) with the digit
// sums S of the block:  acc += d * sigma / 254 * ((254 Dh + Dl) - 8 (254 Sh + Sl)).
template <int J, class Rel>
__device__ __forceinline__ void block_q40(const uint8_t *r0, const uint8_t *dg, const float *sg, int g, int t, bool has,
                                          const Rel &rel, int lane, float (&facc)[2][J]) {
  constexpr int P = Fmt<TCB_Q4_0>::kPitch;
  uint32_t qw[2][8];
  float dd[2][8];
  if (has) {
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const uint8_t *rp = r0 + 8 * q * P;
#pragma unroll
      for (int k = 0; k < 8; k++) {
        qw[q][k] = ld4(rp + 18 * k + 2 + 4 * t);
        dd[q][k] = half_exact(*reinterpret_cast<const uint16_t *>(rp + 18 * k));
      }
    }
  }
  __syncwarp();
  if (lane == 0) rel();
  if (!has) return;
  float sgs[J];
#pragma unroll
  for (int j = 0; j < J; j++) sgs[j] = sg[j] * (1.f / 254.f);
#pragma unroll
  for (int k = 0; k < 8; k++) {
    const uint32_t a0 = qw[0][k] & 0x0F0F0F0Fu, a1 = qw[1][k] & 0x0F0F0F0Fu;
    const uint32_t a2 = (qw[0][k] >> 4) & 0x0F0F0F0Fu, a3 = (qw[1][k] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
    for (int j = 0; j < J; j++) {
      const uint8_t *pj = dg + j * kGroupBytes;
      const uint2 bf = *reinterpret_cast<const uint2 *>(pj + k * kPanel + g * 32 + 8 * t);
      const int so = 8 * reinterpret_cast<const int *>(pj + 8 * kPanel)[k * 4 + t];
      int D[4] = {0, 0, 0, 0};
      imma_u8(D, a0, a1, a2, a3, bf.x, bf.y);
#pragma unroll
      for (int q = 0; q < 2; q++) {
        const int v = 254 * D[2 * q] + D[2 * q + 1] - so;
        facc[q][j] = fmaf(dd[q][k] * sgs[j], (float)v, facc[q][j]);
      }
    }
  }
}

template <int W, int J>
__global__ void __launch_bounds__(32 * kWarps, 1) k_mvrows(const __grid_constant__ CUtensorMap tmap, const Params a) {
  constexpr int kPitch = Fmt<W>::kPitch, kBB = Fmt<W>::kBB;
  constexpr int kStage = kRows * kPitch;
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + kBarOff);  // [S]
  int *relcnt = reinterpret_cast<int *>(full + kMaxS);         // [S] warps' releases of each buffer
  uint64_t *xfull = full + 2 * kMaxS;                          // digits of the K range landed
  uint64_t *tfree = xfull + 1;                                 // [slots] partials summed
  int *cnt = reinterpret_cast<int *>(sm + kCntOff);            // [slots] warps done with the tile
  float *part = reinterpret_cast<float *>(sm + kPartOff);      // [slots][kC][4J][16]
  const uint8_t *digs = sm + a.xoff;                           // [nbr][J][9][8][32]
  const float *sigs = reinterpret_cast<const float *>(sm + a.xoff + a.nbr * J * kGroupBytes);  // [nbr][4][J]
  uint8_t *stages = sm + a.soff;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int range = (int)blockIdx.x % a.ksplit;
  const int gsz = (int)gridDim.x / a.ksplit;     // CTAs of one K range
  const int gidx = (int)blockIdx.x / a.ksplit;
  const int b0 = range * a.nbr;
  const int nbr = min(a.nbr, a.nb - b0);         // superblocks of this range
  const int my_tiles = (a.tiles - gidx + gsz - 1) / gsz;
  const int nstages = my_tiles * a.nch;
  constexpr int kPartFloats = 4 * J * 16;        // one warp's partials of a tile
  const bool producer = threadIdx.x == 0;

  if (producer) {
    for (int s = 0; s < a.S; s++) {
      mbar_init(&full[s], 1);
      relcnt[s] = 0;
    }
    mbar_init(xfull, 1);
    for (int s = 0; s < a.slots; s++) {
      mbar_init(&tfree[s], 1);
      cnt[s] = 0;
    }
    fence_barrier_init();
  }
  __syncthreads();
  // box of stage it: superblocks b0 + 8 (it % nch) .. (8-byte elements; a
  // multiple of 8 superblocks for Q6_K), rows of tile gidx + (it / nch) gsz
  auto bx = [&](int it) { return (b0 + (it % a.nch) * kBlk) * kBB / 8; };
  auto by = [&](int it) { return (gidx + (it / a.nch) * gsz) * kRows; };
  if (producer) {
    // the split-K sum is the next kernel when ksplit > 1: its CTAs would
    // wait on this grid from every SM, so it is released at the end
    if (a.ksplit == 1) pdl_launch_dependents();
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
    // the weights are only read: the first stages go out before the
    // previous kernel has finished; the digits are its successor's
    const int first = nstages < a.S ? nstages : a.S;
    for (int it = 0; it < first; it++) {
      mbar_expect_tx(&full[it], (uint32_t)kStage);
      tma_load_2d(stages + it * kStage, &tmap, bx(it), by(it), &full[it]);
    }
    pdl_wait();
    const uint32_t db = (uint32_t)nbr * J * kGroupBytes, sb = (uint32_t)nbr * 16 * J;
    mbar_expect_tx(xfull, db + sb);
    bulk_g2s(sm + a.xoff, a.dig + (size_t)b0 * J * kGroupBytes, db, xfull);
    bulk_g2s(sm + a.xoff + a.nbr * J * kGroupBytes, a.sig + (size_t)b0 * 4 * J, sb, xfull);
  }
  // x, c and the digits may be written by the previous kernels of the stream
  pdl_wait();
  // a NaN or Inf anywhere in x: TR's float path for the whole call
  uint32_t anyb = 0;
  for (int i = lane; i < a.nb; i += 32) {
    const uint4 v = reinterpret_cast<const uint4 *>(a.bad)[i];
    anyb |= v.x | v.y | v.z | v.w;
  }
  const bool slow = __any_sync(0xFFFFFFFFu, anyb != 0);

  const int g = lane >> 2, t = lane & 3;
  const int bw = warp & (kBlk - 1), hw = warp >> 3;  // superblock of the stage, 16-row half
  {
    bool ok = true;
    if (lane == 0) ok = wait_bar(xfull, 0u, a.err);
    if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return;
  }
  float facc[2][J];
#pragma unroll
  for (int q = 0; q < 2; q++)
#pragma unroll
    for (int j = 0; j < J; j++) facc[q][j] = 0.f;
  int it = 0;
  for (int ti = 0; ti < my_tiles; ti++) {
    for (int ch = 0; ch < a.nch; ch++, it++) {
      const int buf = it % a.S;
      // a warp's release of this stage (lane 0, after the warp's reads of it):
      // the last of the 16 warps refills the buffer with stage it + S at once
      const auto rel = [&]() {
        __threadfence_block();
        if (atomicAdd(&relcnt[buf], 1) % kC == kC - 1 && it + a.S < nstages) {
          mbar_expect_tx(&full[buf], (uint32_t)kStage);
          tma_load_2d(stages + buf * kStage, &tmap, bx(it + a.S), by(it + a.S), &full[buf]);
        }
      };
      bool ok = true;
      if (lane == 0) ok = wait_bar(&full[buf], (uint32_t)((it / a.S) & 1), a.err);
      if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return;
      const int lb = ch * kBlk + bw;  // superblock of the range
      const uint8_t *r0 = stages + buf * kStage + (16 * hw + g) * kPitch + bw * kBB;
      const uint8_t *dg = digs + (size_t)lb * J * kGroupBytes;
      const float *sg = sigs + (size_t)lb * 4 * J + t * J;
      if constexpr (W == TCB_Q4_K) block_q4k<J>(r0, dg, sg, g, t, lb < nbr, rel, lane, facc);
      else if constexpr (W == TCB_Q4_0) block_q40<J>(r0, dg, sg, g, t, lb < nbr, rel, lane, facc);
      else block_q6k<J>(r0, dg, sg, g, t, lb < nbr, rel, lane, facc);
      if (ch == a.nch - 1) {
        // the tile: this warp's partials (rows g + 8q of half hw, x rows
        // 4j + t) into the slot; the last warp to finish sums them
        const int slot = ti % a.slots, use = ti / a.slots;
        if (use > 0) {
          bool okf = true;
          if (lane == 0) okf = spin_bar_ns(&tfree[slot], (uint32_t)((use - 1) & 1), a.err, 32);
          if (!__shfl_sync(0xFFFFFFFFu, okf, 0)) return;
        }
        float *pt = part + (slot * kC + warp) * kPartFloats + g;
#pragma unroll
        for (int j = 0; j < J; j++)
#pragma unroll
          for (int q = 0; q < 2; q++) {
            pt[(4 * j + t) * 16 + 8 * q] = facc[q][j];
            facc[q][j] = 0.f;
          }
        __syncwarp();
        int last = 0;
        if (lane == 0) {
          __threadfence_block();
          last = atomicAdd(&cnt[slot], 1) == kC - 1;
        }
        if (__shfl_sync(0xFFFFFFFFu, last, 0)) {
          __threadfence_block();
          const int row = (gidx + ti * gsz) * kRows + lane;
          if (!slow && row < a.N) {
            // row lane: half lane / 16, the 8 superblock warps in order
            const float *ps = part + (slot * kC + 8 * (lane >> 4)) * kPartFloats + (lane & 15);
            for (int m = 0; m < a.M; m++) {
              float v = 0.f;
#pragma unroll
              for (int w = 0; w < kBlk; w++) v += ps[w * kPartFloats + m * 16];
              if (a.ksplit == 1) store_out(a.c, (long)m * a.ldc + row, a.cdt, v, a.accumulate != 0);
              else a.part[((size_t)range * 4 * J + m) * a.N + row] = v;
            }
          }
          __syncwarp();
          if (lane == 0) {
            cnt[slot] = 0;
            mbar_arrive(&tfree[slot]);
          }
        }
      }
    }
  }
  if (slow && range == 0) {
    // TR's float path, one warp per output
    const long rowBytes = (long)a.nb * kBB;
    for (int ti = 0; ti < my_tiles; ti++) {
      const int r0 = (gidx + ti * gsz) * kRows;
      for (int o = warp; o < kRows * a.M; o += kC) {
        const int n = r0 + o / a.M, m = o % a.M;
        if (n >= a.N) continue;
        float accs[1] = {0.0f};
        const void *xrow = static_cast<const char *>(a.x) + (size_t)m * a.ldx * (a.xdt == TCB_F32 ? 4 : 2);
        lane_row_float<W, 1>(a.w + (long)n * rowBytes, a.K, lane, XGlobal{xrow, 0, a.xdt}, accs);
        const float s = warp_sum(accs[0]);
        if (lane == 0) store_out(a.c, (long)m * a.ldc + n, a.cdt, s, a.accumulate != 0);
      }
    }
  }
}

// ---------------------------------------------------------------- split-K sum

// y[m][n] (+)= sum over ranges r (in order) of part[r][m][n]
__global__ void __launch_bounds__(256) k_rows_red(const float *part, int ksplit, int J4, int M, int N, int nb,
                                                 const uint8_t *bad, void *c, int cdt, long ldc, int accumulate) {
  pdl_wait();
  __shared__ int slow;
  if (threadIdx.x < 32) {
    uint32_t any = 0;
    for (int i = threadIdx.x; i < nb; i += 32) {
      const uint4 v = reinterpret_cast<const uint4 *>(bad)[i];
      any |= v.x | v.y | v.z | v.w;
    }
    const bool s = __any_sync(0xFFFFFFFFu, any != 0);
    if (threadIdx.x == 0) slow = s;
  }
  __syncthreads();
  if (slow) return;  // the product kernel wrote TR's float path
  const long total = (long)M * N;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int m = (int)(i / N), n = (int)(i % N);
    float v = 0.f;
    for (int r = 0; r < ksplit; r++) v += part[((size_t)r * J4 + m) * N + n];
    store_out(c, (long)m * ldc + n, cdt, v, accumulate != 0);
  }
}

}  // namespace mvr

// The plan of the Q4_K / Q6_K float product of 2..16 rows (kind 3; plan.cbc
// holds the format).  ksplit and the stage count come from a cost model in
// units of one stage (32 rows x 8 superblocks): the most a CTA streams, plus
// a fixed charge for the extra launch and partials of a split.
// Q6_K rows (210-byte superblocks) are only 2-byte aligned; the copies need
// whole groups of 8 superblocks (K a multiple of 2048, K ranges of 8k).
MvPlan rows_plan(int wtype, int N, int K, const void *w, int sms, int M) {
  using namespace mvr;
  MvPlan pl{};
  if (wtype != TCB_Q4_K && wtype != TCB_Q6_K && wtype != TCB_Q4_0) return pl;
  const bool q6 = wtype == TCB_Q6_K;  // Q4_0 units of 8 blocks stage like Q4_K superblocks
  const int bb = q6 ? mvr::Fmt<TCB_Q6_K>::kBB : mvr::Fmt<TCB_Q4_K>::kBB;
  const int pitch = q6 ? mvr::Fmt<TCB_Q6_K>::kPitch : mvr::Fmt<TCB_Q4_K>::kPitch;
  const int box8 = q6 ? mvr::Fmt<TCB_Q6_K>::kBox8 : mvr::Fmt<TCB_Q4_K>::kBox8;
  const int stage = kRows * pitch;
  const int nb = K / 256;
  const long rowBytes = (long)nb * bb;
  if (M < 2 || M > 16 || N <= 0 || K % 256 || nb == 0 || rowBytes % 16 || reinterpret_cast<uintptr_t>(w) % 16 ||
      (q6 && nb % 8))
    return pl;
  auto enc = tensor_map_encoder();
  if (!enc) return pl;
  const int J = (M + 3) / 4;
  const int tiles = (N + kRows - 1) / kRows;
  const int slots = J <= 2 ? 2 : 1;
  const int part_bytes = slots * kC * 4 * J * 16 * 4;
  double best = 1e30;
  int bk = 0, bS = 0, bnbr = 0, bxoff = 0, bsoff = 0;
  // K ranges are whole stages (8 superblocks; a box always moves 8): a
  // shorter range would idle warps and fetch its neighbours' superblocks
  for (int ks = 1; ks <= 16 && ks <= sms; ks++) {
    const int nbr = ((nb + ks - 1) / ks + 7) & ~7;
    if ((ks - 1) * nbr >= nb || (ks > 1 && nbr >= nb)) continue;  // an empty range, or no split
    const int xoff = (kPartOff + part_bytes + 127) & ~127;
    const int soff = (xoff + nbr * J * kGroupBytes + nbr * 16 * J + 127) & ~127;
    int S = (kSmemMax - soff) / stage;
    if (S > kMaxS) S = kMaxS;
    if (S < 2) continue;
    // stages the busiest CTA streams (a stage is about 0.9 us at the copy
    // rate), a split's extra launch and partials charged as four stages, a
    // two-deep pipeline as 10 % more
    const int gsz = sms / ks;
    const int per = (tiles + gsz - 1) / gsz;
    const int stg = per * ((nbr + kBlk - 1) / kBlk);
    const double cost = stg * (S < 3 ? 1.1 : 1.0) + (ks > 1 ? 4.0 : 0.0);
    if (cost < best) {
      best = cost;
      bk = ks;
      bS = S;
      bnbr = nbr;
      bxoff = xoff;
      bsoff = soff;
    }
  }
  if (bk == 0) return pl;
  const int gsz = sms / bk;
  pl.kind = 3;
  pl.tiles = tiles;
  pl.ksplit = bk;
  pl.cpk = bnbr;
  pl.nch = (bnbr + kBlk - 1) / kBlk;
  pl.cbc = wtype;
  pl.stages = bS;
  pl.pitch = pitch;
  pl.xoff = bxoff;
  pl.soff = bsoff;
  pl.toff = slots;  // partial slots (kind 3)
  pl.smem = bsoff + bS * stage;
  pl.grid = bk * (tiles < gsz ? tiles : gsz);
  pl.rows = 4 * J;
  pl.xstride = 0;
  pl.split_bytes = layout(nb, J, bk, N).end;
  CUtensorMap tm;
  cuuint64_t gdim[2] = {(cuuint64_t)(rowBytes / 8), (cuuint64_t)N};
  cuuint64_t gstride[1] = {(cuuint64_t)rowBytes};
  cuuint32_t box[2] = {(cuuint32_t)box8, (cuuint32_t)kRows};
  cuuint32_t estr[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), gdim, gstride, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return pl;
  memcpy(pl.tmap, &tm, sizeof tm);
  pl.ok = true;
  return pl;
}

namespace {
cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t s, cudaLaunchAttribute *at) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cfg;
}

template <int W, int J>
cudaError_t rows_launch_j(const MvPlan &pl, mvr::Params &a, cudaStream_t s) {
  using namespace mvr;
  cudaLaunchAttribute at[1];
  const int warps = a.nb * 4 * J;
  cudaLaunchConfig_t c1 = pdl_cfg(dim3((warps + 7) / 8), dim3(256), 0, s, at);
  cudaError_t e = cudaLaunchKernelEx(&c1, k_xdig<J, W>, a.x, a.xdt, a.ldx, a.M, a.nb, const_cast<uint8_t *>(a.dig),
                                     const_cast<float *>(a.sig), const_cast<uint8_t *>(a.bad));
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(k_mvrows<W, J>, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return e;
  CUtensorMap tm;
  memcpy(&tm, pl.tmap, sizeof tm);
  cudaLaunchConfig_t c2 = pdl_cfg(dim3(pl.grid), dim3(32 * mvr::kWarps), pl.smem, s, at);
  e = cudaLaunchKernelEx(&c2, k_mvrows<W, J>, tm, a);
  if (e != cudaSuccess || pl.ksplit == 1) return e;
  const long total = (long)a.M * a.N;
  int blocks = (int)((total + 255) / 256);
  if (blocks > 4 * 148) blocks = 4 * 148;
  cudaLaunchConfig_t c3 = pdl_cfg(dim3(blocks), dim3(256), 0, s, at);
  return cudaLaunchKernelEx(&c3, k_rows_red, (const float *)a.part, a.ksplit, 4 * J, a.M, a.N, a.nb, a.bad, a.c, a.cdt,
                            a.ldc, a.accumulate);
}
}  // namespace

cudaError_t rows_launch(const MvPlan &pl, int N, int K, const void *w, const void *x, int xdt, long ldx, void *c,
                        int cdt, long ldc, int accumulate, int M, int *err, void *scratch, cudaStream_t s) {
  using namespace mvr;
  if (!pl.ok || pl.kind != 3 || M < 1 || M > pl.rows || !scratch) return cudaErrorInvalidValue;
  const int J = pl.rows / 4;
  Params a{};
  a.w = static_cast<const uint8_t *>(w);
  a.N = N;
  a.K = K;
  a.nb = K / 256;
  a.M = M;
  a.x = x;
  a.xdt = xdt;
  a.ldx = ldx;
  a.c = c;
  a.cdt = cdt;
  a.ldc = ldc;
  a.accumulate = accumulate;
  a.tiles = pl.tiles;
  a.ksplit = pl.ksplit;
  a.nbr = pl.cpk;
  a.nch = pl.nch;
  a.S = pl.stages;
  a.slots = pl.toff;
  a.soff = pl.soff;
  a.xoff = pl.xoff;
  const Layout L = layout(a.nb, J, pl.ksplit, N);
  uint8_t *base = static_cast<uint8_t *>(scratch);
  a.dig = base + L.dig;
  a.sig = reinterpret_cast<const float *>(base + L.sig);
  a.bad = base + L.bad;
  a.part = reinterpret_cast<float *>(base + L.part);
  a.err = err;
#define TCB_ROWS_J(JJ)                                                                \
  case JJ:                                                                            \
    return pl.cbc == TCB_Q6_K   ? rows_launch_j<TCB_Q6_K, JJ>(pl, a, s)               \
           : pl.cbc == TCB_Q4_0 ? rows_launch_j<TCB_Q4_0, JJ>(pl, a, s)               \
                                : rows_launch_j<TCB_Q4_K, JJ>(pl, a, s);
  switch (J) {
    TCB_ROWS_J(1)
    TCB_ROWS_J(2)
    TCB_ROWS_J(3)
    TCB_ROWS_J(4)
  }
#undef TCB_ROWS_J
  return cudaErrorInvalidValue;
}

}  // namespace tcb
