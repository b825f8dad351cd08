// tcb_mv_q4k.cu - batch-1 Q4_K matvec, float path (x in f32/bf16/f16):
//
//   y[n] (+)= sum_k x[k] * dequant(W)[n, k]     W: [N, K] Q4_K blocks
//
// The kernel is a weight stream: every byte of W is read once, so its speed
// is HBM bandwidth, and at 25-140 MB per call the launch ramp and tail are a
// large part of it.  The design therefore keeps each CTA small (about
// 90-110 KB of shared memory, 10 warps) so that two fit on an SM: with
// programmatic dependent launch the next call's CTAs start on an SM as soon
// as one of this call's CTAs leaves it, and stream their first weight
// stages while this call finishes.
//
//  * A tile is 32 rows.  A stage is one 2-D TMA box of those 32 rows x 8
//    Q4_K blocks (1152 bytes + 16 bytes of padding per row, so the staged
//    row pitch is 16 mod 128 and the lane reads below are conflict-free),
//    issued by a producer warp; rows past N and bytes past the row end are
//    zero-filled by the copy engine.  Compute warp w (of 8) takes block w of
//    every stage for both 16-row slices of the tile, sharing the x
//    fragments (measured faster than 16-row tiles, although those balance
//    the CTAs better).
//  * x is split per 32-element sub-block into two int8 digits,
//    x ~= sigma * (h + l/254), sigma = amax/127 (relative error of the x
//    representation below 1/(2*127*254) of the sub-block maximum).  Each
//    warp digitises only the blocks it owns, straight into the B-operand
//    layout of its MMAs.
//  * Dot products: int8 mma.sync m16n8k32 (u8 weight codes x s8 digits ->
//    s32, exact).  In MMA set s (s = 0, 1), k-slot group t (lanes with
//    t = lane % 4) carries sub-block c(s, t) = 4*(t/2) + t%2 + 2*s, eight of
//    its elements per round r (0..3).  B column n = 2*t' + digit belongs to
//    k-slot group t' = n/2: lane (g, t) supplies column g only if g/2 == t
//    and zeros otherwise (a per-lane constant, no per-MMA masking), so
//    column n sums the k-slots of its own sub-block alone.  After the four
//    rounds of set s a lane holds, for rows g and g+8, both digit sums of
//    sub-block c(s, t): every (row, sub-block) pair of the 16x8 slice exactly
//    once.  Lanes with t odd read high nibbles in place as 16*q (one LOP3 per
//    four codes); their sigma' carries the 1/16.
//  * Scale epilogue per (row, sub-block): TR's get_scale_min_k4 decode, two
//    sub-blocks at a time in 16-bit lanes, then
//    acc += d*sc*sigma'*(254*Dh + Dl) - dmin*m*S, S the sub-block sum of x.
//    The MMAs of a block are issued before the epilogue of the warp's
//    previous block, so tensor-core latency hides behind ALU work.
//  * Tile partials: each warp's row sums go to shared memory; an epilogue
//    warp adds the 8 warp partials of a row in warp order and stores y.
//    Results do not depend on the grid or on timing.
//  * A NaN or Inf in x (any sub-block sum non-finite) sends the whole call
//    down TR's fp32 path, one warp per row, so NaN/Inf propagate as in TR.
#include <string.h>

#include "tcb_common.cuh"
#include "tcb_matvec.h"
#include "tcb_mv_ptx.cuh"
#include "tcb_simt.cuh"

namespace tcb {
namespace mvk {

using namespace mv;

constexpr int kC = 8;                       // compute warps
constexpr int kProd = kC;                   // producer warp
constexpr int kEpi = kC + 1;                // epilogue warp
constexpr int kWarps = kC + 2;
constexpr int kRows = 32;                   // rows per tile (one box)
constexpr int kHalves = kRows / 16;         // 16-row MMA slices per tile
constexpr int kBlk = 8;                     // Q4_K blocks per box
constexpr int kBox8 = 146;                  // box width, 8-byte elements (8 * 18 + 2)
constexpr int kPitch = kBox8 * 8;           // staged row pitch (1168 = 16 mod 128)
constexpr int kBoxBytes = kRows * kPitch;   // one stage
constexpr int kSlots = 4;                   // tile partial slots in flight
constexpr int kFrag = 512, kScl = 64;       // per block: B fragments, lane scales
constexpr int kBarOff = 0, kFlagOff = 256, kNormOff = 288, kPartOff = 512;
constexpr int kPartBytes = kSlots * kC * kRows * 4;
constexpr int kXOff = kPartOff + kPartBytes;

struct Params {
  const uint8_t *w;
  int N, K, nb;
  const void *x;
  int xdt;
  void *c;
  int cdt;
  int accumulate;
  int tiles, nch, S;
  int *err;
  int soff;         // stage offset in shared memory
  const float *nw;  // RMSNorm weight fused into the prologue (nullptr: none)
  float eps;
  const void *pf;   // weights of the next kernel of a chain, prefetched into L2 (or nullptr)
  size_t pf_bytes;
  int M;            // activation rows of this launch (1 .. MR of the kernel)
  long ldx, ldc;    // row strides of x and c, elements
  int xstride;      // bytes between the x regions of consecutive rows
  float *swi;       // SwiGLU output (M = 1, rows [G | U] of F each), or nullptr
  int swiF;         // F: tile t stages gate rows 16t.. and up rows F + 16t..
};

// x region: [nb][kFrag] B fragments ([set s][round pair rp][column n][16
// digits]), [nb][kScl] lane scales ([t][sigma'_c0, sigma'_c1, S_c0, S_c1]),
// then kFrag zero bytes for the lanes without a column.
__host__ __device__ inline int x_bytes(int nb) { return nb * (kFrag + kScl) + kFrag; }

struct Lane {
  const uint8_t *xb;  // B fragments of block 0 (or the zero bytes)
  int xs;             // per-block stride of xb (0 for the zero bytes)
  uint32_t mq;        // code nibble mask: low (t even) or high, in place (t odd)
  int woff;           // code group 2*(t/2) in a block
  int sh;             // byte of sub-block c(0, t) in its scale word
  bool lo;            // c(0, t) < 4
  uint32_t mlo, mhi;  // scale decode masks
  const float *scl;   // lane scales of block 0
};

__device__ __forceinline__ Lane make_lane(const uint8_t *xr, int nb, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const bool act = (g >> 1) == t;
  Lane q;
  q.xb = act ? xr + g * 16 : xr + nb * (kFrag + kScl);
  q.xs = act ? kFrag : 0;
  q.mq = (t & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
  q.woff = 16 + 64 * (t >> 1);
  q.sh = 8 * (t & 1);
  q.lo = t < 2;
  q.mlo = q.lo ? 0x003F003Fu : 0x000F000Fu;
  q.mhi = q.lo ? 0u : 0x00300030u;
  q.scl = reinterpret_cast<const float *>(xr + nb * kFrag) + t * 4;
  return q;
}

// eight consecutive activations (16-byte aligned when vec)
__device__ __forceinline__ void load8(const void *x, int e, int xdt, bool vec, float (&v)[8]) {
  if (vec && xdt == TCB_F32) {
    const float4 p = *reinterpret_cast<const float4 *>(static_cast<const float *>(x) + e);
    const float4 q = *reinterpret_cast<const float4 *>(static_cast<const float *>(x) + e + 4);
    v[0] = p.x, v[1] = p.y, v[2] = p.z, v[3] = p.w, v[4] = q.x, v[5] = q.y, v[6] = q.z, v[7] = q.w;
  } else if (vec) {
    const uint4 p = *reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(x) + e);
    const uint32_t u[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint16_t lo = (uint16_t)(u[i] & 0xFFFFu), hi = (uint16_t)(u[i] >> 16);
      v[2 * i] = xdt == TCB_BF16 ? bf16_to_f32(lo) : half_exact(lo);
      v[2 * i + 1] = xdt == TCB_BF16 ? bf16_to_f32(hi) : half_exact(hi);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = load_act(x, e + i, xdt);
  }
}

// Digits of the blocks this warp owns (bg = own, own + 8, ...), lane L
// taking elements 8L..8L+7 of a block: t0 = x*id + 1.5*2^23 rounds x*id to
// the nearest integer h in the low mantissa bits (one rounding of the exact
// product), the residual x*id - h is formed by one more fused op, and
// t1 = 254*residual + 1.5*2^23 gives l.  id only has to be consistent with
// sigma = 1/id, not exact, so it is the hardware reciprocal.  Returns false
// if a sub-block sum is not finite (a NaN or Inf in x, or a sum that
// overflows, which only sends the call down the exact fp32 path).
__device__ bool prep_warp(const Params &a, const void *x, uint8_t *xr, int own, int lane, float &ss, uint64_t *xgo) {
  constexpr float MAGIC = 12582912.0f;
  constexpr int NB = 4;  // blocks in flight per lane
  uint8_t *frag = xr;
  float *scl = reinterpret_cast<float *>(xr + a.nb * kFrag);
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  bool fin = true, told = xgo == nullptr;
  ss = 0.f;
  for (int base = own; base < a.nb; base += kC * NB) {
    float xv[NB][8];
#pragma unroll
    for (int j = 0; j < NB; j++) {
      const int bg = base + kC * j;
      if (bg < a.nb) load8(x, bg * 256 + 8 * lane, a.xdt, vec, xv[j]);
    }
    if (!told) {
      // the first x loads are out: the producer may issue the rest of the
      // weight stream behind them
      __syncwarp();
      if (lane == 0) mbar_arrive(xgo);
      told = true;
    }
    if (a.nw) {
      // fused RMSNorm: digits of x * w; the 1/rms factor is applied to the
      // row sums (the product is linear in x)
#pragma unroll
      for (int j = 0; j < NB; j++) {
        const int bg = base + kC * j;
        if (bg >= a.nb) break;
        const float4 w0 = *reinterpret_cast<const float4 *>(a.nw + bg * 256 + 8 * lane);
        const float4 w1 = *reinterpret_cast<const float4 *>(a.nw + bg * 256 + 8 * lane + 4);
        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) {
          ss = fmaf(xv[j][i], xv[j][i], ss);
          xv[j][i] = __fmul_rn(xv[j][i], wv[i]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < NB; j++) {
      const int bg = base + kC * j;
      if (bg >= a.nb) break;  // warp-uniform
      const float *v = xv[j];
      float am = fmaxf(fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))),
                       fmaxf(fmaxf(fabsf(v[4]), fabsf(v[5])), fmaxf(fabsf(v[6]), fabsf(v[7]))));
      float sum = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
      am = fmaxf(am, __shfl_xor_sync(0xFFFFFFFFu, am, 1));
      sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 1);
      am = fmaxf(am, __shfl_xor_sync(0xFFFFFFFFu, am, 2));
      sum += __shfl_xor_sync(0xFFFFFFFFu, sum, 2);
      if (!(__fsub_rn(sum, sum) == 0.0f)) fin = false;
      float id = 0.f, sigma = 0.f;
      if (am > 0.f) {
        const bool tiny = am < 1e-30f;  // keep sigma and id normal
        sigma = (tiny ? am * 18446744073709551616.0f : am) * (1.0f / 127.0f);
        id = rcp_approx(sigma) * (tiny ? 18446744073709551616.0f : 1.0f);
        if (tiny) sigma *= 5.421010862427522e-20f;
      }
      uint32_t bh[8], bl[8];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float t0 = fmaf(v[i], id, MAGIC);
        const float r = fmaf(v[i], id, -(t0 - MAGIC));
        bh[i] = __float_as_uint(t0);
        bl[i] = __float_as_uint(fmaf(r, 254.0f, MAGIC));
      }
      const uint2 ph = make_uint2(
          __byte_perm(__byte_perm(bh[0], bh[1], 0x0040), __byte_perm(bh[2], bh[3], 0x0040), 0x5410),
          __byte_perm(__byte_perm(bh[4], bh[5], 0x0040), __byte_perm(bh[6], bh[7], 0x0040), 0x5410));
      const uint2 pl = make_uint2(
          __byte_perm(__byte_perm(bl[0], bl[1], 0x0040), __byte_perm(bl[2], bl[3], 0x0040), 0x5410),
          __byte_perm(__byte_perm(bl[4], bl[5], 0x0040), __byte_perm(bl[6], bl[7], 0x0040), 0x5410));
      // sub-block c sits in set s = (c/2)%2 at k-slot group t = 2*(c/4) + c%2;
      // its columns are n = 2t (h) and 2t+1 (l)
      const int c = lane >> 2, k = 8 * (lane & 3);
      const int st = (c >> 1) & 1, t = 2 * (c >> 2) + (c & 1);
      uint8_t *p = frag + bg * kFrag + st * 256 + (k >> 4) * 128 + t * 32 + (k & 15);
      *reinterpret_cast<uint2 *>(p) = ph;
      *reinterpret_cast<uint2 *>(p + 16) = pl;
      if ((lane & 3) == 0) {
        // odd sub-blocks are high nibbles, multiplied by 16 in the MMA
        scl[bg * 16 + t * 4 + st] = sigma * ((c & 1) ? (1.0f / (254.0f * 16.0f)) : (1.0f / 254.0f));
        scl[bg * 16 + t * 4 + 2 + st] = sum;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, o);
  if (!told) {
    __syncwarp();
    if (lane == 0) mbar_arrive(xgo);
  }
  return __all_sync(0xFFFFFFFFu, fin);
}

// B fragments of one block: [set][round pair]
__device__ __forceinline__ void bfrag(const uint8_t *xb, uint4 (&B)[2][2]) {
#pragma unroll
  for (int st = 0; st < 2; st++)
#pragma unroll
    for (int rp = 0; rp < 2; rp++) B[st][rp] = *reinterpret_cast<const uint4 *>(xb + st * 256 + rp * 128);
}

// the 8 MMAs of one block for rows g, g+8 of a 16-row slice at r0:
// D[s] = {row g h-digit, row g l-digit, row g+8 h, row g+8 l} of sub-block
// c(s, t)
__device__ __forceinline__ void mma16(const uint8_t *r0, const uint4 (&B)[2][2], const Lane &Q, int (&D)[2][4]) {
  const uint8_t *r1 = r0 + 8 * kPitch;
#pragma unroll
  for (int st = 0; st < 2; st++) {
    D[st][0] = D[st][1] = D[st][2] = D[st][3] = 0;
#pragma unroll
    for (int rp = 0; rp < 2; rp++) {
      const uint4 A0 = *reinterpret_cast<const uint4 *>(r0 + Q.woff + 32 * st + 16 * rp);
      const uint4 A1 = *reinterpret_cast<const uint4 *>(r1 + Q.woff + 32 * st + 16 * rp);
      imma_u8(D[st], A0.x & Q.mq, A1.x & Q.mq, A0.y & Q.mq, A1.y & Q.mq, B[st][rp].x, B[st][rp].y);
      imma_u8(D[st], A0.z & Q.mq, A1.z & Q.mq, A0.w & Q.mq, A1.w & Q.mq, B[st][rp].z, B[st][rp].w);
    }
  }
}

// The A (weight code) operands of mma16, loaded and masked once (several
// rows of x use them): [set][round pair][word], for rows g (0) and g+8 (1).
struct AFrag {
  uint32_t a[2][2][2][4];
};
__device__ __forceinline__ void load_afrag(const uint8_t *r0, const Lane &Q, AFrag &F) {
  const uint8_t *r1 = r0 + 8 * kPitch;
#pragma unroll
  for (int st = 0; st < 2; st++)
#pragma unroll
    for (int rp = 0; rp < 2; rp++) {
      const uint4 A0 = *reinterpret_cast<const uint4 *>(r0 + Q.woff + 32 * st + 16 * rp);
      const uint4 A1 = *reinterpret_cast<const uint4 *>(r1 + Q.woff + 32 * st + 16 * rp);
      F.a[st][rp][0][0] = A0.x & Q.mq, F.a[st][rp][0][1] = A0.y & Q.mq;
      F.a[st][rp][0][2] = A0.z & Q.mq, F.a[st][rp][0][3] = A0.w & Q.mq;
      F.a[st][rp][1][0] = A1.x & Q.mq, F.a[st][rp][1][1] = A1.y & Q.mq;
      F.a[st][rp][1][2] = A1.z & Q.mq, F.a[st][rp][1][3] = A1.w & Q.mq;
    }
}
// mma16 with preloaded A operands (the same MMAs, the same order)
__device__ __forceinline__ void mma16p(const AFrag &F, const uint4 (&B)[2][2], int (&D)[2][4]) {
#pragma unroll
  for (int st = 0; st < 2; st++) {
    D[st][0] = D[st][1] = D[st][2] = D[st][3] = 0;
#pragma unroll
    for (int rp = 0; rp < 2; rp++) {
      const uint32_t(&a0)[4] = F.a[st][rp][0];
      const uint32_t(&a1)[4] = F.a[st][rp][1];
      imma_u8(D[st], a0[0], a1[0], a0[1], a1[1], B[st][rp].x, B[st][rp].y);
      imma_u8(D[st], a0[2], a1[2], a0[3], a1[3], B[st][rp].z, B[st][rp].w);
    }
  }
}

// scales of sub-blocks c(0, t) and c(0, t) + 2 of rows g, g+8 (headers h0,
// h1: d, dmin, the 12 scale bytes; get_scale_min_k4, two at a time in
// 16-bit lanes), applied to the digit sums:
// acc_r += d*sum_s sc_s*sigma'_s*v_s - dmin*sum_s m_s*S_s
__device__ __forceinline__ void epi16(const uint4 (&hd)[2], const float4 sg, const Lane &Q, const int (&D)[2][4],
                                      float &acc0, float &acc1) {
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const uint4 h = hd[r];
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    const float dm = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint32_t ys = h.y >> Q.sh, zs = h.z >> Q.sh, ws = h.w >> Q.sh;
    const uint32_t sc2 = ((Q.lo ? ys : ws) & Q.mlo) | ((ys >> 2) & Q.mhi);
    const uint32_t m2 = ((Q.lo ? zs : (ws >> 4)) & Q.mlo) | ((zs >> 2) & Q.mhi);
    const float v0 = (float)(D[0][2 * r] * 254 + D[0][2 * r + 1]);  // |.| < 2^28
    const float v1 = (float)(D[1][2 * r] * 254 + D[1][2 * r + 1]);
    const float q = fmaf(lane16_f(sc2, 0x7632u) * sg.y, v1, (lane16_f(sc2, 0x7610u) * sg.x) * v0);
    const float mn = fmaf(lane16_f(m2, 0x7632u), sg.w, lane16_f(m2, 0x7610u) * sg.z);
    float &acc = r ? acc1 : acc0;
    acc = fmaf(-dm, mn, fmaf(d, q, acc));
  }
}

// epi16 split for several rows of x: the block scales decoded once
// (d, dmin, sc and m of the lane's two sub-blocks, rows g and g+8), then
// applied per row with epi16's operations in epi16's order.
struct Scl16 {
  float d[2], dm[2], s0[2], s1[2], n0[2], n1[2];
};
__device__ __forceinline__ void decode16(const uint4 (&hd)[2], const Lane &Q, Scl16 &S) {
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const uint4 h = hd[r];
    S.d[r] = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    S.dm[r] = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint32_t ys = h.y >> Q.sh, zs = h.z >> Q.sh, ws = h.w >> Q.sh;
    const uint32_t sc2 = ((Q.lo ? ys : ws) & Q.mlo) | ((ys >> 2) & Q.mhi);
    const uint32_t m2 = ((Q.lo ? zs : (ws >> 4)) & Q.mlo) | ((zs >> 2) & Q.mhi);
    S.s0[r] = lane16_f(sc2, 0x7610u);
    S.s1[r] = lane16_f(sc2, 0x7632u);
    S.n0[r] = lane16_f(m2, 0x7610u);
    S.n1[r] = lane16_f(m2, 0x7632u);
  }
}
__device__ __forceinline__ void apply16(const Scl16 &S, const float4 sg, const int (&D)[2][4], float &acc0,
                                        float &acc1) {
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const float v0 = (float)(D[0][2 * r] * 254 + D[0][2 * r + 1]);
    const float v1 = (float)(D[1][2 * r] * 254 + D[1][2 * r + 1]);
    const float q = fmaf(S.s1[r] * sg.y, v1, (S.s0[r] * sg.x) * v0);
    const float mn = fmaf(S.n1[r], sg.w, S.n0[r] * sg.z);
    float &acc = r ? acc1 : acc0;
    acc = fmaf(-S.dm[r], mn, fmaf(S.d[r], q, acc));
  }
}

// A warp's tile partials (rows g, g+8 of each 16-row slice, each summed over
// the four lanes of its group) into slot ti % kSlots for the epilogue warp.
// Partials of activation row m of slot s: part + ((s * MR + m) * kC + warp) * kRows.
template <int MR>
__device__ __forceinline__ bool tile_partial(int ti, float (&acc)[MR][2 * kHalves], int M, float *part,
                                             uint64_t *tdone, uint64_t *tfree, int warp, int lane, int *err) {
#pragma unroll
  for (int m = 0; m < MR; m++)
#pragma unroll
    for (int i = 0; i < 2 * kHalves; i++) {
      acc[m][i] += __shfl_xor_sync(0xFFFFFFFFu, acc[m][i], 1);
      acc[m][i] += __shfl_xor_sync(0xFFFFFFFFu, acc[m][i], 2);
    }
  const int slot = ti % kSlots;
  bool ok = true;
  if (lane == 0) ok = spin_bar(&tfree[slot], (uint32_t)(((ti / kSlots) & 1) ^ 1), err);
  if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return false;
  if ((lane & 3) == 0) {
#pragma unroll
    for (int m = 0; m < MR; m++) {
      if (m >= M) break;
      float *pt = part + ((slot * MR + m) * kC + warp) * kRows + (lane >> 2);
#pragma unroll
      for (int i = 0; i < 2 * kHalves; i++) pt[8 * i] = acc[m][i];
    }
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&tdone[slot]);
#pragma unroll
  for (int m = 0; m < MR; m++)
#pragma unroll
    for (int i = 0; i < 2 * kHalves; i++) acc[m][i] = 0.f;
  return true;
}

// MR: the most activation rows a launch takes (a.M <= MR); one CTA per SM
// when MR > 1 (more registers for the row accumulators).
template <int MR>
__global__ void __launch_bounds__(32 * kWarps, MR == 1 ? 2 : 1) k_mvq4k(const __grid_constant__ CUtensorMap tmap,
                                                                       const Params a) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + kBarOff);  // [S]     copy engine -> compute
  uint64_t *empty = full + 8;                                  // [S]     compute -> producer
  uint64_t *tdone = full + 16;                                 // [slots] tile partials ready
  uint64_t *tfree = full + 24;                                 // [slots] tile partials summed
  uint64_t *xgo = full + 20;                                   // compute warps -> producer: x loads issued
  int *flag = reinterpret_cast<int *>(sm + kFlagOff);
  float *part = reinterpret_cast<float *>(sm + kPartOff);      // [slots][MR][kC][kRows]
  uint8_t *xr = sm + kPartOff + MR * kPartBytes;               // [MR] x regions, a.xstride apart
  uint8_t *stages = sm + a.soff;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int M = MR == 1 ? 1 : a.M;  // rows of x (a compile-time 1 for the batch-1 kernel)
  const int my_tiles = (a.tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int nstages = my_tiles * a.nch;

  if (threadIdx.x == 0) {
    *flag = 0;
    for (int s = 0; s < a.S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kC);
    }
    for (int s = 0; s < kSlots; s++) {
      mbar_init(&tdone[s], kC);
      mbar_init(&tfree[s], 1);
    }
    mbar_init(xgo, kC);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == kProd) {
    // weights are only read, never written, by these kernels: stream them
    // before the previous kernel of the stream has finished
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
      // box it: tile blockIdx.x + (it / nch) * grid, chunk it % nch.  (An L2
      // prefetch of the boxes beyond the stages measured slower: 6-19 % on
      // 25-66 MB products.)
      auto bx = [&](int it) { return (it % a.nch) * kBlk * 18; };
      auto by = [&](int it) { return ((int)blockIdx.x + (it / a.nch) * (int)gridDim.x) * kRows; };
      for (int it = 0; it < nstages; it++) {
        const int buf = it % a.S;
        // one box goes out before the previous kernel has finished; the rest
        // queue behind this CTA's x loads (issued right after the dependency
        // wait), so x does not wait for the whole weight stream
        if (it == 1 && !spin_bar_ns(xgo, 0u, a.err, 32)) return;
        if (it >= a.S && !spin_bar_ns(&empty[buf], (uint32_t)(((it / a.S) & 1) ^ 1), a.err, 64)) return;
        mbar_expect_tx(&full[buf], (uint32_t)kBoxBytes);
        if (a.swiF) {
          // 16 gate rows and the 16 matching up rows (a 16-row box each)
          const int t = (int)blockIdx.x + (it / a.nch) * (int)gridDim.x;
          tma_load_2d(stages + buf * kBoxBytes, &tmap, bx(it), 16 * t, &full[buf]);
          tma_load_2d(stages + buf * kBoxBytes + 16 * kPitch, &tmap, bx(it), a.swiF + 16 * t, &full[buf]);
        } else {
          tma_load_2d(stages + buf * kBoxBytes, &tmap, bx(it), by(it), &full[buf]);
        }
        if (it == (nstages < a.S ? nstages : a.S) - 1) prefetch_slice_l2(a.pf, a.pf_bytes);
      }
    }
    return;
  }

  // compute and epilogue warps: x (and c) may be written by the previous
  // kernel of the stream
  pdl_wait();
  if (warp < kC) {
    const size_t xel = a.xdt == TCB_F32 ? 4 : 2;
    for (int m = 0; m < M; m++) {
      uint8_t *xm = xr + (size_t)m * a.xstride;
      if (warp == 0) reinterpret_cast<uint4 *>(xm + a.nb * (kFrag + kScl))[lane] = make_uint4(0u, 0u, 0u, 0u);
      float ss;
      const void *xrow = static_cast<const char *>(a.x) + (size_t)m * a.ldx * xel;
      if (!prep_warp(a, xrow, xm, (warp + (int)blockIdx.x) & (kBlk - 1), lane, ss, m == 0 ? xgo : nullptr) &&
          lane == 0)
        *flag = 1;
      if (m == 0 && lane == 0) reinterpret_cast<float *>(sm + kNormOff)[warp] = ss;
    }
  }
  asm volatile("bar.sync 1, %0;" ::"n"(32 * (kC + 1)) : "memory");
  const bool slow = *flag != 0;

  if (!slow && warp == kEpi) {
    // sum the eight partials of each row in block order (block j of a
    // stage is owned by warp (j - blockIdx) mod 8)
    const int rot = (int)blockIdx.x & (kBlk - 1);
    float rms = 1.f;
    if (a.nw) {
      // the warps' sums of squares in warp order: sqrt(mean(x^2) + eps)
      const float *nss = reinterpret_cast<const float *>(sm + kNormOff);
      float tot = 0.f;
      for (int w2 = 0; w2 < kC; w2++) tot += nss[w2];
      rms = sqrtf(__fdiv_rn(tot, (float)a.K) + a.eps);
    }
    for (int ti = 0; ti < my_tiles; ti++) {
      const int row = ((int)blockIdx.x + ti * (int)gridDim.x) * kRows + lane;
      const bool mine = lane < kRows && row < a.N;
      float cold[MR], v[MR];
#pragma unroll
      for (int m = 0; m < MR; m++)
        cold[m] = (a.accumulate && mine && m < M) ? load_out(a.c, (long)m * a.ldc + row, a.cdt) : 0.f;
      const int slot = ti % kSlots;
      if (!spin_bar_ns(&tdone[slot], (uint32_t)((ti / kSlots) & 1), a.err, 128)) return;
#pragma unroll
      for (int m = 0; m < MR; m++) {
        v[m] = 0.f;
        if (m >= M) continue;
        const float *pt = part + (slot * MR + m) * kC * kRows + (lane < kRows ? lane : 0);
#pragma unroll
        for (int j = 0; j < kC; j++) v[m] += pt[((j - rot) & (kBlk - 1)) * kRows];
        if (a.nw) v[m] = __fdiv_rn(v[m], rms);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree[slot]);
      if (a.swiF) {
        // lanes 0-15 hold gate rows 16t + lane, lanes 16-31 the up rows:
        // a = silu(g) * u, as the separate SwiGLU kernel computes it
        const float u = __shfl_down_sync(0xFFFFFFFFu, v[0], 16);
        const int i = 16 * ((int)blockIdx.x + ti * (int)gridDim.x) + lane;
        if (lane < 16 && i < a.swiF) a.swi[i] = __fmul_rn(__fmul_rn(v[0], __frcp_rn(__fadd_rn(1.0f, expf(-v[0])))), u);
        continue;
      }
      if (mine) {
#pragma unroll
        for (int m = 0; m < MR; m++)
          if (m < M) store_out_old(a.c, (long)m * a.ldc + row, a.cdt, v[m], a.accumulate != 0, cold[m]);
      }
    }
    return;
  }

  if (!slow && warp < kC) {
    // warp w owns block (w + blockIdx) mod 8 of every stage (so that CTAs
    // start on different parts of x), both 16-row halves.  All the
    // bytes a block needs (MMA operands, block headers) are read first and
    // the stage is released before the scale math, so the producer can
    // refill it while the epilogue runs.
    const Lane Q = make_lane(xr, a.nb, lane);
    const int g = lane >> 2;
    const int own = (warp + (int)blockIdx.x) & (kBlk - 1);
    const int last_ch = own < a.nb ? (a.nb - 1 - own) / kBlk : -1;  // the warp's last chunk of a tile
    float acc[MR][2 * kHalves] = {};
    int it = 0;
    for (int ti = 0; ti < my_tiles; ti++) {
      for (int ch = 0; ch < a.nch; ch++, it++) {
        const int buf = it % a.S;
        bool ok = true;
        if (lane == 0) ok = wait_bar(&full[buf], (uint32_t)((it / a.S) & 1), a.err);
        if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return;
        const bool has = ch <= last_ch;
        const int bg = ch * kBlk + own;
        const uint8_t *r0 = stages + buf * kBoxBytes + g * kPitch + own * 144;
        if constexpr (MR > 1) {
          // several rows of x: the block's weight operands and scales are
          // read and decoded once, the stage released, then every row's
          // MMAs and scale math run from registers
          AFrag F[kHalves];
          Scl16 Sc[kHalves];
          if (has) {
#pragma unroll
            for (int h = 0; h < kHalves; h++) {
              load_afrag(r0 + 16 * h * kPitch, Q, F[h]);
              uint4 hd[2];
#pragma unroll
              for (int r = 0; r < 2; r++) hd[r] = *reinterpret_cast<const uint4 *>(r0 + (16 * h + 8 * r) * kPitch);
              decode16(hd, Q, Sc[h]);
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&empty[buf]);
          if (has) {
#pragma unroll
            for (int m = 0; m < MR; m++) {
              if (m >= M) break;  // uniform
              uint4 B[2][2];
              bfrag(Q.xb + m * a.xstride + bg * Q.xs, B);
              const float4 sg = *reinterpret_cast<const float4 *>(
                  reinterpret_cast<const uint8_t *>(Q.scl + bg * 16) + m * a.xstride);
#pragma unroll
              for (int h = 0; h < kHalves; h++) {
                int D[2][4];
                mma16p(F[h], B, D);
                apply16(Sc[h], sg, D, acc[m][2 * h], acc[m][2 * h + 1]);
              }
            }
          }
        } else
#pragma unroll
        for (int m = 0; m < MR; m++) {
          if (m >= M) break;  // uniform
          int D[kHalves][2][4];
          uint4 hd[kHalves][2];
          float4 sg = make_float4(0.f, 0.f, 0.f, 0.f);
          if (has) {
            uint4 B[2][2];
            bfrag(Q.xb + m * a.xstride + bg * Q.xs, B);
#pragma unroll
            for (int h = 0; h < kHalves; h++) mma16(r0 + 16 * h * kPitch, B, Q, D[h]);
#pragma unroll
            for (int h = 0; h < kHalves; h++)
#pragma unroll
              for (int r = 0; r < 2; r++)
                hd[h][r] = *reinterpret_cast<const uint4 *>(r0 + (16 * h + 8 * r) * kPitch);
            sg = *reinterpret_cast<const float4 *>(reinterpret_cast<const uint8_t *>(Q.scl + bg * 16) +
                                                    m * a.xstride);
          }
          if (m == M - 1) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[buf]);
          }
          if (has) {
#pragma unroll
            for (int h = 0; h < kHalves; h++) epi16(hd[h], sg, Q, D[h], acc[m][2 * h], acc[m][2 * h + 1]);
          }
        }
        if ((ch == last_ch || (last_ch < 0 && ch == a.nch - 1)) &&
            !tile_partial<MR>(ti, acc, M, part, tdone, tfree, warp, lane, a.err))
          return;
      }
    }
    return;
  }

  if (slow) {
    // NaN/Inf in x: release the stages, then TR's float path, one warp per
    // row over the compute and epilogue warps
    if (warp < kC) {
      for (int it = 0; it < nstages; it++) {
        const int buf = it % a.S;
        bool ok = true;
        if (lane == 0) ok = wait_bar(&full[buf], (uint32_t)((it / a.S) & 1), a.err);
        if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[buf]);
      }
    }
    const int widx = warp == kEpi ? kC : warp;  // 0..kC
    const long rowBytes = (long)a.nb * 144;
    if (a.swiF) {
      for (int ti = 0; ti < my_tiles; ti++) {
        const int i0 = 16 * ((int)blockIdx.x + ti * (int)gridDim.x);
        for (int i = i0 + widx; i < i0 + 16 && i < a.swiF; i += kC + 1) {
          float g = __int_as_float(0x7FC00000), u = g;  // rms(x) with a NaN or Inf: NaN inputs
          if (!a.nw) {
            float ag[1] = {0.0f}, au[1] = {0.0f};
            lane_row_float<TCB_Q4_K, 1>(a.w + (long)i * rowBytes, a.K, lane, XGlobal{a.x, 0, a.xdt}, ag);
            lane_row_float<TCB_Q4_K, 1>(a.w + (long)(a.swiF + i) * rowBytes, a.K, lane, XGlobal{a.x, 0, a.xdt}, au);
            g = warp_sum(ag[0]);
            u = warp_sum(au[0]);
          }
          if (lane == 0) a.swi[i] = __fmul_rn(__fmul_rn(g, __frcp_rn(__fadd_rn(1.0f, expf(-g)))), u);
        }
      }
      return;
    }
    if (a.nw) {
      // rms(x) of an x with a NaN or Inf has a NaN in every row's inputs
      for (int ti = 0; ti < my_tiles; ti++) {
        const int r0 = ((int)blockIdx.x + ti * (int)gridDim.x) * kRows;
        for (int n = r0 + widx * 32 + lane; n < r0 + kRows && n < a.N; n += (kC + 1) * 32)
          store_out(a.c, n, a.cdt, __int_as_float(0x7FC00000), a.accumulate != 0);
      }
      return;
    }
    const size_t xel = a.xdt == TCB_F32 ? 4 : 2;
    for (int ti = 0; ti < my_tiles; ti++) {
      const int r0 = ((int)blockIdx.x + ti * (int)gridDim.x) * kRows;
      for (int n = r0 + widx; n < r0 + kRows && n < a.N; n += kC + 1)
        for (int m = 0; m < M; m++) {
          float accs[1] = {0.0f};
          const void *xrow = static_cast<const char *>(a.x) + (size_t)m * a.ldx * xel;
          lane_row_float<TCB_Q4_K, 1>(a.w + (long)n * rowBytes, a.K, lane, XGlobal{xrow, 0, a.xdt}, accs);
          const float v = warp_sum(accs[0]);
          if (lane == 0) store_out(a.c, (long)m * a.ldc + n, a.cdt, v, a.accumulate != 0);
        }
    }
  }
}

}  // namespace mvk

namespace {
constexpr int kSmemTwo = 113 * 1024;  // per CTA with two CTAs on an SM
constexpr int kSmemOne = 227 * 1024;
}  // namespace

// The plan of a Q4_K float-path matvec of up to mr (1, 2, 4 or 8) rows of x
// per launch: two CTAs per SM when two stages fit in half an SM's shared
// memory (mr = 1 only), else one CTA with more stages.  Every row of x has
// its own digit region and tile partials; the plan fails (ok = false) when
// fewer than two stages fit beside them.
MvPlan q4k_plan(int N, int K, const void *w, int sms, int mr, int pair) {
  using namespace mvk;
  MvPlan pl{};
  const int nb = K / 256;
  const long rowBytes = (long)nb * 144;
  if (K % 256 || nb == 0 || rowBytes % 16 || reinterpret_cast<uintptr_t>(w) % 16) return pl;
  if (mr != 1 && mr != 2 && mr != 4 && mr != 8) return pl;
  if (pair && (mr != 1 || pair % 16 || N != 2 * pair)) return pl;
  auto enc = tensor_map_encoder();
  if (!enc) return pl;
  const int xstride = (x_bytes(nb) + 127) & ~127;
  const int base = (kPartOff + mr * kPartBytes + mr * xstride + 127) & ~127;
  int S, per_sm;
  // two CTAs per SM when the tiles outnumber the SMs; otherwise one CTA per
  // SM streams its (long) rows through the deeper pipeline one CTA affords
  if (mr == 1 && base + 2 * kBoxBytes <= kSmemTwo && (N + kRows - 1) / kRows > sms) {
    S = (kSmemTwo - base) / kBoxBytes;
    if (S > 6) S = 6;
    per_sm = 2;
  } else {
    S = (kSmemOne - base) / kBoxBytes;
    if (S > 6) S = 6;
    per_sm = 1;
  }
  if (S < 2) return pl;
  pl.tiles = pair ? pair / 16 : (N + kRows - 1) / kRows;
  pl.pair = pair;
  pl.nch = (nb + kBlk - 1) / kBlk;
  pl.cbc = kBlk;
  pl.ksplit = 1;
  pl.cpk = pl.nch;
  pl.stages = S;
  pl.pitch = kPitch;
  pl.xoff = kXOff;
  pl.soff = base;
  pl.smem = base + S * kBoxBytes;
  pl.grid = pl.tiles < per_sm * sms ? pl.tiles : per_sm * sms;
  pl.kind = 1;
  pl.rows = mr;
  pl.xstride = xstride;
  CUtensorMap tm;
  cuuint64_t gdim[2] = {(cuuint64_t)(rowBytes / 8), (cuuint64_t)N};
  cuuint64_t gstride[1] = {(cuuint64_t)rowBytes};
  cuuint32_t box[2] = {(cuuint32_t)kBox8, (cuuint32_t)(pair ? 16 : kRows)};
  cuuint32_t estr[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(w), gdim, gstride, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return pl;
  static_assert(sizeof(tm) == sizeof(pl.tmap), "CUtensorMap size");
  memcpy(pl.tmap, &tm, sizeof tm);
  pl.ok = true;
  return pl;
}

cudaError_t q4k_launch(const MvPlan &pl, int N, int K, const void *w, const void *x, int xdt, void *c, int cdt,
                       int accumulate, int *err, void *scratch, cudaStream_t s, const float *nw, float eps,
                       const void *pf, size_t pf_bytes, int M, long ldx, long ldc, float *swi) {
  (void)scratch;  // this kernel keeps no state between launches
  using namespace mvk;
  if (M < 1 || M > pl.rows || (M > 1 && nw)) return cudaErrorInvalidValue;
  if ((pl.pair != 0) != (swi != nullptr) || (swi && (accumulate || xdt != TCB_F32))) return cudaErrorInvalidValue;
  Params a{};
  a.w = static_cast<const uint8_t *>(w);
  a.N = N;
  a.K = K;
  a.nb = K / 256;
  a.x = x;
  a.xdt = xdt;
  a.c = c;
  a.cdt = cdt;
  a.accumulate = accumulate;
  a.tiles = pl.tiles;
  a.nch = pl.nch;
  a.S = pl.stages;
  a.err = err;
  a.soff = pl.soff;
  a.nw = nw;
  a.eps = eps;
  a.pf = pf;
  a.pf_bytes = pf_bytes;
  a.M = M;
  a.ldx = ldx;
  a.ldc = ldc;
  a.xstride = pl.xstride;
  a.swi = swi;
  a.swiF = pl.pair;
  CUtensorMap tm;
  memcpy(&tm, pl.tmap, sizeof tm);
  void (*kern)(const CUtensorMap, const Params) = pl.rows == 8   ? k_mvq4k<8>
                                                  : pl.rows == 4 ? k_mvq4k<4>
                                                  : pl.rows == 2 ? k_mvq4k<2>
                                                                 : k_mvq4k<1>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(32 * mvk::kWarps);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, tm, a);
}

}  // namespace tcb
