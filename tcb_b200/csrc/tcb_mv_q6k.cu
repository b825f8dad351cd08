// tcb_mv_q6k.cu - batch-1 Q6_K matvec, float path (x in f32/bf16/f16):
//
//   y[n] (+)= sum_k x[k] * dequant(W)[n, k]     W: [N, K] Q6_K blocks
//
// Same structure as the Q4_K kernel (tcb_mv_q4k.cu): small CTAs (two per
// SM, programmatic dependent launch), a producer warp streaming 2-D TMA
// boxes (stages in shared memory, later boxes prefetched into L2), 8 compute
// warps each owning one block of every stage, an epilogue warp adding the 8
// warp partials of a row in block order.  What differs:
//
//  * A Q6_K block is 210 bytes: ql[128] (low 4 bits), qh[64] (high 2
//    bits), int8 sc[16] (one per 16 elements), fp16 d; element
//    128n + 32k4 + l (n = 0, 1; k4 = 0..3; l = 0..31) has the code
//    (ql[64n + l + 32(k4%2)] >> 4(k4/2) & 15) | (qh[32n + l] >> 2k4 & 3) << 4
//    and the value d * sc[8n + 2k4 + l/16] * (code - 32) (TR
//    tensor/quant.go:196-221).  Eight blocks make a 1680-byte staged row,
//    16 mod 128: no padding is needed for conflict-free 8-row reads.  The
//    tile is 16 rows, so two stages fit next to the x region in half an SM.
//  * The k-slot mapping of the Q4_K kernel (sub-block c(s, t) =
//    4(t/2) + t%2 + 2s in MMA set s for lanes t = lane%4) lands on the
//    32-element groups (n, k4) = (t/2, t%2 + 2s): a lane reads the same ql
//    and qh bytes in both sets (low nibbles in set 0, high nibbles in set 1,
//    qh bits at 2(t%2) and 2(t%2) + 4).  Codes enter the MMA as u8 0..63;
//    the -32 offset is applied with the sub-block's digit sum.  Rounds 0-1
//    and 2-3 of a group are its two 16-element sub-blocks (two scales).
//  * Blocks start 2-byte aligned in a staged row (210j mod 16 = 2j mod 16):
//    a warp reads each 16-byte field of its block as two aligned 16-byte
//    loads (conflict-free over 8 rows x 2 field offsets) and funnel shifts
//    by the block's offset, which is fixed per warp.
#include <string.h>

#include "tcb_common.cuh"
#include "tcb_matvec.h"
#include "tcb_mv_ptx.cuh"
#include "tcb_simt.cuh"

namespace tcb {
namespace mv6 {

using namespace mv;

constexpr int kC = 8;                       // compute warps
constexpr int kProd = kC;                   // producer warp
constexpr int kEpi = kC + 1;                // epilogue warp
constexpr int kWarps = kC + 2;
constexpr int kRows = 16;                   // rows per tile (one box)
constexpr int kBlk = 8;                     // Q6_K blocks per box
constexpr int kBox8 = 210;                  // box width, 8-byte elements (8 blocks * 210 / 8)
constexpr int kPitch = kBox8 * 8;           // staged row pitch (1680 = 16 mod 128)
constexpr int kBoxBytes = kRows * kPitch;   // one stage
constexpr int kSlots = 4;                   // tile partial slots in flight
constexpr int kFrag = 512, kScl = 128;      // per block: B fragments, lane scales
constexpr int kBarOff = 0, kFlagOff = 256, kPartOff = 512;
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
  int soff;
  const void *pf;    // weights of the next kernel of a chain, prefetched into L2 (or nullptr)
  size_t pf_bytes;
};

// x region: [nb][kFrag] B fragments (as the Q4_K kernel), [nb][kScl] lane
// scales ([t][sigma'_s0, sigma'_s1, -32 Sd(s0, sub 0), -32 Sd(s0, sub 1),
// -32 Sd(s1, sub 0), -32 Sd(s1, sub 1), -, -] with Sd = 254 sum(h) +
// sum(l) over the 16-element sub-block), then kFrag zero bytes.
__host__ __device__ inline int x_bytes(int nb) { return nb * (kFrag + kScl) + kFrag; }

struct Lane {
  const uint8_t *xb;  // B fragments of block 0 (or the zero bytes)
  int xs;             // per-block stride of xb (0 for the zero bytes)
  int qlo, qho;       // ql and qh byte offsets of the lane's 32-element groups
  int sh;             // qh bit position of set 0 (set 1: sh + 4)
  int sco;            // offset of sc[8n + 2(t%2)] (sets/sub-blocks at +0, +1, +4, +5)
  const float *scl;   // lane scales of block 0
};

__device__ __forceinline__ Lane make_lane(const uint8_t *xr, int nb, int lane) {
  const int g = lane >> 2, t = lane & 3, n = t >> 1, odd = t & 1;
  const bool act = (g >> 1) == t;
  Lane q;
  q.xb = act ? xr + g * 16 : xr + nb * (kFrag + kScl);
  q.xs = act ? kFrag : 0;
  q.qlo = 64 * n + 32 * odd;
  q.qho = 128 + 32 * n;
  q.sh = 2 * odd;
  q.sco = 192 + 8 * n + 2 * odd;
  q.scl = reinterpret_cast<const float *>(xr + nb * kFrag) + t * 8;
  return q;
}

__device__ __forceinline__ void load8(const void *x, int e, int xdt, bool vec, float (&v)[8]) {
  if (vec && xdt == TCB_F32) {
    const float4 p = *reinterpret_cast<const float4 *>(static_cast<const float *>(x) + e);
    const float4 q = *reinterpret_cast<const float4 *>(static_cast<const float *>(x) + e + 4);
    v[0] = p.x, v[1] = p.y, v[2] = p.z, v[3] = p.w, v[4] = q.x, v[5] = q.y, v[6] = q.z, v[7] = q.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = load_act(x, e + i, xdt);
  }
}

// Digits of the blocks this warp owns (bg = own, own + 8, ...), lane L
// taking elements 8L..8L+7 of a block (as the Q4_K kernel), plus the digit
// sums of every 16-element sub-block.  Returns false if a sub-block sum of
// x is not finite.
// Blocks [b0, b0 + nbl) of x (every block: b0 = 0), stored at local block
// index bg - b0.
__device__ bool prep_warp(const Params &a, uint8_t *xr, int own, int lane, int b0, int nbl, int nbl_cap,
                          uint64_t *xgo) {
  constexpr float MAGIC = 12582912.0f;
  constexpr int NB = 4;
  uint8_t *frag = xr;
  float *scl = reinterpret_cast<float *>(xr + nbl_cap * kFrag);
  const bool vec = (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (a.K & 3) == 0;
  bool fin = true, told = false;
  for (int base = own; base < nbl; base += kC * NB) {
    float xv[NB][8];
#pragma unroll
    for (int j = 0; j < NB; j++) {
      const int lb = base + kC * j, bg = b0 + lb;
      if (lb < nbl) {
        load8(a.x, bg * 256 + 8 * lane, a.xdt, vec, xv[j]);
      }
    }
    if (!told) {
      // the first x loads are back: the producer may issue the rest of the
      // weight stream behind them
      __syncwarp();
      if (lane == 0) mbar_arrive(xgo);
      told = true;
    }
#pragma unroll
    for (int j = 0; j < NB; j++) {
      const int bg = base + kC * j;  // local block index
      if (bg >= nbl) break;  // warp-uniform
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
        const bool tiny = am < 1e-30f;
        sigma = (tiny ? am * 18446744073709551616.0f : am) * (1.0f / 127.0f);
        id = rcp_approx(sigma) * (tiny ? 18446744073709551616.0f : 1.0f);
        if (tiny) sigma *= 5.421010862427522e-20f;
      }
      uint32_t bh[8], bl[8];
      float fh = 0.f, fl = 0.f;
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const float t0 = fmaf(v[i], id, MAGIC);
        const float h = t0 - MAGIC;
        const float r = fmaf(v[i], id, -h);
        const float t1 = fmaf(r, 254.0f, MAGIC);
        bh[i] = __float_as_uint(t0);
        bl[i] = __float_as_uint(t1);
        fh += h;
        fl += t1 - MAGIC;
      }
      // digit sums of the lane's 16-element sub-block (lane pairs 2m, 2m+1)
      fh += __shfl_xor_sync(0xFFFFFFFFu, fh, 1);
      fl += __shfl_xor_sync(0xFFFFFFFFu, fl, 1);
      const uint2 ph = make_uint2(
          __byte_perm(__byte_perm(bh[0], bh[1], 0x0040), __byte_perm(bh[2], bh[3], 0x0040), 0x5410),
          __byte_perm(__byte_perm(bh[4], bh[5], 0x0040), __byte_perm(bh[6], bh[7], 0x0040), 0x5410));
      const uint2 pl = make_uint2(
          __byte_perm(__byte_perm(bl[0], bl[1], 0x0040), __byte_perm(bl[2], bl[3], 0x0040), 0x5410),
          __byte_perm(__byte_perm(bl[4], bl[5], 0x0040), __byte_perm(bl[6], bl[7], 0x0040), 0x5410));
      const int c = lane >> 2, k = 8 * (lane & 3);
      const int st = (c >> 1) & 1, t = 2 * (c >> 2) + (c & 1);
      uint8_t *p = frag + bg * kFrag + st * 256 + (k >> 4) * 128 + t * 32 + (k & 15);
      *reinterpret_cast<uint2 *>(p) = ph;
      *reinterpret_cast<uint2 *>(p + 16) = pl;
      float *sl = scl + bg * (kScl / 4) + t * 8;
      if ((lane & 3) == 0) sl[st] = sigma * (1.0f / 254.0f);
      if ((lane & 1) == 0) sl[2 + 2 * st + ((lane >> 1) & 1)] = -32.0f * fmaf(fh, 254.0f, fl);
    }
  }
  if (!told) {
    __syncwarp();
    if (lane == 0) mbar_arrive(xgo);
  }
  return __all_sync(0xFFFFFFFFu, fin);
}

__device__ __forceinline__ void bfrag(const uint8_t *xb, uint4 (&B)[2][2]) {
#pragma unroll
  for (int st = 0; st < 2; st++)
#pragma unroll
    for (int rp = 0; rp < 2; rp++) B[st][rp] = *reinterpret_cast<const uint4 *>(xb + st * 256 + rp * 128);
}

// A field of 16 bytes at shared address p with p % 16 = m (even, the same
// for every field of a warp's block): two aligned, conflict-free 16-byte
// loads and funnel shifts.  q = m / 4 words, sh = 8 (m % 4) bits.
struct Align {
  int m, q, sh;
};

__device__ __forceinline__ uint4 ld16u(const uint8_t *p, const Align &al) {
  const uint8_t *a = p - al.m;
  const uint4 x = *reinterpret_cast<const uint4 *>(a), y = *reinterpret_cast<const uint4 *>(a + 16);
  const uint32_t w0 = x.x, w1 = x.y, w2 = x.z, w3 = x.w, w4 = y.x, w5 = y.y, w6 = y.z, w7 = y.w;
  switch (al.q) {  // warp-uniform
  case 0: return make_uint4(__funnelshift_r(w0, w1, al.sh), __funnelshift_r(w1, w2, al.sh),
                            __funnelshift_r(w2, w3, al.sh), __funnelshift_r(w3, w4, al.sh));
  case 1: return make_uint4(__funnelshift_r(w1, w2, al.sh), __funnelshift_r(w2, w3, al.sh),
                            __funnelshift_r(w3, w4, al.sh), __funnelshift_r(w4, w5, al.sh));
  case 2: return make_uint4(__funnelshift_r(w2, w3, al.sh), __funnelshift_r(w3, w4, al.sh),
                            __funnelshift_r(w4, w5, al.sh), __funnelshift_r(w5, w6, al.sh));
  default: return make_uint4(__funnelshift_r(w3, w4, al.sh), __funnelshift_r(w4, w5, al.sh),
                             __funnelshift_r(w5, w6, al.sh), __funnelshift_r(w6, w7, al.sh));
  }
}

// the 8 MMAs of one block for rows g, g+8 of the slice at r0 (block start):
// D[s][rp] = {row g h, row g l, row g+8 h, row g+8 l} over sub-block rp of
// group c(s, t)
__device__ __forceinline__ void mma16(const uint8_t *r0, const Align &al, const uint4 (&B)[2][2], const Lane &Q,
                                      int (&D)[2][2][4]) {
  const uint8_t *r1 = r0 + 8 * kPitch;
#pragma unroll
  for (int rp = 0; rp < 2; rp++) {
    // bytes 16rp..16rp+15 of the lane's ql and qh fields, rows g and g+8
    const uint4 l0 = ld16u(r0 + Q.qlo + 16 * rp, al), l1 = ld16u(r1 + Q.qlo + 16 * rp, al);
    const uint4 h0 = ld16u(r0 + Q.qho + 16 * rp, al), h1 = ld16u(r1 + Q.qho + 16 * rp, al);
    D[0][rp][0] = D[0][rp][1] = D[0][rp][2] = D[0][rp][3] = 0;
    D[1][rp][0] = D[1][rp][1] = D[1][rp][2] = D[1][rp][3] = 0;
#pragma unroll
    for (int q = 0; q < 2; q++) {  // round 2rp + q: words 2q, 2q+1
      const uint32_t ql[4] = {q ? l0.z : l0.x, q ? l1.z : l1.x, q ? l0.w : l0.y, q ? l1.w : l1.y};
      const uint32_t qh[4] = {q ? h0.z : h0.x, q ? h1.z : h1.x, q ? h0.w : h0.y, q ? h1.w : h1.y};
      uint32_t a0[4], a1[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t hs = qh[i] >> Q.sh;
        a0[i] = (ql[i] & 0x0F0F0F0Fu) | ((hs << 4) & 0x30303030u);
        a1[i] = ((ql[i] >> 4) & 0x0F0F0F0Fu) | (hs & 0x30303030u);
      }
      imma_u8(D[0][rp], a0[0], a0[1], a0[2], a0[3], q ? B[0][rp].z : B[0][rp].x, q ? B[0][rp].w : B[0][rp].y);
      imma_u8(D[1][rp], a1[0], a1[1], a1[2], a1[3], q ? B[1][rp].z : B[1][rp].x, q ? B[1][rp].w : B[1][rp].y);
    }
  }
}

// headers of rows g, g+8: d and the lane's four sub-block scales
struct Hdr {
  uint32_t d;   // fp16 bits
  uint32_t s0;  // sc bytes (set 0, sub 0), (set 0, sub 1)
  uint32_t s1;  // sc bytes (set 1, sub 0), (set 1, sub 1)
};

__device__ __forceinline__ Hdr load_hdr(const uint8_t *blk, const Lane &Q) {
  Hdr h;
  h.d = lds16(blk + 208);
  h.s0 = lds16(blk + Q.sco);
  h.s1 = lds16(blk + Q.sco + 4);
  return h;
}

// acc_r += d * sum_{s, sub} sc * sigma'_s * (254 Dh + Dl - 32 Sd)
__device__ __forceinline__ void epi16(const Hdr (&hd)[2], const float *sl, const int (&D)[2][2][4], float &acc0,
                                      float &acc1) {
  const float4 sa = *reinterpret_cast<const float4 *>(sl);      // sigma'_0, sigma'_1, S(0,0), S(0,1)
  const float2 sb = *reinterpret_cast<const float2 *>(sl + 4);  // S(1,0), S(1,1)
  const float S[2][2] = {{sa.z, sa.w}, {sb.x, sb.y}};
#pragma unroll
  for (int r = 0; r < 2; r++) {
    const float d = __half2float(__ushort_as_half((unsigned short)hd[r].d));
    float q = 0.f;
#pragma unroll
    for (int s = 0; s < 2; s++) {
      const uint32_t sw = s ? hd[r].s1 : hd[r].s0;
      float qs = 0.f;
#pragma unroll
      for (int rp = 0; rp < 2; rp++) {
        const float sc = (float)(int8_t)(sw >> (8 * rp));
        const float v = (float)(D[s][rp][2 * r] * 254 + D[s][rp][2 * r + 1]) + S[s][rp];
        qs = fmaf(sc, v, qs);
      }
      q = fmaf(qs, s ? sa.y : sa.x, q);
    }
    float &acc = r ? acc1 : acc0;
    acc = fmaf(d, q, acc);
  }
}

__device__ __forceinline__ bool tile_partial(int ti, float (&acc)[2], float *part, uint64_t *tdone, uint64_t *tfree,
                                             int warp, int lane, int *err) {
#pragma unroll
  for (int i = 0; i < 2; i++) {
    acc[i] += __shfl_xor_sync(0xFFFFFFFFu, acc[i], 1);
    acc[i] += __shfl_xor_sync(0xFFFFFFFFu, acc[i], 2);
  }
  const int slot = ti % kSlots;
  bool ok = true;
  if (lane == 0) ok = spin_bar(&tfree[slot], (uint32_t)(((ti / kSlots) & 1) ^ 1), err);
  if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return false;
  float *pt = part + (slot * kC + warp) * kRows + (lane >> 2);
  if ((lane & 3) == 0) {
    pt[0] = acc[0];
    pt[8] = acc[1];
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(&tdone[slot]);
  acc[0] = acc[1] = 0.f;
  return true;
}

__global__ void __launch_bounds__(32 * kWarps, 2) k_mvq6k(const __grid_constant__ CUtensorMap tmap, const Params a) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t *full = reinterpret_cast<uint64_t *>(sm + kBarOff);
  uint64_t *empty = full + 8;
  uint64_t *tdone = full + 16;
  uint64_t *tfree = full + 24;
  uint64_t *xgo = full + 20;  // compute warps -> producer: first x loads done
  int *flag = reinterpret_cast<int *>(sm + kFlagOff);
  float *part = reinterpret_cast<float *>(sm + kPartOff);  // [slots][kC][16]
  uint8_t *xr = sm + kXOff;
  uint8_t *stages = sm + a.soff;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // tiles t0, t0 + cps, ...; every chunk of K
  const int t0 = (int)blockIdx.x, cps = (int)gridDim.x;
  const int my_tiles = t0 < a.tiles ? (a.tiles - t0 + cps - 1) / cps : 0;
  const int ch0 = 0, ch1 = a.nch, nchl = a.nch;
  const int b0 = 0, nbl = a.nb, nbl_cap = a.nch * kBlk;
  const int nstages = my_tiles * nchl;
  auto tile_of = [&](int ti) { return t0 + ti * cps; };

  if (threadIdx.x == 0) {
    *flag = 0;
    for (int st = 0; st < a.S; st++) {
      mbar_init(&full[st], 1);
      mbar_init(&empty[st], kC);
    }
    for (int st = 0; st < kSlots; st++) {
      mbar_init(&tdone[st], kC);
      mbar_init(&tfree[st], 1);
    }
    mbar_init(xgo, kC);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) pdl_launch_dependents();

  if (warp == kProd) {
    if (lane == 0 && nstages > 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap)) : "memory");
      auto bx = [&](int it) { return (ch0 + it % nchl) * kBox8; };
      auto by = [&](int it) { return tile_of(it / nchl) * kRows; };
      for (int it = 0; it < nstages; it++) {
        const int buf = it % a.S;
        // one box before the dependency wait; the rest queue behind x
        if (it == 1 && !spin_bar_ns(xgo, 0u, a.err, 32)) return;
        if (it >= a.S && !spin_bar_ns(&empty[buf], (uint32_t)(((it / a.S) & 1) ^ 1), a.err, 64)) return;
        mbar_expect_tx(&full[buf], (uint32_t)kBoxBytes);
        tma_load_2d(stages + buf * kBoxBytes, &tmap, bx(it), by(it), &full[buf]);
        if (it == (nstages < a.S ? nstages : a.S) - 1) prefetch_slice_l2(a.pf, a.pf_bytes);
      }
    }
    return;
  }

  pdl_wait();
  if (warp < kC) {
    if (warp == 0) reinterpret_cast<uint4 *>(xr + nbl_cap * (kFrag + kScl))[lane] = make_uint4(0u, 0u, 0u, 0u);
    if (!prep_warp(a, xr, (warp + (int)blockIdx.x) & (kBlk - 1), lane, b0, nbl, nbl_cap, xgo) && lane == 0) *flag = 1;
  }
  asm volatile("bar.sync 1, %0;" ::"n"(32 * (kC + 1)) : "memory");
  const bool slow = *flag != 0;

  if (warp == kEpi) {
    // the 8 partials of each row in block order
    const int rot = (int)blockIdx.x & (kBlk - 1);
    for (int ti = 0; ti < my_tiles; ti++) {
      const int tile = tile_of(ti);
      const int row = tile * kRows + lane;
      const bool mine = lane < kRows && row < a.N;
      const int slot = ti % kSlots;
      if (!spin_bar_ns(&tdone[slot], (uint32_t)((ti / kSlots) & 1), a.err, 128)) return;
      float v = 0.f;
      if (lane < kRows) {
        const float *pt = part + slot * kC * kRows + lane;
#pragma unroll
        for (int j = 0; j < kC; j++) v += pt[((j - rot) & (kBlk - 1)) * kRows];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&tfree[slot]);
      if (mine) store_out(a.c, row, a.cdt, v, a.accumulate != 0);
    }
    return;
  }

  if (warp >= kC) return;
  const Lane Q = make_lane(xr, nbl_cap, lane);
  const int own = (warp + (int)blockIdx.x) & (kBlk - 1);
  const int gl = own < a.nb ? (a.nb - 1 - own) / kBlk : -1;  // the warp's last chunk of a row
  const int last_ch = gl >= ch0 ? min(gl, ch1 - 1) : -1;     // ... within the stages
  const int hand_ch = last_ch >= 0 ? last_ch : ch1 - 1;      // where its tile partial is handed over
  if (!slow) {
    // warp w owns block (w + blockIdx) mod 8 of every stage.  All the bytes
    // a block needs are read first and the stage is released before the
    // scale math.
    const int g = lane >> 2;
    Align al;  // where the block starts within 16 bytes (rows are 16-byte aligned)
    al.m = (own * 210) & 15;
    al.q = al.m >> 2;
    al.sh = 8 * (al.m & 3);
    float acc[2] = {0.f, 0.f};
    int it = 0;
    for (int ti = 0; ti < my_tiles; ti++) {
      for (int ch = ch0; ch < ch1; ch++, it++) {
        const int buf = it % a.S;
        bool ok = true;
        if (lane == 0) ok = wait_bar(&full[buf], (uint32_t)((it / a.S) & 1), a.err);
        if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return;
        const bool has = ch <= last_ch;
        int D[2][2][4];
        Hdr hd[2];
        int lb = 0;
        if (has) {
          lb = (ch - ch0) * kBlk + own;
          const uint8_t *r0 = stages + buf * kBoxBytes + g * kPitch + own * 210;
          uint4 B[2][2];
          bfrag(Q.xb + lb * Q.xs, B);
          mma16(r0, al, B, Q, D);
          hd[0] = load_hdr(r0, Q);
          hd[1] = load_hdr(r0 + 8 * kPitch, Q);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[buf]);
        if (has) epi16(hd, Q.scl + lb * (kScl / 4), D, acc[0], acc[1]);
        if (ch == hand_ch && !tile_partial(ti, acc, part, tdone, tfree, warp, lane, a.err)) return;
      }
    }
    return;
  }
  // NaN/Inf in x: release the stages, then TR's float path over
  // the K range for rows w and w + 8 of each tile (the other rows of
  // the warp's partial column are zero), through the same hand-over
  for (int it = 0; it < nstages; it++) {
    const int buf = it % a.S;
    bool ok = true;
    if (lane == 0) ok = wait_bar(&full[buf], (uint32_t)((it / a.S) & 1), a.err);
    if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return;
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[buf]);
  }
  const long rowBytes = (long)a.nb * 210;
  const int k0 = b0 * 256, kn = nbl * 256;
  const size_t xel = a.xdt == TCB_F32 ? 4 : 2;
  for (int ti = 0; ti < my_tiles; ti++) {
    const int tile = tile_of(ti);
    float v[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; r++) {
      const int n = tile * kRows + warp + 8 * r;
      if (n >= a.N || kn == 0) continue;
      float accs[1] = {0.0f};
      lane_row_float<TCB_Q6_K, 1>(a.w + (long)n * rowBytes + (long)b0 * 210, kn, lane,
                                  XGlobal{static_cast<const char *>(a.x) + (size_t)k0 * xel, 0, a.xdt}, accs);
      v[r] = warp_sum(accs[0]);
    }
    const int slot = ti % kSlots;
    bool ok = true;
    if (lane == 0) ok = spin_bar(&tfree[slot], (uint32_t)(((ti / kSlots) & 1) ^ 1), a.err);
    if (!__shfl_sync(0xFFFFFFFFu, ok, 0)) return;
    // column of block index (warp + blockIdx) mod 8 = own; rows warp, warp + 8
    float *pt = part + (slot * kC + warp) * kRows;
    if (lane < kRows) pt[lane] = lane == warp ? v[0] : (lane == warp + 8 ? v[1] : 0.f);
    __syncwarp();
    if (lane == 0) mbar_arrive(&tdone[slot]);
  }
}

}  // namespace mv6

namespace {
constexpr int kSmemTwo6 = 113 * 1024;
constexpr int kSmemOne6 = 227 * 1024;
}  // namespace

MvPlan q6k_plan(int N, int K, const void *w, int sms) {
  using namespace mv6;
  MvPlan pl{};
  const int nb = K / 256;
  const long rowBytes = (long)nb * 210;
  if (K % 256 || nb == 0 || rowBytes % 16 || reinterpret_cast<uintptr_t>(w) % 16) return pl;
  auto enc = tensor_map_encoder();
  if (!enc) return pl;
  const int tiles = (N + kRows - 1) / kRows, nch = (nb + kBlk - 1) / kBlk;
  // wide products only (the output head): fewer tiles than half the SMs
  // would leave SMs idle, and those products go to the generic kernel
  if (2 * tiles < sms) return pl;
  const int base = (kXOff + x_bytes(nch * kBlk) + 127) & ~127;
  int S, per_sm;
  if (base + 2 * kBoxBytes <= kSmemTwo6) {
    S = (kSmemTwo6 - base) / kBoxBytes;
    if (S > 4) S = 4;
    per_sm = 2;
  } else {
    S = (kSmemOne6 - base) / kBoxBytes;
    if (S > 6) S = 6;
    per_sm = 1;
  }
  if (S < 2) return pl;
  const int slots = per_sm * sms;
  const int cps = slots < tiles ? slots : tiles;
  pl.tiles = tiles;
  pl.nch = nch;
  pl.cbc = kBlk;
  pl.ksplit = 1;
  pl.cpk = nch;
  pl.split_bytes = 0;
  pl.stages = S;
  pl.pitch = kPitch;
  pl.xoff = kXOff;
  pl.soff = base;
  pl.smem = base + S * kBoxBytes;
  pl.grid = cps;
  pl.kind = 2;
  CUtensorMap tm;
  cuuint64_t gdim[2] = {(cuuint64_t)(rowBytes / 8), (cuuint64_t)N};
  cuuint64_t gstride[1] = {(cuuint64_t)rowBytes};
  cuuint32_t box[2] = {(cuuint32_t)kBox8, (cuuint32_t)kRows};
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

cudaError_t q6k_launch(const MvPlan &pl, int N, int K, const void *w, const void *x, int xdt, void *c, int cdt,
                       int accumulate, int *err, cudaStream_t s, const void *pf, size_t pf_bytes,
                       void *scratch) {
  (void)scratch;  // this kernel keeps no state between launches
  using namespace mv6;
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
  a.pf = pf;
  a.pf_bytes = pf_bytes;
  CUtensorMap tm;
  memcpy(&tm, pl.tmap, sizeof tm);
  cudaError_t e = cudaFuncSetAttribute(k_mvq6k, cudaFuncAttributeMaxDynamicSharedMemorySize, pl.smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.grid);
  cfg.blockDim = dim3(32 * mv6::kWarps);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_mvq6k, tm, a);
}

}  // namespace tcb
