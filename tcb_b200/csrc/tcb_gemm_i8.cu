// tcb_gemm_i8.cu - the int8-activation product of many rows (M >= kI8MinM)
// for Q4_K weights on the fifth-generation tensor cores, bit-exact with TR's
// quantGemmQ8 (tensor/cpu_quant_q8.go:186-259; block term dotQ4KQ8Go,
// :91-116):
//
//   per activation row m (quantised per 256 elements: codes q8, scale d8,
//   sums of 16 codes bs) and weight row n, over superblocks b in order:
//     isum = sum_j sc_j * sum_{i in sub-block j} q4_i q8_i
//     msum = sum_j m_j * (sum of the 32 codes of sub-block j)
//     acc  = fp32(acc + fp32(fp32(fp32(d isum) - fp32(dmin msum)) * d8))
//
// The integer sums are exact on the tensor cores.  With w'_i = sc_j q4_i
// (at most 63 * 15 = 945) written as 64 a_i + b_i (a_i <= 14, b_i <= 63),
//   isum = 64 sum a_i q8_i + sum b_i q8_i,   msum = sum m_{j(i)} q8_i,
// three dot products of int8 vectors over one superblock.  The B operand of
// one MMA therefore holds, for 64 weight rows, three 64-row matrices side by
// side -- [b digits | a digits | m expanded] -- and a superblock is 8
// tcgen05.mma.kind::i8 steps (M 128 activation rows, N 192, K 32) into one
// tensor-memory accumulator that starts at zero (no accumulation across
// superblocks).  The epilogue warps read the three sums of each (m, n) and
// fold them into f32 accumulators held in registers, superblock by
// superblock, with TR's operations in TR's order (each one rounded, no FMA).
// The products of a block are never summed across blocks in integers, so the
// result is the single-row kernel's bit for bit.
//
// One CTA per SM walks tiles of 128 activation rows x 64 weight rows:
//   warp 0      TMA: the activation codes of a superblock (two 128-byte
//               swizzled K panels of 128 rows) and the raw Q4_K blocks of the
//               tile's 64 weight rows (144 bytes each)
//   warp 1      tensor-memory allocation (two accumulators of 192 columns)
//               and the MMA issue (one thread)
//   warps 2-5   the B operand: digits and mins of each weight element into
//               the swizzled K-major layout, the rows' d and dmin for the
//               epilogue
//   warps 6-13  epilogue: tensor memory -> the fold -> C (two warps per
//               32-lane quarter of tensor memory, 32 weight rows each)
// Activation rows with a NaN or Inf (a block flag clear) are left to the
// float-path fix-up launch that follows (TR sends such rows down its float
// path, cpu_quant_q8.go:137-144).
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tcb.h"
#include "tcb_common.cuh"
#include "tcb_gemm_i8.h"
#include "tcb_mv_ptx.cuh"
#include "tcb_simt.cuh"

namespace tcb {
namespace i8 {

using mv::mbar_arrive;
using mv::mbar_expect_tx;
using mv::mbar_init;
using mv::mbar_test_wait;
using mv::sa;
using mv::tma_load_2d;

constexpr int kTM = 128;                  // activation rows per tile (MMA M)
constexpr int kTN = 64;                   // weight rows per tile
constexpr int kBN = 3 * kTN;              // MMA N: [b digits | a digits | m]
constexpr int kS = 2;                     // operand stages
constexpr int kAPanel = kTM * 128;        // one 128-byte K panel of the activation codes
constexpr int kBPanel = kBN * 128;
constexpr int kABytes = 2 * kAPanel;      // a superblock: K 0-127 and 128-255
constexpr int kBBytes = 2 * kBPanel;
constexpr int kRawBytes = kTN * 144;
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kS * kABytes;
constexpr int kOffR = kOffB + kS * kBBytes;
constexpr int kDdRing = 8;                // (d, dmin) of the tile's rows per superblock in flight
constexpr int kOffDd = kOffR + kS * kRawBytes;
constexpr int kOffBar = kOffDd + kDdRing * kTN * 8;
// fullA[S] fullR[S] emptyR[S] fullB[S] emptyAB[S] accF[2] accE[2] done ddF[ring]
constexpr int kNumBars = 5 * kS + 5 + kDdRing;
constexpr int kOffMisc = kOffBar + 8 * kNumBars;
constexpr int kSmem = kOffMisc + 64 + 1024;  // + alignment slack
constexpr int kThreads = 14 * 32;
constexpr int kWarpTma = 0, kWarpMma = 1, kWarpDq = 2, kDqWarps = 4, kWarpEp = 6, kEpWarps = 8;
constexpr uint32_t kTmemCols = 512;
// kind::i8: D s32 (2 << 4), A s8 (1 << 7), B s8 (1 << 10), K-major A and B,
// N >> 3 at bit 17, M >> 4 at bit 24
constexpr uint32_t kIdesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kTM >> 4) << 24);
static_assert(kOffB % 1024 == 0 && kABytes % 1024 == 0 && kBBytes % 1024 == 0 && kAPanel % 1024 == 0 &&
                  kBPanel % 1024 == 0,
              "swizzled panels on 1024-byte boundaries");
static_assert(kSmem <= 232448, "shared memory");

struct Args {
  CUtensorMap ta;  // activation codes [M, K] int8
  CUtensorMap tw;  // raw weights [N, nsb * 144] bytes
  const float *d8;       // [M, nsb]
  const uint8_t *rowfin; // [M]: 1 = every block of the row finite
  void *c;
  long ldc;
  int cdt, accumulate, M, N, nsb;
  int *err;
};

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart, descriptor version 1
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(kIdesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
      "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Bounded wait on a barrier phase by one thread: gives up (false) when
// another role has aborted or after 2^26 polls (over a second), recording a
// timeout and aborting the other roles.
__device__ __forceinline__ bool poll(uint64_t *bar, uint32_t ph, volatile int *ab, int *err) {
  for (uint32_t i = 0; i < (1u << 26); i++) {
    if (mbar_test_wait(bar, ph)) return true;
    if (*ab) return false;
  }
  *ab = 1;
  atomicExch(err, TCB_ERR_TIMEOUT);
  return false;
}

// the byte offset of (row R, K byte k) in a 128-byte-swizzled K-major panel
__device__ __forceinline__ uint32_t swz(int R, int k) {
  return (uint32_t)((R >> 3) * 1024 + (R & 7) * 128 + ((((k >> 4) ^ R) & 7) << 4) + (k & 15));
}

// Q4_K 6-bit scale and min of sub-block j (TR tensor/quant.go:158-163)
__device__ __forceinline__ void scale_min(const uint8_t *q, int j, uint32_t &sc, uint32_t &m) {
  if (j < 4) {
    sc = q[j] & 63u;
    m = q[j + 4] & 63u;
  } else {
    sc = (q[j + 4] & 15u) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// four codes (one per byte of u) times sc: the a and b digits of the four
// products (64 a + b), packed one per byte
__device__ __forceinline__ void digits4(uint32_t u, uint32_t sc, uint32_t &a, uint32_t &b) {
  const uint32_t e = (u & 0x00FF00FFu) * sc, o = ((u >> 8) & 0x00FF00FFu) * sc;  // 16-bit lanes, < 946
  a = ((e >> 6) & 0x003F003Fu) | (((o >> 6) & 0x003F003Fu) << 8);
  b = (e & 0x003F003Fu) | ((o & 0x003F003Fu) << 8);
}

__global__ void __launch_bounds__(kThreads, 1) k_qgemm_i8(const __grid_constant__ Args a) {
  extern __shared__ uint8_t smraw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~(uintptr_t)1023);
  uint8_t *sA = sm + kOffA, *sB = sm + kOffB, *sR = sm + kOffR;
  float2 *dd = reinterpret_cast<float2 *>(sm + kOffDd);  // [kDdRing][kTN]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + kOffBar);
  uint64_t *fullA = bars, *fullR = bars + kS, *emptyR = bars + 2 * kS, *fullB = bars + 3 * kS,
           *emptyAB = bars + 4 * kS, *accF = bars + 5 * kS, *accE = accF + 2, *done = accE + 2, *ddF = done + 1;
  uint32_t *slot = reinterpret_cast<uint32_t *>(sm + kOffMisc);
  volatile int *ab = reinterpret_cast<volatile int *>(sm + kOffMisc + 8);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_m = (a.M + kTM - 1) / kTM, tiles_n = (a.N + kTN - 1) / kTN, tiles = tiles_m * tiles_n;

  if (threadIdx.x == 0) {
    *ab = 0;
    for (int s = 0; s < kS; s++) {
      mbar_init(fullA + s, 1);
      mbar_init(fullR + s, 1);
      mbar_init(emptyR + s, kDqWarps);
      mbar_init(fullB + s, kDqWarps);
      mbar_init(emptyAB + s, 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(accF + b, 1);
      mbar_init(accE + b, kEpWarps);
    }
    mbar_init(done, 1);
    for (int r = 0; r < kDdRing; r++) mbar_init(ddF + r, kDqWarps);
    mv::fence_barrier_init();
  }
  if (warp == kWarpMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(sa(slot)), "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *slot;
  mv::pdl_wait();

  if (warp == kWarpTma) {
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.ta)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.tw)) : "memory");
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int tm = t % tiles_m, tn = t / tiles_m;
        for (int sb = 0; sb < a.nsb; sb++, g++) {
          const int s = g % kS;
          const uint32_t ph = ((g / kS) & 1) ^ 1;
          if (g >= kS && !(ok = poll(emptyAB + s, ph, ab, a.err))) break;
          mbar_expect_tx(fullA + s, (uint32_t)kABytes);
          tma_load_2d(sA + s * kABytes, &a.ta, sb * 256, tm * kTM, fullA + s);
          tma_load_2d(sA + s * kABytes + kAPanel, &a.ta, sb * 256 + 128, tm * kTM, fullA + s);
          if (g >= kS && !(ok = poll(emptyR + s, ph, ab, a.err))) {
            // this stage's activation copy is out: drain it below as well
            for (uint32_t i = 0; i < (1u << 26) && !mbar_test_wait(fullA + s, (g / kS) & 1); i++) {
            }
            break;
          }
          mbar_expect_tx(fullR + s, (uint32_t)kRawBytes);
          tma_load_2d(sR + s * kRawBytes, &a.tw, sb * 144, tn * kTN, fullR + s);
        }
      }
      // copies still in flight land before the CTA exits (already complete
      // unless another role aborted)
      for (int j = g - kS > 0 ? g - kS : 0; j < g; j++)
        for (uint32_t i = 0; i < (1u << 26); i++)
          if (mbar_test_wait(fullA + j % kS, (j / kS) & 1) && mbar_test_wait(fullR + j % kS, (j / kS) & 1)) break;
    }
  } else if (warp == kWarpMma) {
    if (lane == 0) {
      const uint64_t da0 = sw128_desc(sa(sA)), db0 = sw128_desc(sa(sB));
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        for (int sb = 0; sb < a.nsb; sb++, g++) {
          const int s = g % kS, buf = g & 1;
          if (g >= 2 && !(ok = poll(accE + buf, ((g >> 1) & 1) ^ 1, ab, a.err))) break;
          if (!(ok = poll(fullA + s, (g / kS) & 1, ab, a.err)) || !(ok = poll(fullB + s, (g / kS) & 1, ab, a.err)))
            break;
          fence_after();
          const uint32_t d = tmem + (uint32_t)(buf * kBN);
#pragma unroll
          for (int p = 0; p < 2; p++) {
            // descriptor addresses in 16-byte units: stage, panel, 32-byte K steps
            const uint64_t da = da0 + (uint64_t)((s * kABytes + p * kAPanel) >> 4);
            const uint64_t db = db0 + (uint64_t)((s * kBBytes + p * kBPanel) >> 4);
#pragma unroll
            for (int kk = 0; kk < 4; kk++) mma_i8(d, da + 2 * kk, db + 2 * kk, (p | kk) != 0);
          }
          commit(sa(emptyAB + s));
          commit(sa(accF + buf));
        }
      }
      // every MMA issued above has finished once this arrives (waited for
      // even after an abort: tensor memory is freed below)
      commit(sa(done));
      for (uint32_t i = 0; i < (1u << 26) && !mbar_test_wait(done, 0); i++) {
      }
    }
  } else if (warp < kWarpEp) {
    // B operand: thread i of the 128 takes items (weight row r, 16-byte K
    // chunk c) i, i + 128, ... of the 64 x 16 per superblock
    const int ti = threadIdx.x - kWarpDq * 32;
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      for (int sb = 0; sb < a.nsb; sb++, g++) {
        const int s = g % kS;
        bool w = true;
        if (lane == 0) {
          w = poll(fullR + s, (g / kS) & 1, ab, a.err);
          if (w && g >= kS) w = poll(emptyAB + s, ((g / kS) & 1) ^ 1, ab, a.err);
        }
        if (!(ok = __shfl_sync(0xFFFFFFFFu, w, 0))) break;
        const uint8_t *raw = sR + s * kRawBytes;
        uint8_t *B = sB + s * kBBytes;
        for (int it = ti; it < kTN * 16; it += kDqWarps * 32) {
          const int r = it >> 4, c = it & 15;
          const uint8_t *row = raw + r * 144;
          const int j = c >> 1;  // sub-block
          uint32_t sc, m;
          scale_min(row + 4, j, sc, m);
          // 16 codes: low nibbles of q[32 g + 16 (c % 2) ..] for c % 4 < 2, else high nibbles
          const uint4 q = *reinterpret_cast<const uint4 *>(row + 16 + 32 * (c >> 2) + 16 * (c & 1));
          const int sh = ((c >> 1) & 1) * 4;
          const uint32_t u[4] = {(q.x >> sh) & 0x0F0F0F0Fu, (q.y >> sh) & 0x0F0F0F0Fu, (q.z >> sh) & 0x0F0F0F0Fu,
                                 (q.w >> sh) & 0x0F0F0F0Fu};
          uint4 da4, db4;
          digits4(u[0], sc, da4.x, db4.x);
          digits4(u[1], sc, da4.y, db4.y);
          digits4(u[2], sc, da4.z, db4.z);
          digits4(u[3], sc, da4.w, db4.w);
          const uint32_t mm = m * 0x01010101u;
          const int p = c >> 3, kb = (c & 7) * 16;  // panel, K byte in the panel
          uint8_t *P = B + p * kBPanel;
          *reinterpret_cast<uint4 *>(P + swz(r, kb)) = db4;
          *reinterpret_cast<uint4 *>(P + swz(kTN + r, kb)) = da4;
          *reinterpret_cast<uint4 *>(P + swz(2 * kTN + r, kb)) = make_uint4(mm, mm, mm, mm);
          if (c == 0) {
            const uint32_t hd = *reinterpret_cast<const uint32_t *>(row);
            dd[(g % kDdRing) * kTN + r] = make_float2(half_exact((uint16_t)(hd & 0xFFFFu)),
                                                      half_exact((uint16_t)(hd >> 16)));
          }
        }
        // generic-proxy stores, read by the tensor core's async proxy
        mv::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(fullB + s);
          mbar_arrive(emptyR + s);
          mbar_arrive(ddF + g % kDdRing);  // the (d, dmin) entries for the epilogue
        }
      }
    }
  } else {
    // epilogue: TMEM lanes 32 (warp % 4) .. are this warp's activation rows,
    // weight rows 32 h .. 32 h + 31 of the tile its columns
    const int q = warp & 3, h = (warp - kWarpEp) >> 2, rl = 32 * q + lane;
    int g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
      const int tm = t % tiles_m, tn = t / tiles_m;
      const int mrow = tm * kTM + rl;
      const bool live = mrow < a.M && a.rowfin[mrow < a.M ? mrow : 0];
      const float *d8row = a.d8 + (size_t)(mrow < a.M ? mrow : 0) * a.nsb;
      float acc[32];
#pragma unroll
      for (int i = 0; i < 32; i++) acc[i] = 0.f;
      float d8n = d8row[0];
      for (int sb = 0; sb < a.nsb; sb++, g++) {
        const int buf = g & 1;
        const float d8 = d8n;
        if (sb + 1 < a.nsb) d8n = d8row[sb + 1];
        bool w = true;
        if (lane == 0) {
          w = poll(accF + buf, (g >> 1) & 1, ab, a.err);
          if (w) w = poll(ddF + g % kDdRing, (g / kDdRing) & 1, ab, a.err);
        }
        if (!(ok = __shfl_sync(0xFFFFFFFFu, w, 0))) break;
        fence_after();
        const float2 *ddr = dd + (g % kDdRing) * kTN;
#pragma unroll
        for (int part = 0; part < 2; part++) {
          uint32_t vb[16], va[16], vm[16];
          const uint32_t base = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * kBN + 32 * h + 16 * part);
          tmem_ld16(base, vb);
          tmem_ld16(base + kTN, va);
          tmem_ld16(base + 2 * kTN, vm);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; i++) {
            const float2 dm = ddr[32 * h + 16 * part + i];
            const int isum = 64 * (int)va[i] + (int)vb[i];
            const float u = __fmul_rn(dm.x, __int2float_rn(isum));
            const float v = __fmul_rn(dm.y, __int2float_rn((int)vm[i]));
            acc[16 * part + i] = __fadd_rn(acc[16 * part + i], __fmul_rn(__fsub_rn(u, v), d8));
          }
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(accE + buf);
      }
      if (ok && live) {
        const int n0 = tn * kTN + 32 * h;
#pragma unroll
        for (int i = 0; i < 32; i++)
          if (n0 + i < a.N) store_out(a.c, (long)mrow * a.ldc + n0 + i, a.cdt, acc[i], a.accumulate != 0);
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == kWarpMma) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// rowfin[m] = every block flag of row m set; *nbad counts the rows that are not
__global__ void k_rowfin(const uint8_t *flags, int M, int nbk, uint8_t *rowfin, int *nbad) {
  for (int m = blockIdx.x * blockDim.x + threadIdx.x; m < M; m += gridDim.x * blockDim.x) {
    bool f = true;
    for (int b = 0; b < nbk; b++) f = f && flags[(size_t)m * nbk + b];
    rowfin[m] = f ? 1 : 0;
    if (!f) atomicAdd(nbad, 1);
  }
}

// The rows k_qgemm_i8 leaves: TR's float path (quantGemm's row, the float
// quantDot of every weight row), one warp per weight row.  Nothing to do
// (one load per CTA) when every row is finite.
__global__ void __launch_bounds__(256) k_fix_rows(const uint8_t *w, int M, int N, int K, const uint8_t *rowfin,
                                                  const int *nbad, const void *x, int xdt, long ldx, void *c, int cdt,
                                                  long ldc, int accumulate) {
  if (*nbad == 0) return;
  const int lane = threadIdx.x & 31;
  const long rowBytes = (long)K / 256 * 144;
  for (int n = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; n < N; n += (gridDim.x * blockDim.x) >> 5) {
    for (int m0 = 0; m0 < M; m0 += 32) {
      unsigned bad = __ballot_sync(0xFFFFFFFFu, m0 + lane < M && !rowfin[m0 + lane]);
      while (bad) {
        const int m = m0 + __ffs(bad) - 1;
        bad &= bad - 1;
        float accs[1] = {0.0f};
        const char *xm = static_cast<const char *>(x) + (long)m * ldx * (xdt == TCB_F32 ? 4 : 2);
        lane_row_float<TCB_Q4_K, 1>(w + (long)n * rowBytes, K, lane, XGlobal{xm, 0, xdt}, accs);
        const float v = warp_sum(accs[0]);
        if (lane == 0) store_out(c, (long)m * ldc + n, cdt, v, accumulate != 0);
      }
    }
  }
}

}  // namespace i8

bool i8_eligible(int wtype, int M, int N, int K, const void *w) {
  return wtype == TCB_Q4_K && M >= kI8MinM && N > 0 && K >= 256 && K % 256 == 0 &&
         (reinterpret_cast<uintptr_t>(w) & 15) == 0 && tensor_map_encoder() != nullptr;
}

size_t i8_extra_bytes(int M) { return (((size_t)M + 255) & ~(size_t)255) + 256; }

cudaError_t launch_qgemm_i8(const void *w, int M, int N, int K, const Act8Scratch &sc, void *extra, const void *x,
                            int xdt, long ldx, void *c, int cdt, long ldc, int accumulate, int *err, int sms,
                            cudaStream_t s) {
  using namespace i8;
  const int nsb = K / 256;
  uint8_t *rowfin = static_cast<uint8_t *>(extra);
  int *nbad = reinterpret_cast<int *>(static_cast<uint8_t *>(extra) + (((size_t)M + 255) & ~(size_t)255));
  cudaError_t e = cudaMemsetAsync(nbad, 0, sizeof(int), s);
  if (e != cudaSuccess) return e;
  k_rowfin<<<(M + 255) / 256, 256, 0, s>>>(sc.flags, M, nsb, rowfin, nbad);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  Args a{};
  auto enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  {
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
    cuuint64_t strides[1] = {(cuuint64_t)K};
    cuuint32_t box[2] = {128, (cuuint32_t)kTM}, es[2] = {1, 1};
    if (enc(&a.ta, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, sc.q8, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  {
    const size_t rb = (size_t)nsb * 144;
    cuuint64_t dims[2] = {(cuuint64_t)rb, (cuuint64_t)N};
    cuuint64_t strides[1] = {(cuuint64_t)rb};
    cuuint32_t box[2] = {144, (cuuint32_t)kTN}, es[2] = {1, 1};
    if (enc(&a.tw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(w), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
  }
  a.d8 = sc.d8;
  a.rowfin = rowfin;
  a.c = c;
  a.ldc = ldc;
  a.cdt = cdt;
  a.accumulate = accumulate;
  a.M = M;
  a.N = N;
  a.nsb = nsb;
  a.err = err;
  if ((e = cudaFuncSetAttribute(k_qgemm_i8, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem)) != cudaSuccess)
    return e;
  const int tiles = ((M + kTM - 1) / kTM) * ((N + kTN - 1) / kTN);
  const int grid = tiles < sms ? tiles : sms;
  k_qgemm_i8<<<grid, kThreads, kSmem, s>>>(a);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  k_fix_rows<<<sms * 4, 256, 0, s>>>(static_cast<const uint8_t *>(w), M, N, K, rowfin, nbad, x, xdt, ldx, c, cdt, ldc,
                                      accumulate);
  return cudaGetLastError();
}

}  // namespace tcb
