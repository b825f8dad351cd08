// tcb_attn_prefill.cu - causal grouped-query attention for a block of prompt
// rows over the fp16 K/V cache (the prompt pass of the decoder engine).
//
// Follows TR's attention for a cached chunk (lib/layers.tr 166-215): the
// rows of a chunk at positions p0 .. p0+M-1 look at every cached position up
// to their own (causality aligned to the end), softmax(q.k / sqrt(hd)) v,
// consecutive query heads sharing a KV head.  TR runs this through its
// flash-attention GPU backend; here it is a flash-attention kernel of its
// own.
//
// CTA = (64 query rows, one query head), four warps of 16 rows.  The rotated
// query rows (f32) are rounded to fp16 once into shared memory (read back
// per K step); 64-position K and V tiles stream from the cache by cp.async
// into one buffer each, K(t+1) loading while the warps form P V(t) and
// V(t+1) while they form S(t+1) (positions past the needed range are
// zero-filled).  51 KB of shared memory and at most 168 registers per
// thread let three CTAs share an SM.
// Per tile a warp forms S = Q K^T with m16n8k16 fp16 MMAs (f32
// accumulators), applies the causal mask, keeps the running row maximum and
// sum in the log2 domain (scores scaled by log2(e)/sqrt(hd)), rescales its
// output accumulators, and adds P V with P rounded to fp16 straight from the
// score registers.  The row sum adds the rounded P, so the output is an
// exact weighted mean of the V rows under the weights used.  Query blocks
// are issued longest first across all heads (grid x = head, y = block from
// the end); the mask is applied only on tiles that reach past a warp's first
// row, and the output is rescaled only when a row maximum changes.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "tcb_launch.h"

namespace tcb {
namespace pf {

constexpr int kHd = 128;         // head dimension
constexpr int kBq = 64;          // query rows per CTA
constexpr int kBk = 64;          // cached positions per tile
constexpr int kLd = kHd + 8;     // shared-memory row stride in halves (272 B: ldmatrix rows fall in distinct banks)
constexpr int kThreads = 128;
constexpr int kMinCtas = 3;      // CTAs per SM the register budget is sized for
constexpr size_t kSmem = (size_t)(kBq + 2 * kBk) * kLd * sizeof(__half);

struct Args {
  const float *q;        // rotated query rows: row r, head h at q + r*ldq + h*kHd
  long ldq;
  const __half *kc, *vc; // this layer's cache [KVH][max_ctx][kHd]
  float *out;            // row r, head h at out + r*ldo + h*kHd
  long ldo;
  int p0, M, H, KVH, max_ctx;
  float scale_log2;      // log2(e) / sqrt(kHd)
};

__device__ __forceinline__ uint32_t su32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void ldsm4(uint32_t a, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void ldsm4t(uint32_t a, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void mma(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// 16-byte copy; src_bytes 0 fills the destination with zeros
__device__ __forceinline__ void cp16(uint32_t dst, const void *src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }

__global__ void __launch_bounds__(kThreads, kMinCtas) k_attn_prefill(const __grid_constant__ Args a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __half *qs = reinterpret_cast<__half *>(smem);  // [kBq][kLd]
  __half *ks = qs + kBq * kLd;                    // [kBk][kLd]
  __half *vs = ks + kBk * kLd;                    // [kBk][kLd]
  const int nqb = (a.M + kBq - 1) / kBq;
  const int qb = nqb - 1 - (int)blockIdx.y;  // the longest query blocks of every head first
  const int h = blockIdx.x, kh = h / (a.H / a.KVH);
  const int r0 = qb * kBq, rows = min(kBq, a.M - r0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kv_end = a.p0 + r0 + rows;  // cached positions [0, kv_end) are read
  const int ntiles = (kv_end + kBk - 1) / kBk;
  const __half *kb = a.kc + (size_t)kh * a.max_ctx * kHd, *vb = a.vc + (size_t)kh * a.max_ctx * kHd;

  // one 64-position tile of K or V into its buffer (one commit group)
  auto load_tile = [&](const __half *src, __half *dst, int t) {
    const int j0 = t * kBk;
    for (int i = tid; i < kBk * (kHd / 8); i += kThreads) {
      const int r = i / (kHd / 8), c = (i % (kHd / 8)) * 8, j = j0 + r;
      const bool ok = j < kv_end;
      cp16(su32(dst + r * kLd + c), src + (size_t)(ok ? j : 0) * kHd + c, ok ? 16 : 0);
    }
    cp_commit();
  };
  load_tile(kb, ks, 0);
  load_tile(vb, vs, 0);
  for (int i = tid; i < kBq * (kHd / 4); i += kThreads) {
    const int r = i / (kHd / 4), c = (i % (kHd / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < rows) v = *reinterpret_cast<const float4 *>(a.q + (size_t)(r0 + r) * a.ldq + (size_t)h * kHd + c);
    // the score scale log2(e)/sqrt(hd) rides on q
    __half2 *d = reinterpret_cast<__half2 *>(qs + r * kLd + c);
    d[0] = __floats2half2_rn(v.x * a.scale_log2, v.y * a.scale_log2);
    d[1] = __floats2half2_rn(v.z * a.scale_log2, v.w * a.scale_log2);
  }
  float o[kHd / 8][4];
#pragma unroll
  for (int d = 0; d < kHd / 8; d++) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int g = lane >> 2, tq = lane & 3;
  const int pos0 = a.p0 + r0 + warp * 16 + g, pos1 = pos0 + 8;  // this thread's two rows
  const int wlast = a.p0 + r0 + warp * 16 + 15;                 // the warp's last position
  // the warp's Q rows in shared memory, read per K step (ldmatrix x4 address)
  const uint32_t qa = su32(qs + (warp * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * kLd + (lane >> 4) * 8);

  // K(t) and V(t) alternate in their buffers: K(t+1) streams while the warps
  // form P V(t), V(t+1) while they form S(t+1)
  for (int t = 0; t < ntiles; t++) {
    const int j0 = t * kBk;
    const bool act = j0 <= wlast;
    cp_wait<1>();  // K(t) has landed (V(t) may still be in flight)
    __syncthreads();
    float s[kBk / 8][4];
    if (act) {
#pragma unroll
      for (int n = 0; n < kBk / 8; n++) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < kHd / 16; kk++) {
        uint32_t qf[4];
        ldsm4(qa + kk * 32, qf[0], qf[1], qf[2], qf[3]);
#pragma unroll
        for (int np = 0; np < kBk / 16; np++) {
          const int row = np * 16 + ((lane >> 4) & 1) * 8 + (lane & 7), col = kk * 16 + ((lane >> 3) & 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldsm4(su32(ks + row * kLd + col), b0, b1, b2, b3);
          mma(s[2 * np], qf, b0, b1);
          mma(s[2 * np + 1], qf, b2, b3);
        }
      }
    }
    __syncthreads();  // every warp is done with K(t)
    if (t + 1 < ntiles) load_tile(kb, ks, t + 1);
    else cp_commit();  // an empty group keeps the wait counts uniform
    uint32_t pa[kBk / 16][4];
    if (act) {
      float x0 = -INFINITY, x1 = -INFINITY;
      if (j0 + kBk - 1 > wlast - 15) {  // the tile reaches past the warp's first row: causal mask
#pragma unroll
        for (int n = 0; n < kBk / 8; n++)
#pragma unroll
          for (int e = 0; e < 2; e++) {
            const int key = j0 + n * 8 + 2 * tq + e;
            if (key > pos0) s[n][e] = -INFINITY;
            if (key > pos1) s[n][2 + e] = -INFINITY;
          }
      }
#pragma unroll
      for (int n = 0; n < kBk / 8; n++) {
        x0 = fmaxf(x0, fmaxf(s[n][0], s[n][1]));
        x1 = fmaxf(x1, fmaxf(s[n][2], s[n][3]));
      }
      x0 = fmaxf(x0, __shfl_xor_sync(0xFFFFFFFFu, x0, 1));
      x0 = fmaxf(x0, __shfl_xor_sync(0xFFFFFFFFu, x0, 2));
      x1 = fmaxf(x1, __shfl_xor_sync(0xFFFFFFFFu, x1, 1));
      x1 = fmaxf(x1, __shfl_xor_sync(0xFFFFFFFFu, x1, 2));
      // tile 0 holds position 0, which every row sees: the maxima are finite
      // from the first tile on
      const float n0 = fmaxf(m0, x0), n1 = fmaxf(m1, x1);
      // rescale only when some row of the warp has a new maximum
      if (__any_sync(0xFFFFFFFFu, n0 != m0 || n1 != m1)) {
        const float c0 = exp2f(m0 - n0), c1 = exp2f(m1 - n1);
        l0 *= c0;
        l1 *= c1;
#pragma unroll
        for (int d = 0; d < kHd / 8; d++) {
          o[d][0] *= c0;
          o[d][1] *= c0;
          o[d][2] *= c1;
          o[d][3] *= c1;
        }
      }
      m0 = n0;
      m1 = n1;
#pragma unroll
      for (int n = 0; n < kBk / 8; n++) {
        const __half2 p0 = __floats2half2_rn(exp2f(s[n][0] - n0), exp2f(s[n][1] - n0));
        const __half2 p1 = __floats2half2_rn(exp2f(s[n][2] - n1), exp2f(s[n][3] - n1));
        const float2 f0 = __half22float2(p0), f1 = __half22float2(p1);
        l0 += f0.x + f0.y;
        l1 += f1.x + f1.y;
        pa[n >> 1][(n & 1) * 2] = h2u(p0);
        pa[n >> 1][(n & 1) * 2 + 1] = h2u(p1);
      }
    }
    cp_wait<1>();  // V(t) has landed (K(t+1) may still be in flight)
    __syncthreads();
    if (act) {
#pragma unroll
      for (int kq = 0; kq < kBk / 16; kq++)
#pragma unroll
        for (int dp = 0; dp < kHd / 16; dp++) {
          const int row = kq * 16 + ((lane >> 3) & 1) * 8 + (lane & 7), col = dp * 16 + ((lane >> 4) & 1) * 8;
          uint32_t b0, b1, b2, b3;
          ldsm4t(su32(vs + row * kLd + col), b0, b1, b2, b3);
          mma(o[2 * dp], pa[kq], b0, b1);
          mma(o[2 * dp + 1], pa[kq], b2, b3);
        }
    }
    __syncthreads();  // every warp is done with V(t)
    if (t + 1 < ntiles) load_tile(vb, vs, t + 1);
    else cp_commit();
  }
  cp_wait<0>();
  l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 1);
  l0 += __shfl_xor_sync(0xFFFFFFFFu, l0, 2);
  l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 1);
  l1 += __shfl_xor_sync(0xFFFFFFFFu, l1, 2);
  const int ra = warp * 16 + g, rb = ra + 8;
  float *oa = a.out + (size_t)(r0 + ra) * a.ldo + (size_t)h * kHd + 2 * tq;
  float *ob = a.out + (size_t)(r0 + rb) * a.ldo + (size_t)h * kHd + 2 * tq;
#pragma unroll
  for (int d = 0; d < kHd / 8; d++) {
    if (ra < rows)
      *reinterpret_cast<float2 *>(oa + d * 8) = make_float2(__fdiv_rn(o[d][0], l0), __fdiv_rn(o[d][1], l0));
    if (rb < rows)
      *reinterpret_cast<float2 *>(ob + d * 8) = make_float2(__fdiv_rn(o[d][2], l1), __fdiv_rn(o[d][3], l1));
  }
}

}  // namespace pf

cudaError_t launch_attn_prefill(const float *q, long ldq, const __half *kc, const __half *vc, float *out, long ldo,
                                int p0, int M, int H, int KVH, int max_ctx, cudaStream_t s) {
  if (M <= 0) return cudaSuccess;
  if (H % KVH || p0 < 0 || p0 + M > max_ctx || (ldq % 4) || (ldo % 2)) return cudaErrorInvalidValue;
  static bool attr = [] {
    return cudaFuncSetAttribute(pf::k_attn_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pf::kSmem) ==
           cudaSuccess;
  }();
  if (!attr) return cudaErrorInvalidDeviceFunction;
  pf::Args a{q, ldq, kc, vc, out, ldo, p0, M, H, KVH, max_ctx, (float)(1.4426950408889634 / sqrt((double)pf::kHd))};
  const dim3 grid(H, (M + pf::kBq - 1) / pf::kBq);
  pf::k_attn_prefill<<<grid, pf::kThreads, pf::kSmem, s>>>(a);
  return cudaGetLastError();
}

}  // namespace tcb
