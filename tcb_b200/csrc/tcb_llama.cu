// tcb_llama.cu - batch-1 decode step of a Llama-shaped model over quantized
// weights: the callers on either side of the quantized product (embedding
// lookup, RMSNorm, rotary position, grouped-query attention over an fp16 KV
// cache, SwiGLU, greedy token) around the batch-1 matvec kernels.
//
// Follows TR's GPT (lib/layers.tr): x = embed(token); per block
// h = x + attn(rms(x)); x = h + ffn(rms(h)) (348-389); logits =
// head(rms(x)) (658-666).  RMSNorm is x / sqrt(mean(x^2) + eps) * w
// (68-79); the rotary table uses theta^(-2i/hd) and rotates the two halves
// (a, b) of a head to (a cos - b sin, a sin + b cos) (85-107); attention is
// causal softmax(q.k / sqrt(hd)) v with consecutive query heads sharing a KV
// head (126-215); the merged SwiGLU is silu(g) * u over [G | U] (224-276).
// The K/V cache is fp16.
//
// Every step runs on the caller's stream.  The current token, the position
// and the prompt live in device memory, so one captured CUDA graph serves
// every step of a sequence (prompt feeding and greedy decoding alike).  The
// launches use programmatic dependent launch: each kernel waits
// (griddepcontrol.wait) before reading what the previous kernel wrote, and
// lets the next kernel start its independent prologue (the weight stream of
// a matvec) early.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <dlfcn.h>
#include <stdio.h>

#include <utility>
#include <vector>

#include "../../include/tcb.h"
#include "tcb_common.cuh"
#include "tcb_ctx.h"
#include "tcb_gemm_tc.h"
#include "tcb_launch.h"
#include "tcb_matvec.h"
#include "tcb_mv_ptx.cuh"

namespace tcb {
namespace ll {

// L2 loads kept in program order with the dependency wait: the asm of
// __ldcg is not volatile and names no memory, so the compiler may move it
// past griddepcontrol.wait; these may not be moved across it
__device__ __forceinline__ uint4 ldcg_v4_ordered(const void *p) {
  uint4 r;
  asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ uint2 ldcg_v2_ordered(const void *p) {
  uint2 r;
  asm volatile("ld.global.cg.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

constexpr int kHd = 128;        // head dimension supported by the attention kernel
constexpr int kChunk = 64;      // positions per attention CTA
constexpr int kMaxChunks = 256; // chunks a merge holds in shared memory (max_ctx <= 16384)
constexpr int kArgBlocks = 148;
constexpr int kPrefillRows = 2048;  // prompt rows per pass of tcb_llama_prefill

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}
__device__ __forceinline__ float warp_add(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
  return v;
}

// out = x / sqrt(mean(x^2) + eps) * w   (one CTA per row)
__global__ void k_rmsnorm(const float *x, const float *w, float *out, int D, float eps) {
  __shared__ float red[32];
  x += (size_t)blockIdx.x * D;
  out += (size_t)blockIdx.x * D;
  mv::pdl_wait();
  float ss = 0.f;
  for (int i = threadIdx.x; i < D; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
  ss = warp_add(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_add(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  mv::pdl_launch_dependents();
  const float s = sqrtf(__fdiv_rn(red[0], (float)D) + eps);
  for (int i = threadIdx.x; i < D; i += blockDim.x) out[i] = __fmul_rn(__fdiv_rn(x[i], s), w[i]);
}

// One sequence of a batched decode step (tcb_llama_batch): where its
// position, current token and (layer 0 of its) K/V cache live.
struct BatchSeq {
  const int *pos;
  __half *kc, *vc;
  const int64_t *tok;
};
// where a batch's greedy pick writes each sequence's next token
struct BatchPick {
  int *pos;
  int64_t *tok, *hist;
  const int64_t *prompt;
  const int *nprompt;
};

// The current tokens of a batch's sequences, gathered into one array.
__global__ void k_gather_tok(const BatchSeq *bs, int B, int64_t *tok) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) tok[b] = *bs[b].tok;
}

// One layer's attention at position *pos: CTA (query heads GS*blockIdx.x ..
// + GS - 1, chunk blockIdx.y of kChunk positions), 256 threads.  The G query
// heads of a KV head are spread over gsplit = G/GS CTAs (KV head
// blockIdx.x / gsplit), chosen by the host so that the grid fills the SMs
// when the KV heads are few (a tensor-parallel rank holds one of the 70B
// model's eight).  In a batched step
// (bs != nullptr) blockIdx.z is the sequence: its position and cache come
// from bs[z] (plus layer_off), and its qkv row, output row, chunk partials
// and chunk counters are z strides into the batch's buffers.  Every cached K and V byte of
// the chunk is requested before the dependency wait (K: thread = (position
// t/4, 32 dimensions (t%4)*32); V: thread = (dimensions (t%32)*4, positions
// t/32 + 8j)), so the loads overlap the qkv product.  The CTA rotates the
// query rows of its GS query heads; the CTAs whose chunk holds pos also
// rotate the new key and use it and the new value from shared memory for
// that position, and the first of the KV head's CTAs stores both into the
// fp16 cache.  Each CTA writes its chunk's (max, sum, unnormalised output)
// per query head; the last CTA of a head group to finish (a counter per
// group, reset by that CTA) merges the chunks in chunk order, so the result
// does not depend on timing.
template <int GS>
__global__ void __launch_bounds__(256) k_attn(const float *qkv, const float *cosT, const float *sinT, const int *pos,
                                              __half *kc, __half *vc, float *part, unsigned *count, float *out, int H,
                                              int KVH, int gsplit, int max_ctx, int nch_max, float scale, const BatchSeq *bs,
                                              size_t layer_off) {
  constexpr int half = kHd / 2;
  if (bs) {
    const int z = blockIdx.z;
    pos = bs[z].pos;
    kc = bs[z].kc + layer_off;
    vc = bs[z].vc + layer_off;
    qkv += (size_t)z * (H + 2 * KVH) * kHd;
    out += (size_t)z * H * kHd;
    part += (size_t)z * H * nch_max * (2 + kHd);
    count += (size_t)z * H;
  }
  __shared__ __align__(16) float qs[GS][kHd];
  __shared__ float knew[kHd], vnew[kHd];
  __shared__ float sc[GS][kChunk];
  __shared__ float gm[GS], gl[GS];
  __shared__ float wo[8][GS][kHd];
  __shared__ int last;
  // The position and the cached K/V rows before it were written by earlier
  // steps (every step starts with a plain launch, after the previous one has
  // completed) or by the prompt pass: they are read before the dependency
  // wait, while the qkv product finishes.  Row p is this step's, written
  // below by the CTA that holds it.
  const int p = *pos, n = p + 1, kh = blockIdx.x / gsplit, c = blockIdx.y, t0 = c * kChunk;
  const int hq = blockIdx.x * GS;  // the CTA's first query head
  if (t0 >= n) return;
  const int tid = threadIdx.x;
  const __half *kbase = kc + (size_t)kh * max_ctx * kHd, *vbase = vc + (size_t)kh * max_ctx * kHd;
  // K: position tk, dims 32*sk..; V: dims 4*(tid%32).., positions tv + 8j
  const int tk = t0 + (tid >> 2), sk = tid & 3, dv = 4 * (tid & 31), tv = t0 + (tid >> 5);
  uint4 kr[4];
  uint2 vr[kChunk / 8];
  const bool kok = tk < n && tk != p;
  if (kok) {
#pragma unroll
    for (int j = 0; j < 4; j++) kr[j] = ldcg_v4_ordered(reinterpret_cast<const uint4 *>(kbase + (size_t)tk * kHd + 32 * sk) + j);
  }
#pragma unroll
  for (int j = 0; j < kChunk / 8; j++) {
    const int t = tv + 8 * j;
    if (t < n && t != p) vr[j] = ldcg_v2_ordered(reinterpret_cast<const uint2 *>(vbase + (size_t)t * kHd + dv));
  }
  mv::pdl_wait();
  // the next kernel (the o projection) may launch now: its weight stream does
  // not depend on this one, and it waits for this grid before reading `out`
  mv::pdl_launch_dependents();
  const float *cs = cosT + (size_t)p * half, *sn = sinT + (size_t)p * half;
  for (int i = tid; i < GS * half; i += blockDim.x) {
    const int g = i / half, j = i % half;
    const float *row = qkv + (size_t)(hq + g) * kHd;
    const float a = row[j], b = row[j + half];
    qs[g][j] = __fsub_rn(__fmul_rn(a, cs[j]), __fmul_rn(b, sn[j]));
    qs[g][j + half] = __fadd_rn(__fmul_rn(a, sn[j]), __fmul_rn(b, cs[j]));
  }
  const bool tail = p < t0 + kChunk;
  if (tail) {
    const float *krow = qkv + (size_t)(H + kh) * kHd, *vrow = qkv + (size_t)(H + KVH + kh) * kHd;
    __half *kd = kc + ((size_t)kh * max_ctx + p) * kHd, *vd = vc + ((size_t)kh * max_ctx + p) * kHd;
    if (tid < half) {
      const float a = krow[tid], b = krow[tid + half];
      const __half ka = __float2half_rn(__fsub_rn(__fmul_rn(a, cs[tid]), __fmul_rn(b, sn[tid])));
      const __half kb = __float2half_rn(__fadd_rn(__fmul_rn(a, sn[tid]), __fmul_rn(b, cs[tid])));
      if (blockIdx.x % gsplit == 0) {
        kd[tid] = ka;
        kd[tid + half] = kb;
      }
      knew[tid] = __half2float(ka);
      knew[tid + half] = __half2float(kb);
    } else if (tid < half + kHd) {
      const __half v = __float2half_rn(vrow[tid - half]);
      if (blockIdx.x % gsplit == 0) vd[tid - half] = v;
      vnew[tid - half] = __half2float(v);
    }
  }
  __syncthreads();
  // scores: four threads per position, 32 dimensions each
  {
    float s[GS];
#pragma unroll
    for (int g = 0; g < GS; g++) s[g] = 0.f;
    if (tk < n) {
      float kv[32];
      if (tk == p) {
#pragma unroll
        for (int i = 0; i < 32; i++) kv[i] = knew[32 * sk + i];
      } else {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const __half2 *h2 = reinterpret_cast<const __half2 *>(&kr[j]);
#pragma unroll
          for (int i = 0; i < 4; i++) {
            const float2 f = __half22float2(h2[i]);
            kv[8 * j + 2 * i] = f.x;
            kv[8 * j + 2 * i + 1] = f.y;
          }
        }
      }
      // 16-byte q loads (a broadcast among the lanes of one sk) and the GS
      // heads' chains interleaved
#pragma unroll
      for (int i4 = 0; i4 < 8; i4++)
#pragma unroll
        for (int g = 0; g < GS; g++) {
          const float4 q4 = *reinterpret_cast<const float4 *>(&qs[g][32 * sk + 4 * i4]);
          s[g] = fmaf(q4.x, kv[4 * i4], s[g]);
          s[g] = fmaf(q4.y, kv[4 * i4 + 1], s[g]);
          s[g] = fmaf(q4.z, kv[4 * i4 + 2], s[g]);
          s[g] = fmaf(q4.w, kv[4 * i4 + 3], s[g]);
        }
    }
#pragma unroll
    for (int g = 0; g < GS; g++) {
      s[g] += __shfl_xor_sync(0xFFFFFFFFu, s[g], 1);
      s[g] += __shfl_xor_sync(0xFFFFFFFFu, s[g], 2);
      if (sk == 0) sc[g][tid >> 2] = tk < n ? s[g] * scale : -INFINITY;
    }
  }
  __syncthreads();
  // chunk softmax: warp g, two positions per lane
  {
    const int w = tid >> 5, lane = tid & 31;
    if (w < GS) {
      const float a = sc[w][lane], b = sc[w][lane + 32];
      const float m = warp_max(fmaxf(a, b));
      const float ea = a == -INFINITY ? 0.f : __expf(a - m), eb = b == -INFINITY ? 0.f : __expf(b - m);
      const float l = warp_add(ea + eb);
      sc[w][lane] = ea;
      sc[w][lane + 32] = eb;
      if (lane == 0) {
        gm[w] = m;
        gl[w] = l;
      }
    }
  }
  __syncthreads();
  // values: thread = 4 dimensions x positions tv + 8j
  {
    float o[GS][4];
#pragma unroll
    for (int g = 0; g < GS; g++) o[g][0] = o[g][1] = o[g][2] = o[g][3] = 0.f;
#pragma unroll
    for (int j = 0; j < kChunk / 8; j++) {
      const int t = tv + 8 * j;
      if (t >= n) break;
      float v[4];
      if (t == p) {
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = vnew[dv + i];
      } else {
        const __half2 *h2 = reinterpret_cast<const __half2 *>(&vr[j]);
        const float2 a = __half22float2(h2[0]), b = __half22float2(h2[1]);
        v[0] = a.x, v[1] = a.y, v[2] = b.x, v[3] = b.y;
      }
#pragma unroll
      for (int g = 0; g < GS; g++) {
        const float pj = sc[g][t - t0];
#pragma unroll
        for (int i = 0; i < 4; i++) o[g][i] = fmaf(pj, v[i], o[g][i]);
      }
    }
#pragma unroll
    for (int g = 0; g < GS; g++)
#pragma unroll
      for (int i = 0; i < 4; i++) wo[tid >> 5][g][dv + i] = o[g][i];
  }
  __syncthreads();
  for (int i = tid; i < GS * kHd; i += blockDim.x) {
    const int g = i / kHd, d = i % kHd;
    float O = 0.f;
#pragma unroll
    for (int w = 0; w < 8; w++) O += wo[w][g][d];
    float *pp = part + ((size_t)(hq + g) * nch_max + c) * (2 + kHd);
    pp[2 + d] = O;
    if (d == 0) {
      pp[0] = gm[g];
      pp[1] = gl[g];
    }
  }
  // the last CTA of this KV head merges the chunks
  __threadfence();
  __syncthreads();
  const int nch = (n + kChunk - 1) / kChunk;
  if (tid == 0) last = atomicAdd(&count[blockIdx.x], 1u) == (unsigned)(nch - 1);
  __syncthreads();
  if (!last) return;
  __threadfence();
  // merge: every chunk's (max, sum) into shared memory at once (the per-warp
  // output buffer is free again), one warp per query head forms the chunk
  // weights exp(m_c - M) and L, then each thread sums its output element over
  // the chunks in chunk order with the loads issued ahead
  float *cw = &wo[0][0][0], *cl = cw + GS * nch;  // [GS][nch] each
  for (int i = tid; i < GS * nch; i += blockDim.x) {
    const int g = i / nch, cc = i % nch;
    const float *pc = part + ((size_t)(hq + g) * nch_max + cc) * (2 + kHd);
    cw[i] = __ldcg(pc);
    cl[i] = __ldcg(pc + 1);
  }
  __syncthreads();
  {
    const int w = tid >> 5, lane = tid & 31;
    if (w < GS) {
      float M = -INFINITY;
      for (int cc = lane; cc < nch; cc += 32) M = fmaxf(M, cw[w * nch + cc]);
      M = warp_max(M);
      __syncwarp();
      for (int cc = lane; cc < nch; cc += 32) cw[w * nch + cc] = __expf(cw[w * nch + cc] - M);
      __syncwarp();
      if (lane == 0) {
        float L = 0.f;
        for (int cc = 0; cc < nch; cc++) L = fmaf(cl[w * nch + cc], cw[w * nch + cc], L);
        gl[w] = L;
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < GS * kHd; i += blockDim.x) {
    const int g = i / kHd, d = i % kHd;
    const float *ph = part + (size_t)(hq + g) * nch_max * (2 + kHd) + 2 + d;
    float O = 0.f;
    int cc = 0;
    for (; cc + 4 <= nch; cc += 4) {
      const float o0 = __ldcg(ph + (size_t)cc * (2 + kHd)), o1 = __ldcg(ph + (size_t)(cc + 1) * (2 + kHd));
      const float o2 = __ldcg(ph + (size_t)(cc + 2) * (2 + kHd)), o3 = __ldcg(ph + (size_t)(cc + 3) * (2 + kHd));
      O = fmaf(o0, cw[g * nch + cc], O);
      O = fmaf(o1, cw[g * nch + cc + 1], O);
      O = fmaf(o2, cw[g * nch + cc + 2], O);
      O = fmaf(o3, cw[g * nch + cc + 3], O);
    }
    for (; cc < nch; cc++) O = fmaf(__ldcg(ph + (size_t)cc * (2 + kHd)), cw[g * nch + cc], O);
    out[(size_t)(hq + g) * kHd + d] = __fdiv_rn(O, gl[g]);
  }
  if (tid == 0) count[blockIdx.x] = 0u;
}

// ---- all-reduce of the residual over peer memory (tensor parallelism)
//
// Every rank's exchange buffer (cudaMalloc'd, mapped into the other ranks by
// CUDA IPC) holds slots [2][tp][stride] of 8-byte words, of which a call uses
// the first D of each (stride is fixed per buffer, so a call of D values
// never reaches into the other parity, whatever D the calls around it had): the low half a value's
// bits, the high half the number e of the call that wrote it.  Call e (a
// per-rank counter that all ranks advance alike) uses parity e & 1.  Block b
// of rank r stores its slice of r's partial, each value paired with e in
// one 8-byte store, into slot [par][r] of every rank (peer stores over
// NVLink); it then polls the same slice of its own slots [par][r'] until
// every word carries e, and adds the ranks' values in rank order to the
// residual: x += ((y_0 + y_1) + ...) -- the same operations on every rank, so
// the ranks keep identical residuals.  An aligned 8-byte store is seen whole
// or not at all, so a word that carries e carries e's value: no fence or
// flag sits between the data and the signal that it is there.  A slot
// parity is written again only two calls later, when every rank has
// finished the call in between and therefore read the old contents.  Waits
// are bounded (about a second); a timeout records TCB_ERR_TIMEOUT.
constexpr int kArBlocks = 16, kArThreads = 128, kMaxTp = 8;
constexpr int kPeerRows = 16;  // rows of d_model values a slot holds (a batched step of up to 16 sequences)
struct PeerBufs {
  unsigned long long *slot[kMaxTp];  // rank r's slots [2][tp][stride] (this process's mapping)
};

__device__ __forceinline__ void st_words(unsigned long long *p, unsigned long long a, unsigned long long b) {
  asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_words(const unsigned long long *p, unsigned long long &a, unsigned long long &b) {
  asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

constexpr unsigned kArPolls = 1u << 22;  // polls of a word pair before a wait gives up (about a second)
__global__ void __launch_bounds__(kArThreads) k_peer_ar(const __grid_constant__ PeerBufs pb, const float *yp, float *x, int D, long stride,
                                                       int tp, int rank, unsigned *epoch, unsigned *done, int *err,
                                                       unsigned polls) {
  mv::pdl_wait();
  mv::pdl_launch_dependents();
  const unsigned e = *reinterpret_cast<volatile unsigned *>(epoch) + 1u;
  const int par = (int)(e & 1u), b = blockIdx.x, nb = gridDim.x;
  const int per = ((D + nb - 1) / nb + 1) & ~1;
  const int i0 = b * per, i1 = min(D, i0 + per);
  const unsigned long long tag = (unsigned long long)e << 32;
  for (int i = i0 + 2 * (int)threadIdx.x; i < i1; i += 2 * blockDim.x) {
    const float2 v = *reinterpret_cast<const float2 *>(yp + i);
    const unsigned long long a = tag | __float_as_uint(v.x), c = tag | __float_as_uint(v.y);
    for (int r = 0; r < tp; r++) st_words(pb.slot[r] + ((size_t)par * tp + rank) * stride + i, a, c);
  }
  const unsigned long long *mine = pb.slot[rank] + (size_t)par * tp * stride;
  bool ok = true;
  for (int i = i0 + 2 * (int)threadIdx.x; i < i1; i += 2 * blockDim.x) {
    float s0 = 0.f, s1 = 0.f;
    for (int r = 0; r < tp; r++) {
      unsigned long long a = 0, c = 0;
      for (uint32_t it = 0; ok; it++) {
        ld_words(mine + (size_t)r * stride + i, a, c);
        if ((unsigned)(a >> 32) == e && (unsigned)(c >> 32) == e) break;
        if (it + 1 >= polls) ok = false;  // gave up: no further waits in this call
        else __nanosleep(32);
      }
      const float va = __uint_as_float((unsigned)a), vc = __uint_as_float((unsigned)c);
      s0 = r == 0 ? va : __fadd_rn(s0, va);
      s1 = r == 0 ? vc : __fadd_rn(s1, vc);
    }
    float2 xv = *reinterpret_cast<float2 *>(x + i);
    xv.x = __fadd_rn(xv.x, s0);
    xv.y = __fadd_rn(xv.y, s1);
    *reinterpret_cast<float2 *>(x + i) = xv;
  }
  if (!ok) atomicExch(err, TCB_ERR_TIMEOUT);
  // the last block to finish advances the counter (every block has read it)
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(done, 1u) == (unsigned)nb - 1u) {
      *done = 0u;
      *reinterpret_cast<volatile unsigned *>(epoch) = e;
      __threadfence();
    }
  }
}

// a = silu(g) * u over the merged [G | U] rows
__global__ void k_swiglu(const float *gu, float *a, int F) {
  mv::pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  mv::pdl_launch_dependents();
  if (i < F) {
    const float g = gu[i], u = gu[F + i];
    a[i] = __fmul_rn(__fmul_rn(g, __frcp_rn(__fadd_rn(1.0f, expf(-g)))), u);
  }
}

// ---- prompt rows (tcb_llama_prefill)

// Row r of the chunk (position p0 + r): rotate its query and key heads with
// the decode step's arithmetic, query heads in place, and store the rotated
// key and the value heads into the fp16 cache.  One CTA per row.
__global__ void k_rope_rows(float *qkv, const float *cosT, const float *sinT, int p0, __half *kc, __half *vc, int H,
                            int KVH, int max_ctx) {
  constexpr int half = kHd / 2;
  const int r = blockIdx.x, p = p0 + r;
  float *row = qkv + (size_t)r * (H + 2 * KVH) * kHd;
  const float *cs = cosT + (size_t)p * half, *sn = sinT + (size_t)p * half;
  for (int i = threadIdx.x; i < (H + KVH) * half; i += blockDim.x) {
    const int hh = i / half, j = i % half;
    float *v = row + (size_t)hh * kHd;
    const float a = v[j], b = v[j + half];
    const float ra = __fsub_rn(__fmul_rn(a, cs[j]), __fmul_rn(b, sn[j]));
    const float rb = __fadd_rn(__fmul_rn(a, sn[j]), __fmul_rn(b, cs[j]));
    if (hh < H) {
      v[j] = ra;
      v[j + half] = rb;
    } else {
      __half *kd = kc + ((size_t)(hh - H) * max_ctx + p) * kHd;
      kd[j] = __float2half_rn(ra);
      kd[j + half] = __float2half_rn(rb);
    }
  }
  for (int i = threadIdx.x; i < KVH * kHd; i += blockDim.x) {
    const int kh = i / kHd, d = i % kHd;
    vc[((size_t)kh * max_ctx + p) * kHd + d] = __float2half_rn(row[(size_t)(H + KVH + kh) * kHd + d]);
  }
}

// a[r][i] = silu(g) * u over rows of merged [G | U] (k_swiglu per row)
__global__ void k_swiglu_rows(const float *gu, float *a, int F, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const long r = i / F;
    const int c = (int)(i - r * F);
    const float g = gu[r * 2 * F + c], u = gu[r * 2 * F + F + c];
    a[i] = __fmul_rn(__fmul_rn(g, __frcp_rn(__fadd_rn(1.0f, expf(-g)))), u);
  }
}

// the state n-1 prompt steps leave: history = prompt[0..n-1], position n-1,
// current token prompt[n-1]
__global__ void k_prefill_done(const int64_t *prompt, int n, int *pos, int64_t *tok, int64_t *hist) {
  for (int i = threadIdx.x; i < n; i += blockDim.x) hist[i] = prompt[i];
  if (threadIdx.x == 0) {
    *pos = n - 1;
    *tok = prompt[n - 1];
  }
}

// (max, first index) per CTA
// blockIdx.y: the row of v (n apart) in a batch, partials gridDim.x apart
__global__ void k_argmax_part(const float *v, int n, float *pm, int *pi) {
  __shared__ float sm_v[32];
  __shared__ int sm_i[32];
  v += (size_t)blockIdx.y * n;
  pm += (size_t)blockIdx.y * gridDim.x;
  pi += (size_t)blockIdx.y * gridDim.x;
  mv::pdl_wait();
  float best = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float x = v[i];
    if (x > best) {
      best = x;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sm_v[threadIdx.x >> 5] = best;
    sm_i[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  mv::pdl_launch_dependents();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      if (sm_v[w] > best || (sm_v[w] == best && sm_i[w] < bi)) {
        best = sm_v[w];
        bi = sm_i[w];
      }
    pm[blockIdx.x] = best;
    pi[blockIdx.x] = bi;
  }
}

// The next token: the prompt's next id while the prompt lasts, else the
// first maximum of the logits; recorded at tokens[pos + 1]; pos advances.
// One warp; with bp, warp (CTA) b picks sequence b of a batch.
__global__ void k_next_token(const float *pm, const int *pi, int nb, int *pos, int64_t *tok, int64_t *hist,
                             const int64_t *prompt, const int *nprompt, int max_ctx, const BatchPick *bp) {
  if (bp) {
    const BatchPick q = bp[blockIdx.x];
    pm += (size_t)blockIdx.x * nb;
    pi += (size_t)blockIdx.x * nb;
    pos = q.pos, tok = q.tok, hist = q.hist, prompt = q.prompt, nprompt = q.nprompt;
  }
  mv::pdl_wait();
  const int lane = threadIdx.x;
  float best = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int b = lane; b < nb; b += 32) {
    const float v = pm[b];
    const int i = pi[b];
    if (i != 0x7FFFFFFF && (bi == 0x7FFFFFFF || v > best || (v == best && i < bi))) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
    if (oi != 0x7FFFFFFF && (bi == 0x7FFFFFFF || ob > best || (ob == best && oi < bi))) {
      best = ob;
      bi = oi;
    }
  }
  if (lane == 0) {
    const int p = *pos;
    const int64_t next = (p + 1 < *nprompt) ? prompt[p + 1] : (int64_t)(bi == 0x7FFFFFFF ? 0 : bi);
    if (p + 1 < max_ctx) hist[p + 1] = next;
    *tok = next;
    *pos = p + 1;
  }
  mv::pdl_launch_dependents();
}

// Tensor parallelism: this rank's greedy candidate (first maximum of its
// vocabulary rows, as a global index), for the all-gather.
// CTA b: candidate b of a batch (partials nb apart)
__global__ void k_local_best(const float *pm, const int *pi, int nb, int off, int2 *cand) {
  pm += (size_t)blockIdx.x * nb;
  pi += (size_t)blockIdx.x * nb;
  cand += blockIdx.x;
  mv::pdl_wait();
  const int lane = threadIdx.x;
  float best = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int b = lane; b < nb; b += 32) {
    const float v = pm[b];
    const int i = pi[b];
    if (i != 0x7FFFFFFF && (bi == 0x7FFFFFFF || v > best || (v == best && i < bi))) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xFFFFFFFFu, best, o);
    const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
    if (oi != 0x7FFFFFFF && (bi == 0x7FFFFFFF || ob > best || (ob == best && oi < bi))) {
      best = ob;
      bi = oi;
    }
  }
  if (lane == 0) *cand = make_int2(__float_as_int(best), bi == 0x7FFFFFFF ? bi : bi + off);
  mv::pdl_launch_dependents();
}

// the next token from the ranks' candidates (rank order = vocabulary order,
// so ties still go to the lowest index)
__global__ void k_pick_tp(const int2 *cand, int n, int stride, int *pos, int64_t *tok, int64_t *hist,
                          const int64_t *prompt, const int *nprompt, int max_ctx, const BatchPick *bp) {
  if (bp) {
    const BatchPick q = bp[blockIdx.x];
    cand += blockIdx.x;
    pos = q.pos, tok = q.tok, hist = q.hist, prompt = q.prompt, nprompt = q.nprompt;
  }
  mv::pdl_wait();
  if (threadIdx.x != 0) return;
  float best = -INFINITY;
  int bi = 0x7FFFFFFF;
  for (int r = 0; r < n; r++) {
    const float v = __int_as_float(cand[(size_t)r * stride].x);
    const int i = cand[(size_t)r * stride].y;
    if (i != 0x7FFFFFFF && (bi == 0x7FFFFFFF || v > best || (v == best && i < bi))) {
      best = v;
      bi = i;
    }
  }
  const int p = *pos;
  const int64_t next = (p + 1 < *nprompt) ? prompt[p + 1] : (int64_t)(bi == 0x7FFFFFFF ? 0 : bi);
  if (p + 1 < max_ctx) hist[p + 1] = next;
  *tok = next;
  *pos = p + 1;
  mv::pdl_launch_dependents();
}

template <typename... Exp, typename... Act>
cudaError_t launch(void (*k)(Exp...), dim3 grid, dim3 block, cudaStream_t s, Act &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Act>(args)...);
}

}  // namespace ll
}  // namespace tcb

// ----------------------------------------------------------------- NCCL

namespace {

// NCCL, loaded at run time (no link dependency): the copy a process has
// already loaded (e.g. by its framework) is reused, else libnccl.so.2 from
// the loader's path.  Types restated from nccl.h: an opaque communicator, a
// 128-byte id passed by value, int enums (float32 = 7, int32 = 2, sum = 0).
struct NcclId {
  char internal[128];
};
struct Nccl {
  void *h = nullptr;
  int (*get_id)(NcclId *) = nullptr;
  int (*init_rank)(void **, int, NcclId, int) = nullptr;
  int (*all_reduce)(const void *, void *, size_t, int, int, void *, cudaStream_t) = nullptr;
  int (*all_gather)(const void *, void *, size_t, int, void *, cudaStream_t) = nullptr;
  int (*destroy)(void *) = nullptr;
  const char *(*err)(int) = nullptr;
};
constexpr int kNcclInt32 = 2, kNcclFloat32 = 7, kNcclSum = 0;

const Nccl *nccl() {
  static Nccl n = [] {
    Nccl r;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return r;
    r.get_id = reinterpret_cast<int (*)(NcclId *)>(dlsym(h, "ncclGetUniqueId"));
    r.init_rank = reinterpret_cast<int (*)(void **, int, NcclId, int)>(dlsym(h, "ncclCommInitRank"));
    r.all_reduce =
        reinterpret_cast<int (*)(const void *, void *, size_t, int, int, void *, cudaStream_t)>(dlsym(h, "ncclAllReduce"));
    r.all_gather =
        reinterpret_cast<int (*)(const void *, void *, size_t, int, void *, cudaStream_t)>(dlsym(h, "ncclAllGather"));
    r.destroy = reinterpret_cast<int (*)(void *)>(dlsym(h, "ncclCommDestroy"));
    r.err = reinterpret_cast<const char *(*)(int)>(dlsym(h, "ncclGetErrorString"));
    if (r.get_id && r.init_rank && r.all_reduce && r.all_gather && r.destroy && r.err) r.h = h;
    return r;
  }();
  return n.h ? &n : nullptr;
}

}  // namespace

// ----------------------------------------------------------------- engine

namespace {

struct Mat {
  const void *w = nullptr;
  int type = 0, N = 0, K = 0;
  // Q6_K rows of 210 * K/256 bytes, not a multiple of 16 (a tensor-parallel
  // shard of o or down, e.g. K = 1024 or 3584) or not 16-byte aligned, cannot
  // be mapped by TMA: the engine keeps a copy with every row padded to ldw
  // bytes (a multiple of 16) for the matvec kernels, and plan reads it
  const void *wp = nullptr;
  long ldw = 0;
  tcb::MvPlan plan{};
  tcb::MvPlan swi{};         // gate_up (Q4_K): the launch that writes silu(g) * u itself
  const void *pf = nullptr;  // the next matvec's weights in the step (L2 prefetch while this one runs)
  size_t pf_bytes = 0;
  size_t bytes() const { return (size_t)N * K / tcb::block_elems(type) * tcb::block_bytes(type); }
  const void *wk() const { return wp ? wp : w; }                    // the weights the matvec plans read
  size_t kbytes() const { return wp ? (size_t)N * ldw : bytes(); }  // and their size
};

}  // namespace

struct tcb_llama {
  tcb_ctx *ctx = nullptr;
  tcb_llama_config cfg{};
  const void *tok_emb = nullptr;
  int tok_emb_type = 0;
  const float *final_norm = nullptr;
  std::vector<const float *> attn_norm, ffn_norm;
  Mat head;
  std::vector<Mat> qkv, o, gu, down;
  std::vector<Mat> qkv_v;  // a layer's v rows when their block type differs from q/k's (N = 0: none)
  // device state
  float *x = nullptr, *h = nullptr, *qkvb = nullptr, *att = nullptr, *gub = nullptr, *a = nullptr, *logits = nullptr;
  float *part = nullptr, *am_v = nullptr, *cosT = nullptr, *sinT = nullptr;
  int *am_i = nullptr, *pos = nullptr, *nprompt = nullptr;
  unsigned *acount = nullptr;  // per attention head group: chunks finished
  int gsplit = 1;              // attention CTAs per KV head (query heads split between them)
  __half *kc = nullptr, *vc = nullptr;
  int64_t *tok = nullptr, *hist = nullptr, *prompt = nullptr;
  int nch_max = 0;
  int host_pos = 0;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaStream_t cap = nullptr;  // capture stream (the caller's may be the legacy default stream)
  std::vector<void *> allocs;
  // tensor parallelism: cfg holds this rank's local dimensions
  int tp = 1, tr = 0, vocab_all = 0, vocab_off = 0;
  void *comm = nullptr;  // ncclComm_t
  int2 *cand = nullptr;  // greedy candidates [tp]
  void *sk = nullptr;    // split-K scratch shared by the step's matvecs (they run one after another)
  int nccl_rc = 0;       // last NCCL error
  // peer-memory all-reduce (tcb_llama_peer_init); NCCL's when not set up
  char *xbuf = nullptr;              // this rank's exchange buffer (slots of the peer all-reduce)
  size_t xbuf_bytes = 0;
  tcb::ll::PeerBufs pb{};
  std::vector<void *> opened;        // peers' buffers opened through CUDA IPC
  bool peer = false;
  float *yp = nullptr;               // this rank's partial of o / down
  unsigned *ar_epoch = nullptr, *ar_done = nullptr;
  // prompt pass (tcb_llama_prefill): row buffers of pf_rows rows, made on first use
  int host_n = 0;                    // prompt length given to tcb_llama_start
  int pf_pass = 0;                   // rows per pass (tcb_llama_set_prefill_rows; 0: kPrefillRows)
  int pf_rows = 0;
  float *px = nullptr, *ph = nullptr, *pqkv = nullptr, *patt = nullptr, *pgu = nullptr, *pa = nullptr;
};

namespace {

int fail(tcb_llama *m, cudaError_t e) {
  if (m && m->ctx) {
    if (m->nccl_rc && nccl())
      snprintf(m->ctx->err, sizeof m->ctx->err, "NCCL: %s", nccl()->err(m->nccl_rc));
    else if (e == cudaErrorNotReady && m->tp > 1 && !m->comm)
      snprintf(m->ctx->err, sizeof m->ctx->err, "tensor parallelism: tcb_llama_tp_init was not called");
    else
      snprintf(m->ctx->err, sizeof m->ctx->err, "%s", cudaGetErrorString(e));
  }
  return TCB_ERR_CUDA;
}

template <class T>
cudaError_t alloc(tcb_llama *m, T **p, size_t n) {
  void *q = nullptr;
  cudaError_t e = cudaMalloc(&q, n * sizeof(T) + 16);
  if (e == cudaSuccess) {
    m->allocs.push_back(q);
    *p = static_cast<T *>(q);
  }
  return e;
}

bool wtype_ok(int t) { return t == TCB_Q4_0 || t == TCB_Q8_0 || t == TCB_Q4_K || t == TCB_Q6_K; }

Mat make_mat(const void *w, int type, int N, int K, int sms) {
  Mat mt;
  mt.w = w;
  mt.type = type;
  mt.N = N;
  mt.K = K;
  mt.plan = tcb::matvec_plan(type, 0, 1, N, K, w, sms);
  return mt;
}

// y (+)= W x for one row of activations (f32 in, f32 out)
cudaError_t matvec(tcb_llama *m, const Mat &mt, const float *x, float *y, int accumulate, cudaStream_t s) {
  if (mt.plan.ok)
    return tcb::matvec_launch(mt.plan, mt.type, 0, mt.N, mt.K, mt.wk(), x, TCB_F32, y, TCB_F32, accumulate,
                              m->ctx->derr, s, mt.pf, mt.pf_bytes, m->sk);
  return tcb::launch_qgemm_simt(mt.type, mt.w, 1, mt.N, mt.K, x, TCB_F32, mt.K, y, TCB_F32, mt.N, accumulate,
                                m->ctx->sms, s);
}

// y = W rms(x) * w: the RMSNorm is fused into the Q4_K matvec's prologue
// when that kernel takes the weight, else a separate pass into h
cudaError_t norm_matvec(tcb_llama *m, const Mat &mt, const float *nw, float *y, cudaStream_t s) {
  const tcb_llama_config &c = m->cfg;
  if (mt.plan.ok && mt.plan.kind == 1)
    return tcb::q4k_launch(mt.plan, mt.N, mt.K, mt.w, m->x, TCB_F32, y, TCB_F32, 0, m->ctx->derr, m->sk, s, nw, c.eps,
                           mt.pf, mt.pf_bytes);
  cudaError_t e = tcb::ll::launch(tcb::ll::k_rmsnorm, dim3(1), dim3(1024), s, m->x, nw, m->h, c.d_model, c.eps);
  return e == cudaSuccess ? matvec(m, mt, m->h, y, 0, s) : e;
}

// x <- sum over ranks (in place), tensor parallelism only.  With the peer
// all-reduce every rank's partial is in yp and x holds the residual.
cudaError_t all_reduce_x(tcb_llama *m, cudaStream_t s) {
  if (m->tp == 1) return cudaSuccess;
  if (m->peer)
    return tcb::ll::launch(tcb::ll::k_peer_ar, dim3(tcb::ll::kArBlocks), dim3(tcb::ll::kArThreads), s, m->pb,
                           (const float *)m->yp, m->x, m->cfg.d_model, (long)tcb::ll::kPeerRows * m->cfg.d_model,
                           m->tp, m->tr, m->ar_epoch, m->ar_done,
                           m->ctx->derr, tcb::ll::kArPolls);
  const Nccl *nc = nccl();
  if (!nc || !m->comm) return cudaErrorNotReady;
  m->nccl_rc = nc->all_reduce(m->x, m->x, (size_t)m->cfg.d_model, kNcclFloat32, kNcclSum, m->comm, s);
  return m->nccl_rc ? cudaErrorUnknown : cudaSuccess;
}

// Attention CTAs per KV head: the most (a power of two dividing the G query
// heads of a KV head) that keep the grid of every chunk of B sequences
// within four CTAs per SM (a CTA is 256 threads and at most 42 KB of shared
// memory; four measured faster than two: 8B decode 472 against 465 tok/s,
// 70B 71.2 against 69.2).  A CTA's time is a chain of dependent steps over
// its G/gsplit heads, so with few KV heads (a tensor-parallel rank) spreading
// the heads over more SMs shortens the launch.
int attn_split(int G, int KVH, int nch_max, int B, int sms) {
  int gs = 1;
  while (G % (2 * gs) == 0 && (long)KVH * 2 * gs * nch_max * B <= 4L * sms) gs *= 2;
  return gs;
}

cudaError_t issue_step(tcb_llama *m, cudaStream_t s) {
  using namespace tcb::ll;
  const tcb_llama_config &c = m->cfg;
  const int H = c.n_heads, KVH = c.n_kv_heads, hd = c.head_dim, D = c.d_model, F = c.ffn_dim;
  const int G = H / KVH;
  const float scale = 1.0f / sqrtf((float)hd);
  const size_t cache_layer = (size_t)KVH * c.max_ctx * hd;
  // a plain launch (no programmatic dependency): the step starts after the
  // previous one has completed, which k_attn relies on when it reads the
  // cached K/V before its dependency wait
  cudaError_t e = tcb::launch_dequant_rows(m->tok_emb_type, m->tok_emb, 1, D, m->tok, m->x, TCB_F32, m->ctx->sms, s);
  for (int l = 0; l < c.n_layers && e == cudaSuccess; l++) {
    __half *kc = m->kc + l * cache_layer, *vc = m->vc + l * cache_layer;
    if (m->qkv_v[l].N) {
      // q/k and v rows of different block types: the norm once, two products
      if ((e = launch(k_rmsnorm, dim3(1), dim3(1024), s, m->x, m->attn_norm[l], m->h, D, c.eps)) != cudaSuccess ||
          (e = matvec(m, m->qkv[l], m->h, m->qkvb, 0, s)) != cudaSuccess ||
          (e = matvec(m, m->qkv_v[l], m->h, m->qkvb + (size_t)(H + KVH) * hd, 0, s)) != cudaSuccess)
        break;
    } else if ((e = norm_matvec(m, m->qkv[l], m->attn_norm[l], m->qkvb, s)) != cudaSuccess) {
      break;
    }
    const dim3 ag(KVH * m->gsplit, m->nch_max);
    switch (G / m->gsplit) {
#define TCB_ATTN(GG)                                                                                              \
  case GG:                                                                                                        \
    e = launch(k_attn<GG>, ag, dim3(256), s, m->qkvb, m->cosT, m->sinT, m->pos, kc, vc, m->part, m->acount, m->att, H, \
               KVH, m->gsplit, c.max_ctx, m->nch_max, scale, (const BatchSeq *)nullptr, (size_t)0);               \
    break;
      TCB_ATTN(1)
      TCB_ATTN(2)
      TCB_ATTN(4)
      TCB_ATTN(8)
#undef TCB_ATTN
    default: e = cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) break;
    // rank 0 adds its partial to the residual, the others write theirs; the
    // all-reduce then leaves x + sum of partials on every rank
    // NCCL: rank 0 adds its partial to the residual, the others write theirs,
    // and the in-place all-reduce sums x.  Peer: every rank writes its partial
    // to yp and the all-reduce adds the ranks' partials to x.
    float *dst = m->peer ? m->yp : m->x;
    const int acc = m->peer ? 0 : m->tr == 0;
    if ((e = matvec(m, m->o[l], m->att, dst, acc, s)) != cudaSuccess) break;
    if ((e = all_reduce_x(m, s)) != cudaSuccess) break;
    const Mat &gm = m->gu[l];
    if (gm.swi.ok) {
      // the FFN RMSNorm in the prologue and SwiGLU in the epilogue of one launch
      e = tcb::q4k_launch(gm.swi, gm.N, gm.K, gm.w, m->x, TCB_F32, nullptr, TCB_F32, 0, m->ctx->derr, m->sk, s,
                          m->ffn_norm[l], c.eps, gm.pf, gm.pf_bytes, 1, 0, 0, m->a);
    } else if ((e = norm_matvec(m, gm, m->ffn_norm[l], m->gub, s)) == cudaSuccess) {
      e = launch(k_swiglu, dim3((F + 255) / 256), dim3(256), s, m->gub, m->a, F);
    }
    if (e != cudaSuccess) break;
    e = matvec(m, m->down[l], m->a, dst, acc, s);
    if (e != cudaSuccess) break;
    e = all_reduce_x(m, s);
  }
  if (e != cudaSuccess) return e;
  if ((e = launch(k_rmsnorm, dim3(1), dim3(1024), s, m->x, m->final_norm, m->h, D, c.eps)) != cudaSuccess) return e;
  if ((e = matvec(m, m->head, m->h, m->logits, 0, s)) != cudaSuccess) return e;
  if ((e = launch(k_argmax_part, dim3(kArgBlocks), dim3(256), s, m->logits, c.vocab, m->am_v, m->am_i)) != cudaSuccess)
    return e;
  if (m->tp == 1)
    return launch(k_next_token, dim3(1), dim3(32), s, m->am_v, m->am_i, kArgBlocks, m->pos, m->tok, m->hist,
                  m->prompt, m->nprompt, c.max_ctx, (const BatchPick *)nullptr);
  if ((e = launch(k_local_best, dim3(1), dim3(32), s, m->am_v, m->am_i, kArgBlocks, m->vocab_off, m->cand + m->tr)) !=
      cudaSuccess)
    return e;
  const Nccl *nc = nccl();
  if (!nc || !m->comm) return cudaErrorNotReady;
  if ((m->nccl_rc = nc->all_gather(m->cand + m->tr, m->cand, 2, kNcclInt32, m->comm, s)) != 0) return cudaErrorUnknown;
  return launch(k_pick_tp, dim3(1), dim3(32), s, m->cand, m->tp, 1, m->pos, m->tok, m->hist, m->prompt, m->nprompt,
                c.max_ctx, (const BatchPick *)nullptr);
}

}  // namespace

extern "C" {

int tcb_llama_create(tcb_ctx *ctx, const tcb_llama_config *cfg, const tcb_llama_weights *w, tcb_llama **out) {
  if (!ctx || !cfg || !w || !out) return TCB_ERR_NULL;
  *out = nullptr;
  const tcb_llama_config &cg = *cfg;
  const int tp = cg.tp_size > 1 ? cg.tp_size : 1, tr = tp > 1 ? cg.tp_rank : 0;
  if (cg.n_layers < 1 || cg.d_model < 1 || cg.n_heads < 1 || cg.n_kv_heads < 1 || cg.head_dim != tcb::ll::kHd ||
      cg.n_heads % cg.n_kv_heads || cg.ffn_dim < 1 || cg.vocab < 1 || cg.max_ctx < 2 ||
      cg.max_ctx > tcb::ll::kChunk * tcb::ll::kMaxChunks || !(cg.eps > 0.f) ||
      !(cg.rope_theta > 0.f) || tr < 0 || tr >= tp || cg.n_heads % tp || cg.n_kv_heads % tp || cg.ffn_dim % tp ||
      cg.vocab % tp)
    return TCB_ERR_SHAPE;
  // this rank's dimensions
  tcb_llama_config lc = cg;
  lc.n_heads /= tp;
  lc.n_kv_heads /= tp;
  lc.ffn_dim /= tp;
  lc.vocab /= tp;
  const tcb_llama_config &c = lc;
  const int G = c.n_heads / c.n_kv_heads;
  if (G != 1 && G != 2 && G != 4 && G != 8) return TCB_ERR_UNSUPPORTED;
  if (!w->tok_emb || !w->final_norm || !w->head || !w->attn_norm || !w->ffn_norm || !w->qkv || !w->o ||
      !w->gate_up || !w->down)
    return TCB_ERR_NULL;
  if (!wtype_ok(w->tok_emb_type) || !wtype_ok(w->head_type) || !wtype_ok(w->qkv_type) || !wtype_ok(w->o_type) ||
      !wtype_ok(w->gate_up_type) || !wtype_ok(w->down_type))
    return TCB_ERR_DTYPE;
  const int D = c.d_model, H = c.n_heads, KVH = c.n_kv_heads, hd = c.head_dim, F = c.ffn_dim;
  auto kok = [](int type, int K) { return K % tcb::block_elems(type) == 0; };
  if (!kok(w->tok_emb_type, D) || !kok(w->head_type, D) || !kok(w->qkv_type, D) || !kok(w->o_type, H * hd) ||
      !kok(w->gate_up_type, D) || !kok(w->down_type, F))
    return TCB_ERR_SHAPE;
  // the block types of layer l: q/k rows, v rows, o, gate_up, down
  auto ltype = [w](int l, int j) {
    const int cls[5] = {w->qkv_type, w->qkv_type, w->o_type, w->gate_up_type, w->down_type};
    return w->layer_types ? w->layer_types[5 * l + j] : cls[j];
  };
  if (w->layer_types)
    for (int l = 0; l < c.n_layers; l++) {
      for (int j = 0; j < 5; j++)
        if (!wtype_ok(ltype(l, j))) return TCB_ERR_DTYPE;
      if (!kok(ltype(l, 0), D) || !kok(ltype(l, 1), D) || !kok(ltype(l, 2), H * hd) || !kok(ltype(l, 3), D) ||
          !kok(ltype(l, 4), F))
        return TCB_ERR_SHAPE;
    }
  cudaError_t e = cudaSetDevice(ctx->dev);
  if (e != cudaSuccess) return TCB_ERR_CUDA;
  tcb_llama *m = new tcb_llama();
  m->ctx = ctx;
  m->cfg = c;
  m->tp = tp;
  m->tr = tr;
  m->vocab_all = cg.vocab;
  m->vocab_off = tr * c.vocab;
  m->tok_emb = w->tok_emb;
  m->tok_emb_type = w->tok_emb_type;
  m->final_norm = w->final_norm;
  m->head = make_mat(w->head, w->head_type, c.vocab, D, ctx->sms);
  for (int l = 0; l < c.n_layers; l++) {
    if (!w->attn_norm[l] || !w->ffn_norm[l] || !w->qkv[l] || !w->o[l] || !w->gate_up[l] || !w->down[l]) {
      tcb_llama_destroy(m);
      return TCB_ERR_NULL;
    }
    m->attn_norm.push_back(w->attn_norm[l]);
    m->ffn_norm.push_back(w->ffn_norm[l]);
    const int qk_t = ltype(l, 0), v_t = ltype(l, 1), gu_t = ltype(l, 3);
    if (qk_t == v_t) {
      m->qkv.push_back(make_mat(w->qkv[l], qk_t, (H + 2 * KVH) * hd, D, ctx->sms));
      m->qkv_v.push_back(Mat{});
    } else {
      // q and k rows, then the v rows in their own block type
      m->qkv.push_back(make_mat(w->qkv[l], qk_t, (H + KVH) * hd, D, ctx->sms));
      const size_t off = (size_t)(H + KVH) * hd * (D / tcb::block_elems(qk_t)) * tcb::block_bytes(qk_t);
      m->qkv_v.push_back(make_mat(static_cast<const char *>(w->qkv[l]) + off, v_t, KVH * hd, D, ctx->sms));
    }
    m->o.push_back(make_mat(w->o[l], ltype(l, 2), D, H * hd, ctx->sms));
    m->gu.push_back(make_mat(w->gate_up[l], gu_t, 2 * F, D, ctx->sms));
    if (gu_t == TCB_Q4_K && F % 16 == 0)
      m->gu.back().swi = tcb::q4k_plan(2 * F, D, w->gate_up[l], ctx->sms, 1, F);
    m->down.push_back(make_mat(w->down[l], ltype(l, 4), D, F, ctx->sms));
  }
  // Q6_K matrices the TMA kernels cannot map in place: a row-padded copy
  {
    std::vector<Mat *> all{&m->head};
    for (int l = 0; l < c.n_layers; l++)
      for (Mat *mt : {&m->qkv[l], &m->qkv_v[l], &m->o[l], &m->gu[l], &m->down[l]}) all.push_back(mt);
    for (Mat *mt : all) {
      if (!mt->N || mt->plan.ok || mt->type != TCB_Q6_K) continue;
      const long rb = (long)(mt->K / 256) * 210, ldw = (rb + 15) & ~15L;
      uint8_t *wp = nullptr;
      if ((e = alloc(m, &wp, (size_t)mt->N * ldw)) != cudaSuccess ||
          (e = cudaMemset(wp, 0, (size_t)mt->N * ldw)) != cudaSuccess ||
          (e = cudaMemcpy2D(wp, ldw, mt->w, rb, rb, mt->N, cudaMemcpyDeviceToDevice)) != cudaSuccess) {
        tcb_llama_destroy(m);
        return e == cudaErrorMemoryAllocation ? TCB_ERR_NOMEM : TCB_ERR_CUDA;
      }
      const tcb::MvPlan pl = tcb::matvec_plan(mt->type, 0, 1, mt->N, mt->K, wp, ctx->sms, ldw);
      if (pl.ok) {
        mt->wp = wp;
        mt->ldw = ldw;
        mt->plan = pl;
      }
    }
  }
  // each matvec streams the next one's weights into L2 (qkv -> o -> gate_up
  // -> down -> next layer's qkv ... -> head -> layer 0's qkv), at most
  // kPrefetchMax bytes of them, half the L2
  {
    constexpr size_t kPrefetchMax = 64u << 20;
    std::vector<Mat *> chain;
    for (int l = 0; l < c.n_layers; l++) {
      chain.push_back(&m->qkv[l]);
      if (m->qkv_v[l].N) chain.push_back(&m->qkv_v[l]);
      chain.push_back(&m->o[l]);
      chain.push_back(&m->gu[l]);
      chain.push_back(&m->down[l]);
    }
    chain.push_back(&m->head);
    for (size_t i = 0; i < chain.size(); i++) {
      const Mat *nx = chain[(i + 1) % chain.size()];
      chain[i]->pf = nx->wk();
      chain[i]->pf_bytes = nx->kbytes() < kPrefetchMax ? nx->kbytes() : kPrefetchMax;
    }
  }
  size_t sk_bytes = m->head.plan.split_bytes;
  for (int l = 0; l < c.n_layers; l++)
    for (const Mat *mt : {&m->qkv[l], &m->qkv_v[l], &m->o[l], &m->gu[l], &m->down[l]})
      sk_bytes = mt->plan.split_bytes > sk_bytes ? mt->plan.split_bytes : sk_bytes;
  m->nch_max = (c.max_ctx + tcb::ll::kChunk - 1) / tcb::ll::kChunk;
  m->gsplit = attn_split(H / KVH, KVH, m->nch_max, 1, ctx->sms);
  const size_t cache = (size_t)c.n_layers * KVH * c.max_ctx * hd;
  const int qkvn = (H + 2 * KVH) * hd;
  if ((e = alloc(m, &m->x, D)) != cudaSuccess || (e = alloc(m, &m->h, D)) != cudaSuccess ||
      (e = alloc(m, &m->qkvb, qkvn)) != cudaSuccess || (e = alloc(m, &m->att, H * hd)) != cudaSuccess ||
      (e = alloc(m, &m->gub, 2 * (size_t)F)) != cudaSuccess || (e = alloc(m, &m->a, F)) != cudaSuccess ||
      (e = alloc(m, &m->logits, c.vocab)) != cudaSuccess ||
      (e = alloc(m, &m->part, (size_t)H * m->nch_max * (2 + hd))) != cudaSuccess ||
      (e = alloc(m, &m->am_v, tcb::ll::kArgBlocks)) != cudaSuccess ||
      (e = alloc(m, &m->am_i, tcb::ll::kArgBlocks)) != cudaSuccess ||
      (e = alloc(m, &m->cosT, (size_t)c.max_ctx * hd / 2)) != cudaSuccess ||
      (e = alloc(m, &m->sinT, (size_t)c.max_ctx * hd / 2)) != cudaSuccess || (e = alloc(m, &m->kc, cache)) != cudaSuccess ||
      (e = alloc(m, &m->vc, cache)) != cudaSuccess || (e = alloc(m, &m->pos, 1)) != cudaSuccess ||
      (e = alloc(m, &m->nprompt, 1)) != cudaSuccess || (e = alloc(m, &m->tok, 1)) != cudaSuccess ||
      (e = alloc(m, &m->hist, c.max_ctx)) != cudaSuccess || (e = alloc(m, &m->prompt, c.max_ctx)) != cudaSuccess ||
      (e = alloc(m, &m->acount, H)) != cudaSuccess || (e = alloc(m, &m->cand, tp)) != cudaSuccess ||
      (e = alloc(m, reinterpret_cast<char **>(&m->sk), sk_bytes + 256)) != cudaSuccess) {
    tcb_llama_destroy(m);
    return e == cudaErrorMemoryAllocation ? TCB_ERR_NOMEM : TCB_ERR_CUDA;
  }
  // rotary table (TR's rotary_table: theta^(-2i/hd) in double, then float32
  // angles t * f and their cosine / sine)
  const int half = hd / 2;
  std::vector<float> ct((size_t)c.max_ctx * half), st((size_t)c.max_ctx * half);
  for (int i = 0; i < half; i++) {
    const float f = (float)pow((double)c.rope_theta, -2.0 * i / hd);
    for (int t = 0; t < c.max_ctx; t++) {
      const float ang = (float)t * f;
      ct[(size_t)t * half + i] = (float)cos((double)ang);
      st[(size_t)t * half + i] = (float)sin((double)ang);
    }
  }
  if ((e = cudaMemcpy(m->cosT, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(m->sinT, st.data(), st.size() * 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemset(m->kc, 0, cache * 2)) != cudaSuccess || (e = cudaMemset(m->vc, 0, cache * 2)) != cudaSuccess ||
      (e = cudaMemset(m->acount, 0, H * sizeof(unsigned))) != cudaSuccess ||
      (e = cudaMemset(m->sk, 0, sk_bytes + 256)) != cudaSuccess) {
    tcb_llama_destroy(m);
    return TCB_ERR_CUDA;
  }
  *out = m;
  return TCB_OK;
}

int tcb_llama_destroy(tcb_llama *m) {
  if (!m) return TCB_ERR_NULL;
  if (m->exec) cudaGraphExecDestroy(m->exec);
  if (m->graph) cudaGraphDestroy(m->graph);
  if (!m->allocs.empty()) cudaDeviceSynchronize();
  if (m->cap) cudaStreamDestroy(m->cap);
  if (m->comm) nccl()->destroy(m->comm);
  for (void *p : m->opened) cudaIpcCloseMemHandle(p);
  for (void *p : m->allocs) cudaFree(p);
  delete m;
  return TCB_OK;
}

int tcb_llama_start(tcb_llama *m, const int64_t *prompt, int n, void *stream) {
  if (!m || !prompt) return TCB_ERR_NULL;
  if (n < 1 || n > m->cfg.max_ctx) return TCB_ERR_SHAPE;
  for (int i = 0; i < n; i++)
    if (prompt[i] < 0 || prompt[i] >= m->vocab_all) return TCB_ERR_BOUNDS;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int zero = 0;
  cudaError_t e;
  // synchronous copies from pageable host memory: the caller's buffers may
  // go away after the call
  if ((e = cudaSetDevice(m->ctx->dev)) != cudaSuccess || (e = cudaStreamSynchronize(s)) != cudaSuccess ||
      (e = cudaMemcpy(m->prompt, prompt, (size_t)n * 8, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(m->hist, prompt, 8, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(m->tok, prompt, 8, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(m->nprompt, &n, 4, cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(m->pos, &zero, 4, cudaMemcpyHostToDevice)) != cudaSuccess)
    return fail(m, e);
  m->host_pos = 0;
  m->host_n = n;
  return TCB_OK;
}

namespace {
// rows out = W · rms(px) for the prompt pass: the RMSNorm in the tensor-core
// product's activation prologue when that path takes the shape, else a pass
// of its own into ph
int norm_gemm(tcb_llama *m, const Mat &mt, const float *nw, int M, float *out, long ldo, cudaStream_t s) {
  const tcb_llama_config &c = m->cfg;
  tcb::TcPrologue pro;
  pro.kind = tcb::kTcProRms;
  pro.w = nw;
  pro.eps = c.eps;
  int rc = tcb::qgemm_tc_prologue(m->ctx, mt.type, M, mt.N, mt.K, mt.w, m->px, c.d_model, out, ldo, 0, pro, s);
  if (rc != TCB_ERR_UNSUPPORTED) return rc;
  tcb::ll::k_rmsnorm<<<M, 1024, 0, s>>>(m->px, nw, m->ph, c.d_model, c.eps);
  return tcb_qgemm(m->ctx, mt.type, M, mt.N, mt.K, mt.w, m->ph, TCB_F32, mt.K, out, TCB_F32, ldo, 0, s);
}

// One pass of the prompt over the rows of several sequences that share the
// model: sq[i] feeds rows p0 .. p0+rows-1 of engine sq[i].m's prompt.  The
// products run once over all the rows (m0's row buffers); rotary, the cache
// append and attention run per sequence on its own cache.
struct PfSeq {
  tcb_llama *m;
  int p0, rows;
};

int prefill_pass(tcb_llama *m0, const PfSeq *sq, int ns, cudaStream_t s) {
  using namespace tcb::ll;
  const tcb_llama_config &c = m0->cfg;
  const int H = c.n_heads, KVH = c.n_kv_heads, hd = c.head_dim, D = c.d_model, F = c.ffn_dim;
  const int qkvn = (H + 2 * KVH) * hd;
  const size_t cache_layer = (size_t)KVH * c.max_ctx * hd;
  int M = 0;
  for (int i = 0; i < ns; i++) M += sq[i].rows;
  // NCCL: rank 0 adds its partial to the residual rows, the others write
  // theirs, and the in-place all-reduce sums them (as in the decode step)
  const int acc = m0->tr == 0;
  auto reduce = [&]() -> int {
    if (m0->tp == 1) return TCB_OK;
    m0->nccl_rc = nccl()->all_reduce(m0->px, m0->px, (size_t)M * D, kNcclFloat32, kNcclSum, m0->comm, s);
    return m0->nccl_rc ? fail(m0, cudaErrorUnknown) : TCB_OK;
  };
  cudaError_t e;
  for (int i = 0, r = 0; i < ns; r += sq[i].rows, i++)
    if ((e = tcb::launch_dequant_rows(m0->tok_emb_type, m0->tok_emb, sq[i].rows, D, sq[i].m->prompt + sq[i].p0,
                                      m0->px + (size_t)r * D, TCB_F32, m0->ctx->sms, s)) != cudaSuccess)
      return fail(m0, e);
  int rc = TCB_OK;
  for (int l = 0; l < c.n_layers && rc == TCB_OK; l++) {
    const Mat &q = m0->qkv[l], &o = m0->o[l], &gu = m0->gu[l], &dn = m0->down[l];
    if ((rc = norm_gemm(m0, q, m0->attn_norm[l], M, m0->pqkv, qkvn, s)) != TCB_OK) break;
    const Mat &qv = m0->qkv_v[l];
    if (qv.N && (rc = norm_gemm(m0, qv, m0->attn_norm[l], M, m0->pqkv + (size_t)(H + KVH) * hd, qkvn, s)) != TCB_OK)
      break;
    for (int i = 0, r = 0; i < ns; r += sq[i].rows, i++) {
      const tcb_llama *m = sq[i].m;
      __half *kc = m->kc + l * cache_layer, *vc = m->vc + l * cache_layer;
      float *qr = m0->pqkv + (size_t)r * qkvn;
      k_rope_rows<<<sq[i].rows, 256, 0, s>>>(qr, m->cosT, m->sinT, sq[i].p0, kc, vc, H, KVH, c.max_ctx);
      if ((e = tcb::launch_attn_prefill(qr, qkvn, kc, vc, m0->patt + (size_t)r * H * hd, (long)H * hd, sq[i].p0,
                                        sq[i].rows, H, KVH, c.max_ctx, s)) != cudaSuccess)
        return fail(m0, e);
    }
    if ((rc = tcb_qgemm(m0->ctx, o.type, M, o.N, o.K, o.w, m0->patt, TCB_F32, o.K, m0->px, TCB_F32, o.N, acc, s)) !=
            TCB_OK ||
        (rc = reduce()) != TCB_OK)
      break;
    if ((rc = norm_gemm(m0, gu, m0->ffn_norm[l], M, m0->pgu, gu.N, s)) != TCB_OK) break;
    // SwiGLU in the down product's activation prologue, else a pass of its own
    tcb::TcPrologue sw;
    sw.kind = tcb::kTcProSwiglu;
    rc = tcb::qgemm_tc_prologue(m0->ctx, dn.type, M, dn.N, dn.K, dn.w, m0->pgu, 2L * F, m0->px, dn.N, acc, sw, s);
    if (rc == TCB_ERR_UNSUPPORTED) {
      const long na = (long)M * F;
      k_swiglu_rows<<<(int)((na + 255) / 256 < 4096 ? (na + 255) / 256 : 4096), 256, 0, s>>>(m0->pgu, m0->pa, F, na);
      rc = tcb_qgemm(m0->ctx, dn.type, M, dn.N, dn.K, dn.w, m0->pa, TCB_F32, dn.K, m0->px, TCB_F32, dn.N, acc, s);
    }
    if (rc == TCB_OK) rc = reduce();
  }
  if (rc == TCB_OK && (e = cudaGetLastError()) != cudaSuccess) return fail(m0, e);
  return rc;
}

// row buffers of the prompt pass for at least `rows` rows (grown once the
// stream has drained)
int pf_alloc(tcb_llama *m, int rows, cudaStream_t s) {
  if (m->pf_rows >= rows) return TCB_OK;
  const tcb_llama_config &c = m->cfg;
  const int H = c.n_heads, KVH = c.n_kv_heads, hd = c.head_dim, D = c.d_model, F = c.ffn_dim;
  const int qkvn = (H + 2 * KVH) * hd;
  cudaError_t e;
  if (m->pf_rows) {
    if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return fail(m, e);
    for (float *p : {m->px, m->ph, m->pqkv, m->patt, m->pgu, m->pa})
      for (size_t i = 0; i < m->allocs.size(); i++)
        if (m->allocs[i] == p) {
          cudaFree(p);
          m->allocs.erase(m->allocs.begin() + i);
          break;
        }
    m->pf_rows = 0;
  }
  if ((e = alloc(m, &m->px, (size_t)rows * D)) != cudaSuccess || (e = alloc(m, &m->ph, (size_t)rows * D)) != cudaSuccess ||
      (e = alloc(m, &m->pqkv, (size_t)rows * qkvn)) != cudaSuccess ||
      (e = alloc(m, &m->patt, (size_t)rows * H * hd)) != cudaSuccess ||
      (e = alloc(m, &m->pgu, (size_t)rows * 2 * F)) != cudaSuccess || (e = alloc(m, &m->pa, (size_t)rows * F)) != cudaSuccess) {
    (void)cudaGetLastError();
    return e == cudaErrorMemoryAllocation ? TCB_ERR_NOMEM : fail(m, e);
  }
  m->pf_rows = rows;
  return TCB_OK;
}

// the model (weights, shapes, parallelism) of two engines is the same
bool same_model(const tcb_llama *a, const tcb_llama *b) {
  const tcb_llama_config &x = a->cfg, &y = b->cfg;
  if (a->ctx != b->ctx || a->tp != b->tp || a->tr != b->tr || x.n_layers != y.n_layers || x.d_model != y.d_model ||
      x.n_heads != y.n_heads || x.n_kv_heads != y.n_kv_heads || x.head_dim != y.head_dim || x.ffn_dim != y.ffn_dim ||
      x.vocab != y.vocab || x.max_ctx != y.max_ctx || x.eps != y.eps || x.rope_theta != y.rope_theta ||
      a->tok_emb != b->tok_emb || a->tok_emb_type != b->tok_emb_type)
    return false;
  for (int l = 0; l < x.n_layers; l++)
    if (a->attn_norm[l] != b->attn_norm[l] || a->ffn_norm[l] != b->ffn_norm[l] || a->qkv[l].w != b->qkv[l].w ||
        a->o[l].w != b->o[l].w || a->gu[l].w != b->gu[l].w || a->down[l].w != b->down[l].w)
      return false;
  return true;
}

int finish_prefill(tcb_llama *m, cudaStream_t s) {
  const int n = m->host_n;
  tcb::ll::k_prefill_done<<<1, 256, 0, s>>>(m->prompt, n, m->pos, m->tok, m->hist);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(m, e);
  m->host_pos = n - 1;
  return TCB_OK;
}
}  // namespace

int tcb_llama_set_prefill_rows(tcb_llama *m, int rows) {
  if (!m) return TCB_ERR_NULL;
  if (rows < 0) return TCB_ERR_SHAPE;
  m->pf_pass = rows;
  return TCB_OK;
}

int tcb_llama_prefill(tcb_llama *m, void *stream) {
  if (!m) return TCB_ERR_NULL;
  const int n = m->host_n;
  if (n < 1 || m->host_pos != 0) return TCB_ERR_UNSUPPORTED;
  if (n == 1) return TCB_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSetDevice(m->ctx->dev);
  if (e != cudaSuccess) return fail(m, e);
  if (m->tp > 1 && (!nccl() || !m->comm)) return fail(m, cudaErrorNotReady);
  int rows = m->pf_pass > 0 ? m->pf_pass : tcb::ll::kPrefillRows;
  if (rows > n - 1) rows = n - 1;
  int rc = m->pf_rows >= rows ? TCB_OK : pf_alloc(m, rows, s);
  for (int p0 = 0; p0 < n - 1 && rc == TCB_OK; p0 += rows) {
    const PfSeq one{m, p0, n - 1 - p0 < rows ? n - 1 - p0 : rows};
    rc = prefill_pass(m, &one, 1, s);
  }
  return rc == TCB_OK ? finish_prefill(m, s) : rc;
}

int tcb_llama_prefill_batch(tcb_llama *const *ms, int count, void *stream) {
  if (!ms || count < 1) return TCB_ERR_NULL;
  tcb_llama *m0 = ms[0];
  for (int i = 0; i < count; i++) {
    if (!ms[i]) return TCB_ERR_NULL;
    if (ms[i]->host_n < 1 || ms[i]->host_pos != 0) return TCB_ERR_UNSUPPORTED;
    if (!same_model(m0, ms[i])) return TCB_ERR_SHAPE;
    for (int j = 0; j < i; j++)
      if (ms[j] == ms[i]) return TCB_ERR_UNSUPPORTED;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSetDevice(m0->ctx->dev);
  if (e != cudaSuccess) return fail(m0, e);
  if (m0->tp > 1 && (!nccl() || !m0->comm)) return fail(m0, cudaErrorNotReady);
  std::vector<PfSeq> sq;
  long total = 0;
  for (int i = 0; i < count; i++)
    if (ms[i]->host_n > 1) {
      sq.push_back(PfSeq{ms[i], 0, ms[i]->host_n - 1});
      total += ms[i]->host_n - 1;
    }
  if (total > 0x7FFFFFFFL / 8) return TCB_ERR_SHAPE;
  int rc = TCB_OK;
  if (total > 0 && (rc = pf_alloc(m0, (int)total, s)) == TCB_OK) rc = prefill_pass(m0, sq.data(), (int)sq.size(), s);
  for (int i = 0; i < count && rc == TCB_OK; i++)
    if (ms[i]->host_n > 1) rc = finish_prefill(ms[i], s);
  return rc;
}

int tcb_llama_step(tcb_llama *m, void *stream) {
  if (!m) return TCB_ERR_NULL;
  if (m->host_pos + 1 >= m->cfg.max_ctx) return TCB_ERR_BOUNDS;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = m->exec ? cudaGraphLaunch(m->exec, s) : issue_step(m, s);
  if (e != cudaSuccess) return fail(m, e);
  m->host_pos++;
  return TCB_OK;
}

int tcb_llama_capture(tcb_llama *m, void *stream) {
  if (!m) return TCB_ERR_NULL;
  cudaError_t e = cudaSetDevice(m->ctx->dev);
  if (e == cudaSuccess && !m->cap) e = cudaStreamCreateWithFlags(&m->cap, cudaStreamNonBlocking);
  // the capture stream starts after the caller's work
  if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(m, e);
  cudaStream_t s = m->cap;
  if (m->exec) {
    cudaGraphExecDestroy(m->exec);
    m->exec = nullptr;
  }
  if (m->graph) {
    cudaGraphDestroy(m->graph);
    m->graph = nullptr;
  }
  e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
  if (e != cudaSuccess) return fail(m, e);
  cudaError_t ei = issue_step(m, s);
  cudaGraph_t g = nullptr;
  e = cudaStreamEndCapture(s, &g);
  if (ei != cudaSuccess || e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return fail(m, ei != cudaSuccess ? ei : e);
  }
  m->graph = g;
  if ((e = cudaGraphInstantiate(&m->exec, g, 0)) != cudaSuccess) {
    m->exec = nullptr;
    return fail(m, e);
  }
  return TCB_OK;
}

// ----------------------------------------------------------------- batch

// A batch of sequences decoded together (tcb_llama_batch_*): engines made from
// the same weights, each with its own K/V cache, position and token history.
// A step runs every product once over the batch's rows, attention per
// sequence in one launch (blockIdx.z), and each sequence's greedy pick.
// how a batch step runs one product over its B rows (fixed at creation)
struct BatchMat {
  int how = 0;  // 0: multi-row matvec launches, 1: tensor cores, 2: a matvec launch per row, 3: portable kernel,
                // 4: the Q4_K kernel of up to 16 rows (row groups of plan.rows)
  tcb::MvPlan plan{};
};

struct tcb_llama_batch {
  std::vector<tcb_llama *> ms;
  tcb_llama *m0 = nullptr;
  int B = 0;
  // the products' launch plans and the scratch they use: owned here, so a
  // captured step never refers to the context's workspace, which later calls
  // may grow (and so move)
  std::vector<BatchMat> qkv_, qkv_v, o, gu_, down;
  BatchMat head;
  void *ws = nullptr, *sk = nullptr;
  float *x = nullptr, *h = nullptr, *qkv = nullptr, *att = nullptr, *gu = nullptr, *a = nullptr, *logits = nullptr;
  float *yp = nullptr;  // tensor parallelism over peer memory: this rank's o / down partial rows
  float *part = nullptr, *am_v = nullptr;
  int *am_i = nullptr;
  unsigned *count = nullptr;
  int gsplit = 1;  // attention CTAs per KV head
  int64_t *tok = nullptr;
  tcb::ll::BatchSeq *seq = nullptr;
  tcb::ll::BatchPick *pick = nullptr;
  int2 *cand = nullptr;
  std::vector<void *> allocs;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaStream_t cap = nullptr;
};

namespace {

cudaError_t balloc_bytes(tcb_llama_batch *b, void **p, size_t bytes) {
  void *q = nullptr;
  cudaError_t e = cudaMalloc(&q, bytes + 16);
  if (e == cudaSuccess) {
    b->allocs.push_back(q);
    *p = q;
  }
  return e;
}
#define balloc(b, pp, n) balloc_bytes((b), reinterpret_cast<void **>(pp), (n) * sizeof(**(pp)))

// How B rows of a product run.  From kBatchTcRows rows on, the tensor cores
// take the product when the shape allows it with a workspace under 1 GiB:
// the weights stream once for all rows (fp16 operands, about 2e-4 relative
// L2).  Below that, tcb_qgemm's routing for few rows: up to 8 rows of x per
// matvec launch (the weights streamed once per launch); shapes the
// multi-row matvec kernels do not take (long Q6_K rows, the wide head) on
// the tensor cores as above, else one matvec launch per row.  ws / sk: the
// workspace and matvec scratch this product needs.
constexpr int kBatchTcRows = 16;
BatchMat batch_mat(const tcb_llama *m0, const Mat &mt, int B, size_t &ws, size_t &sk) {
  BatchMat bm;
  const int sms = m0->ctx->sms;
  // Q4_K / Q6_K with up to 16 rows: one weight stream for all rows, integer scale
  // math (faster than the tensor-core product, whose weight dequant is
  // amortised over 16 of the 256 rows it is built for)
  if ((mt.type == TCB_Q4_K || mt.type == TCB_Q6_K || mt.type == TCB_Q4_0) && B >= 2 && B <= 16) {
    // groups of fewer rows when the digits of 16 leave too little shared memory
    for (int r = B; r >= 2 && !bm.plan.ok; r = (r + 1) / 2 == r ? 1 : (r + 1) / 2)
      bm.plan = tcb::rows_plan(mt.type, mt.N, mt.K, mt.w, sms, r);
    if (bm.plan.ok) {
      bm.how = 4;
      if (bm.plan.split_bytes > sk) sk = bm.plan.split_bytes;
      return bm;
    }
  }
  const bool tc = B > 1 && tcb::tc_eligible_rows(mt.type, mt.N, mt.K, mt.w) &&
                  tcb::tc_workspace_bytes(mt.type, B, mt.N, mt.K) <= ((size_t)1 << 30);
  if (B > 1 && !(tc && B >= kBatchTcRows))
    for (int mr = 8; mr >= 2 && !bm.plan.ok; mr /= 2)
      if (mr <= 2 * B - 1 || mr == 2) bm.plan = tcb::matvec_plan_rows(mt.type, 0, mt.N, mt.K, mt.wk(), sms, mr, mt.ldw);
  if (bm.plan.ok) {
    bm.how = 0;
  } else if (tc) {
    bm.how = 1;
    const size_t w = tcb::tc_workspace_bytes(mt.type, B, mt.N, mt.K);
    ws = w > ws ? w : ws;
  } else {
    bm.plan = tcb::matvec_plan(mt.type, 0, 1, mt.N, mt.K, mt.wk(), sms, mt.ldw);
    bm.how = bm.plan.ok ? 2 : 3;
  }
  if (bm.plan.ok && bm.plan.split_bytes > sk) sk = bm.plan.split_bytes;
  return bm;
}

// rows y (+)= W x_rows for the batch's B rows
// ldy: the row stride of y (0: mt.N)
int rows_product(tcb_llama_batch *bt, const Mat &mt, const BatchMat &bm, const float *x, float *y, int acc,
                 cudaStream_t s, long ldy = 0) {
  tcb_llama *m0 = bt->m0;
  if (ldy == 0) ldy = mt.N;
  const int B = bt->B;
  cudaError_t e = cudaSuccess;
  switch (bm.how) {
  case 0:
    for (int r0 = 0; r0 < B && e == cudaSuccess; r0 += bm.plan.rows) {
      const int rows = B - r0 < bm.plan.rows ? B - r0 : bm.plan.rows;
      e = tcb::matvec_launch(bm.plan, mt.type, 0, mt.N, mt.K, mt.wk(), x + (size_t)r0 * mt.K, TCB_F32,
                             y + (size_t)r0 * ldy, TCB_F32, acc, m0->ctx->derr, s, nullptr, 0, bt->sk, rows, mt.K,
                             ldy);
    }
    break;
  case 4:
    for (int r0 = 0; r0 < B && e == cudaSuccess; r0 += bm.plan.rows) {
      const int rows = B - r0 < bm.plan.rows ? B - r0 : bm.plan.rows;
      e = tcb::rows_launch(bm.plan, mt.N, mt.K, mt.w, x + (size_t)r0 * mt.K, TCB_F32, mt.K, y + (size_t)r0 * ldy,
                           TCB_F32, ldy, acc, rows, m0->ctx->derr, bt->sk, s);
    }
    break;
  case 1:
    e = tcb::launch_qgemm_tc(mt.type, mt.w, B, mt.N, mt.K, x, TCB_F32, mt.K, y, TCB_F32, ldy, acc, bt->ws,
                             m0->ctx->derr, s, nullptr);
    break;
  case 2:
    for (int r = 0; r < B && e == cudaSuccess; r++)
      e = tcb::matvec_launch(bm.plan, mt.type, 0, mt.N, mt.K, mt.wk(), x + (size_t)r * mt.K, TCB_F32, y + (size_t)r * ldy,
                             TCB_F32, acc, m0->ctx->derr, s, nullptr, 0, bt->sk);
    break;
  default:
    e = tcb::launch_qgemm_simt(mt.type, mt.w, B, mt.N, mt.K, x, TCB_F32, mt.K, y, TCB_F32, ldy, acc, m0->ctx->sms, s);
  }
  return e == cudaSuccess ? TCB_OK : fail(m0, e);
}

int issue_batch_step(tcb_llama_batch *bt, cudaStream_t s) {
  using namespace tcb::ll;
  tcb_llama *m0 = bt->m0;
  const tcb_llama_config &c = m0->cfg;
  const int H = c.n_heads, KVH = c.n_kv_heads, hd = c.head_dim, D = c.d_model, F = c.ffn_dim, B = bt->B;
  const int G = H / KVH, V = c.vocab, qkvn = (H + 2 * KVH) * hd;
  const float scale = 1.0f / sqrtf((float)hd);
  const size_t cache_layer = (size_t)KVH * c.max_ctx * hd;
  // NCCL: rank 0 adds its o/down partial to the residual rows, the others
  // write theirs, and the in-place all-reduce of B rows sums them
  // NCCL: rank 0 adds its partial to the residual rows, the others write
  // theirs, and the in-place all-reduce sums them.  Peer memory (up to
  // kPeerRows sequences): every rank writes its partial rows to yp and the
  // peer all-reduce adds the ranks' partials to the residual rows.
  const bool peer = bt->yp != nullptr;
  const int acc = peer ? 0 : m0->tr == 0;
  float *dst = peer ? bt->yp : bt->x;
  auto reduce = [&]() -> int {
    if (m0->tp == 1) return TCB_OK;
    if (peer) {
      const int nb = kArBlocks * B < 4 * m0->ctx->sms ? kArBlocks * B : 4 * m0->ctx->sms;
      cudaError_t le = launch(k_peer_ar, dim3(nb), dim3(kArThreads), s, m0->pb, (const float *)bt->yp, bt->x, B * D,
                              (long)kPeerRows * D, m0->tp, m0->tr, m0->ar_epoch, m0->ar_done, m0->ctx->derr, kArPolls);
      return le == cudaSuccess ? TCB_OK : fail(m0, le);
    }
    m0->nccl_rc = nccl()->all_reduce(bt->x, bt->x, (size_t)B * D, kNcclFloat32, kNcclSum, m0->comm, s);
    return m0->nccl_rc ? fail(m0, cudaErrorUnknown) : TCB_OK;
  };
  // plain launches first: the step starts after the previous one has
  // completed (k_attn reads the cached K/V and positions before its wait)
  k_gather_tok<<<(B + 31) / 32, 32, 0, s>>>(bt->seq, B, bt->tok);
  cudaError_t e = tcb::launch_dequant_rows(m0->tok_emb_type, m0->tok_emb, B, D, bt->tok, bt->x, TCB_F32,
                                           m0->ctx->sms, s);
  if (e != cudaSuccess) return fail(m0, e);
  int rc = TCB_OK;
  for (int l = 0; l < c.n_layers && rc == TCB_OK; l++) {
    k_rmsnorm<<<B, 1024, 0, s>>>(bt->x, m0->attn_norm[l], bt->h, D, c.eps);
    if ((rc = rows_product(bt, m0->qkv[l], bt->qkv_[l], bt->h, bt->qkv, 0, s, qkvn)) != TCB_OK) break;
    if (m0->qkv_v[l].N && (rc = rows_product(bt, m0->qkv_v[l], bt->qkv_v[l], bt->h, bt->qkv + (size_t)(H + KVH) * hd,
                                             0, s, qkvn)) != TCB_OK)
      break;
    const dim3 ag(KVH * bt->gsplit, m0->nch_max, B);
    switch (G / bt->gsplit) {
#define TCB_ATTN(GG)                                                                                              \
  case GG:                                                                                                        \
    e = launch(k_attn<GG>, ag, dim3(256), s, (const float *)bt->qkv, (const float *)m0->cosT,                    \
               (const float *)m0->sinT, (const int *)nullptr, (__half *)nullptr, (__half *)nullptr, bt->part,    \
               bt->count, bt->att, H, KVH, bt->gsplit, c.max_ctx, m0->nch_max, scale,                            \
               (const BatchSeq *)bt->seq, (size_t)l * cache_layer);                                              \
    break;
      TCB_ATTN(1)
      TCB_ATTN(2)
      TCB_ATTN(4)
      TCB_ATTN(8)
#undef TCB_ATTN
    default: e = cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return fail(m0, e);
    if ((rc = rows_product(bt, m0->o[l], bt->o[l], bt->att, dst, acc, s)) != TCB_OK || (rc = reduce()) != TCB_OK)
      break;
    k_rmsnorm<<<B, 1024, 0, s>>>(bt->x, m0->ffn_norm[l], bt->h, D, c.eps);
    if ((rc = rows_product(bt, m0->gu[l], bt->gu_[l], bt->h, bt->gu, 0, s)) != TCB_OK) break;
    const long na = (long)B * F;
    k_swiglu_rows<<<(int)((na + 255) / 256 < 4096 ? (na + 255) / 256 : 4096), 256, 0, s>>>(bt->gu, bt->a, F, na);
    if ((rc = rows_product(bt, m0->down[l], bt->down[l], bt->a, dst, acc, s)) != TCB_OK ||
        (rc = reduce()) != TCB_OK)
      break;
  }
  if (rc != TCB_OK) return rc;
  k_rmsnorm<<<B, 1024, 0, s>>>(bt->x, m0->final_norm, bt->h, D, c.eps);
  if ((rc = rows_product(bt, m0->head, bt->head, bt->h, bt->logits, 0, s)) != TCB_OK) return rc;
  // every sequence's pick in one launch per stage (blockIdx: the sequence)
  if ((e = launch(k_argmax_part, dim3(kArgBlocks, B), dim3(256), s, (const float *)bt->logits, V, bt->am_v,
                  bt->am_i)) != cudaSuccess)
    return fail(m0, e);
  if (m0->tp == 1) {
    if ((e = launch(k_next_token, dim3(B), dim3(32), s, (const float *)bt->am_v, (const int *)bt->am_i, kArgBlocks,
                    (int *)nullptr, (int64_t *)nullptr, (int64_t *)nullptr, (const int64_t *)nullptr,
                    (const int *)nullptr, c.max_ctx, (const BatchPick *)bt->pick)) != cudaSuccess)
      return fail(m0, e);
    return TCB_OK;
  }
  // tensor parallelism: each rank's candidate per sequence ([rank][B]), one
  // all-gather, then each sequence's pick over the ranks
  if ((e = launch(k_local_best, dim3(B), dim3(32), s, (const float *)bt->am_v, (const int *)bt->am_i, kArgBlocks,
                  m0->vocab_off, bt->cand + (size_t)m0->tr * B)) != cudaSuccess)
    return fail(m0, e);
  if ((m0->nccl_rc = nccl()->all_gather(bt->cand + (size_t)m0->tr * B, bt->cand, 2 * (size_t)B, kNcclInt32, m0->comm,
                                        s)) != 0)
    return fail(m0, cudaErrorUnknown);
  if ((e = launch(k_pick_tp, dim3(B), dim3(32), s, (const int2 *)bt->cand, m0->tp, B, (int *)nullptr,
                  (int64_t *)nullptr, (int64_t *)nullptr, (const int64_t *)nullptr, (const int *)nullptr, c.max_ctx,
                  (const BatchPick *)bt->pick)) != cudaSuccess)
    return fail(m0, e);
  return TCB_OK;
}

}  // namespace

int tcb_llama_batch_destroy(tcb_llama_batch *bt) {
  if (!bt) return TCB_OK;
  if (bt->m0) cudaSetDevice(bt->m0->ctx->dev);
  if (bt->exec) cudaGraphExecDestroy(bt->exec);
  if (bt->graph) cudaGraphDestroy(bt->graph);
  if (bt->cap) cudaStreamDestroy(bt->cap);
  for (void *p : bt->allocs) cudaFree(p);
  delete bt;
  return TCB_OK;
}

int tcb_llama_batch_create(tcb_llama *const *ms, int count, tcb_llama_batch **out) {
  if (!ms || !out) return TCB_ERR_NULL;
  *out = nullptr;
  if (count < 1 || count > TCB_LLAMA_MAX_BATCH) return TCB_ERR_SHAPE;
  tcb_llama *m0 = ms[0];
  for (int i = 0; i < count; i++) {
    if (!ms[i]) return TCB_ERR_NULL;
    if (!same_model(m0, ms[i])) return TCB_ERR_SHAPE;
    for (int j = 0; j < i; j++)
      if (ms[j] == ms[i]) return TCB_ERR_UNSUPPORTED;
  }
  const tcb_llama_config &c = m0->cfg;
  if (c.head_dim != tcb::ll::kHd) return TCB_ERR_UNSUPPORTED;
  cudaError_t e = cudaSetDevice(m0->ctx->dev);
  if (e != cudaSuccess) return fail(m0, e);
  tcb_llama_batch *bt = new (std::nothrow) tcb_llama_batch;
  if (!bt) return TCB_ERR_NOMEM;
  bt->ms.assign(ms, ms + count);
  bt->m0 = m0;
  bt->B = count;
  const int H = c.n_heads, KVH = c.n_kv_heads, hd = c.head_dim, D = c.d_model, F = c.ffn_dim, B = count;
  const size_t qkvn = (size_t)(H + 2 * KVH) * hd;
  bt->gsplit = attn_split(H / KVH, KVH, m0->nch_max, B, m0->ctx->sms);
  std::vector<tcb::ll::BatchSeq> hs(B);
  for (int i = 0; i < B; i++) hs[i] = tcb::ll::BatchSeq{ms[i]->pos, ms[i]->kc, ms[i]->vc, ms[i]->tok};
  std::vector<tcb::ll::BatchPick> hp(B);
  for (int i = 0; i < B; i++)
    hp[i] = tcb::ll::BatchPick{ms[i]->pos, ms[i]->tok, ms[i]->hist, ms[i]->prompt, ms[i]->nprompt};
  if ((e = balloc(bt, &bt->x, (size_t)B * D)) != cudaSuccess || (e = balloc(bt, &bt->h, (size_t)B * D)) != cudaSuccess ||
      (e = balloc(bt, &bt->qkv, (size_t)B * qkvn)) != cudaSuccess ||
      (e = balloc(bt, &bt->att, (size_t)B * H * hd)) != cudaSuccess ||
      (e = balloc(bt, &bt->gu, (size_t)B * 2 * F)) != cudaSuccess || (e = balloc(bt, &bt->a, (size_t)B * F)) != cudaSuccess ||
      (e = balloc(bt, &bt->logits, (size_t)B * c.vocab)) != cudaSuccess ||
      (e = balloc(bt, &bt->part, (size_t)B * H * m0->nch_max * (2 + hd))) != cudaSuccess ||
      (e = balloc(bt, &bt->am_v, (size_t)B * tcb::ll::kArgBlocks)) != cudaSuccess ||
      (e = balloc(bt, &bt->am_i, (size_t)B * tcb::ll::kArgBlocks)) != cudaSuccess ||
      (e = balloc(bt, &bt->count, (size_t)B * H)) != cudaSuccess || (e = balloc(bt, &bt->tok, (size_t)B)) != cudaSuccess ||
      (e = balloc(bt, &bt->seq, (size_t)B)) != cudaSuccess || (e = balloc(bt, &bt->pick, (size_t)B)) != cudaSuccess ||
      (e = balloc(bt, &bt->cand, (size_t)B * m0->tp)) != cudaSuccess ||
      (e = cudaMemset(bt->count, 0, (size_t)B * H * sizeof(unsigned))) != cudaSuccess ||
      (e = cudaMemcpy(bt->seq, hs.data(), B * sizeof(tcb::ll::BatchSeq), cudaMemcpyHostToDevice)) != cudaSuccess ||
      (e = cudaMemcpy(bt->pick, hp.data(), B * sizeof(tcb::ll::BatchPick), cudaMemcpyHostToDevice)) != cudaSuccess ||
      // the residual rows' sums over peer memory when every row fits a slot
      (m0->peer && B <= tcb::ll::kPeerRows && (e = balloc(bt, &bt->yp, (size_t)B * D)) != cudaSuccess)) {
    tcb_llama_batch_destroy(bt);
    return e == cudaErrorMemoryAllocation ? TCB_ERR_NOMEM : fail(m0, e);
  }
  size_t ws = 0, sk = 0;
  for (int l = 0; l < c.n_layers; l++) {
    bt->qkv_.push_back(batch_mat(m0, m0->qkv[l], B, ws, sk));
    bt->qkv_v.push_back(m0->qkv_v[l].N ? batch_mat(m0, m0->qkv_v[l], B, ws, sk) : BatchMat{});
    bt->o.push_back(batch_mat(m0, m0->o[l], B, ws, sk));
    bt->gu_.push_back(batch_mat(m0, m0->gu[l], B, ws, sk));
    bt->down.push_back(batch_mat(m0, m0->down[l], B, ws, sk));
  }
  bt->head = batch_mat(m0, m0->head, B, ws, sk);
  if ((ws && (e = balloc_bytes(bt, &bt->ws, ws)) != cudaSuccess) ||
      (e = balloc_bytes(bt, &bt->sk, sk + tcb::kScratchCntBytes)) != cudaSuccess ||
      (e = cudaMemset(bt->sk, 0, sk + tcb::kScratchCntBytes)) != cudaSuccess) {
    tcb_llama_batch_destroy(bt);
    return e == cudaErrorMemoryAllocation ? TCB_ERR_NOMEM : fail(m0, e);
  }
  *out = bt;
  return TCB_OK;
}

int tcb_llama_batch_step(tcb_llama_batch *bt, void *stream) {
  if (!bt) return TCB_ERR_NULL;
  tcb_llama *m0 = bt->m0;
  for (tcb_llama *m : bt->ms)
    if (m->host_n < 1 || m->host_pos + 1 >= m->cfg.max_ctx) return TCB_ERR_BOUNDS;
  if (m0->tp > 1 && (!nccl() || !m0->comm)) return fail(m0, cudaErrorNotReady);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSetDevice(m0->ctx->dev);
  if (e != cudaSuccess) return fail(m0, e);
  int rc = TCB_OK;
  if (bt->exec) {
    if ((e = cudaGraphLaunch(bt->exec, s)) != cudaSuccess) return fail(m0, e);
  } else if ((rc = issue_batch_step(bt, s)) != TCB_OK) {
    return rc;
  }
  for (tcb_llama *m : bt->ms) m->host_pos++;
  return TCB_OK;
}

int tcb_llama_batch_capture(tcb_llama_batch *bt, void *stream) {
  if (!bt) return TCB_ERR_NULL;
  tcb_llama *m0 = bt->m0;
  if (m0->tp > 1 && (!nccl() || !m0->comm)) return fail(m0, cudaErrorNotReady);
  cudaError_t e = cudaSetDevice(m0->ctx->dev);
  if (e == cudaSuccess && !bt->cap) e = cudaStreamCreateWithFlags(&bt->cap, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(m0, e);
  if (bt->exec) {
    cudaGraphExecDestroy(bt->exec);
    bt->exec = nullptr;
  }
  if (bt->graph) {
    cudaGraphDestroy(bt->graph);
    bt->graph = nullptr;
  }
  if ((e = cudaStreamBeginCapture(bt->cap, cudaStreamCaptureModeThreadLocal)) != cudaSuccess) return fail(m0, e);
  const int rc = issue_batch_step(bt, bt->cap);
  cudaGraph_t g = nullptr;
  e = cudaStreamEndCapture(bt->cap, &g);
  if (rc != TCB_OK || e != cudaSuccess) {
    if (g) cudaGraphDestroy(g);
    return rc != TCB_OK ? rc : fail(m0, e);
  }
  bt->graph = g;
  if ((e = cudaGraphInstantiate(&bt->exec, g, 0)) != cudaSuccess) {
    bt->exec = nullptr;
    return fail(m0, e);
  }
  return TCB_OK;
}

int tcb_llama_batch_logits(tcb_llama_batch *bt, float **logits) {
  if (!bt || !logits) return TCB_ERR_NULL;
  *logits = bt->logits;
  return TCB_OK;
}

int tcb_nccl_unique_id(unsigned char *id128) {
  if (!id128) return TCB_ERR_NULL;
  const Nccl *nc = nccl();
  if (!nc) return TCB_ERR_UNSUPPORTED;
  NcclId id;
  if (nc->get_id(&id) != 0) return TCB_ERR_CUDA;
  memcpy(id128, id.internal, sizeof id.internal);
  return TCB_OK;
}

int tcb_llama_tp_init(tcb_llama *m, const unsigned char *id128) {
  if (!m || !id128) return TCB_ERR_NULL;
  if (m->tp == 1) return TCB_OK;
  const Nccl *nc = nccl();
  if (!nc) return TCB_ERR_UNSUPPORTED;
  if (m->comm) return TCB_OK;
  if (cudaSetDevice(m->ctx->dev) != cudaSuccess) return TCB_ERR_CUDA;
  NcclId id;
  memcpy(id.internal, id128, sizeof id.internal);
  const int rc = nc->init_rank(&m->comm, m->tp, id, m->tr);
  if (rc != 0) {
    snprintf(m->ctx->err, sizeof m->ctx->err, "NCCL: %s", nc->err(rc));
    m->comm = nullptr;
    return TCB_ERR_CUDA;
  }
  return TCB_OK;
}

int tcb_llama_peer_handle(tcb_llama *m, unsigned char *handle64) {
  if (!m || !handle64) return TCB_ERR_NULL;
  memset(handle64, 0, 64);
  if (m->tp == 1) return TCB_OK;
  if (m->tp > tcb::ll::kMaxTp || m->cfg.d_model % 4) return TCB_ERR_UNSUPPORTED;
  cudaError_t e = cudaSetDevice(m->ctx->dev);
  if (e == cudaSuccess && !m->xbuf) {
    m->xbuf_bytes = (size_t)2 * m->tp * tcb::ll::kPeerRows * m->cfg.d_model * 8;
    if ((e = alloc(m, &m->xbuf, m->xbuf_bytes)) == cudaSuccess && (e = cudaMemset(m->xbuf, 0, m->xbuf_bytes)) == cudaSuccess &&
        (e = alloc(m, &m->yp, (size_t)m->cfg.d_model)) == cudaSuccess && (e = alloc(m, &m->ar_epoch, 2)) == cudaSuccess)
      e = cudaMemset(m->ar_epoch, 0, 2 * sizeof(unsigned));
    m->ar_done = m->ar_epoch + 1;
  }
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, m->xbuf);
  if (e != cudaSuccess) return fail(m, e);
  memcpy(handle64, &h, 64);
  return TCB_OK;
}

int tcb_llama_peer_init(tcb_llama *m, const unsigned char *handles) {
  if (!m || !handles) return TCB_ERR_NULL;
  if (m->tp == 1) return TCB_OK;
  if (!m->xbuf) {  // tcb_llama_peer_handle makes the buffer first
    snprintf(m->ctx->err, sizeof m->ctx->err, "tcb_llama_peer_init before tcb_llama_peer_handle");
    return TCB_ERR_UNSUPPORTED;
  }
  if (m->peer) return TCB_OK;
  cudaError_t e = cudaSetDevice(m->ctx->dev);
  for (int r = 0; r < m->tp && e == cudaSuccess; r++) {
    char *base = m->xbuf;
    if (r != m->tr) {
      cudaIpcMemHandle_t h;
      memcpy(&h, handles + 64 * r, 64);
      void *p = nullptr;
      if ((e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess)) != cudaSuccess) break;
      m->opened.push_back(p);
      base = static_cast<char *>(p);
    }
    m->pb.slot[r] = reinterpret_cast<unsigned long long *>(base);
  }
  if (e != cudaSuccess) {
    for (void *p : m->opened) cudaIpcCloseMemHandle(p);
    m->opened.clear();
    return fail(m, e);
  }
  m->peer = true;
  return TCB_OK;
}

int tcb_peer_ar_selftest(tcb_ctx *ctx, int tp, int rank, int d_model, unsigned polls, void *stream) {
  using namespace tcb::ll;
  if (!ctx) return TCB_ERR_NULL;
  if (tp < 1 || tp > kMaxTp || rank < 0 || rank >= tp || d_model <= 0 || d_model % 4 || polls == 0)
    return TCB_ERR_UNSUPPORTED;
  auto cuda_fail = [ctx](cudaError_t err) {
    snprintf(ctx->err, sizeof ctx->err, "%s: %s", cudaGetErrorName(err), cudaGetErrorString(err));
    return TCB_ERR_CUDA;
  };
  cudaError_t e = cudaSetDevice(ctx->dev);
  if (e != cudaSuccess) return cuda_fail(e);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // every rank's exchange buffer local to this device; nothing but this
  // call writes them, so the other ranks' values never arrive
  const size_t bytes = (size_t)2 * tp * d_model * 8;
  char *buf = nullptr;
  float *vec = nullptr;
  unsigned *cnt = nullptr;
  PeerBufs pb{};
  if ((e = cudaMalloc(&buf, bytes * tp)) == cudaSuccess && (e = cudaMalloc(&vec, (size_t)2 * d_model * 4)) == cudaSuccess &&
      (e = cudaMalloc(&cnt, 2 * sizeof(unsigned))) == cudaSuccess && (e = cudaMemsetAsync(buf, 0, bytes * tp, s)) == cudaSuccess &&
      (e = cudaMemsetAsync(vec, 0, (size_t)2 * d_model * 4, s)) == cudaSuccess &&
      (e = cudaMemsetAsync(cnt, 0, 2 * sizeof(unsigned), s)) == cudaSuccess) {
    for (int r = 0; r < tp; r++) pb.slot[r] = reinterpret_cast<unsigned long long *>(buf + bytes * r);
    e = launch(k_peer_ar, dim3(kArBlocks), dim3(kArThreads), s, pb, (const float *)vec, vec + d_model, d_model,
               (long)d_model, tp, rank,
               cnt, cnt + 1, ctx->derr, polls);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  }
  cudaFree(buf);
  cudaFree(vec);
  cudaFree(cnt);
  return e == cudaSuccess ? TCB_OK : cuda_fail(e);
}

int tcb_llama_step_kernels(tcb_llama *m, int *kernels) {
  if (!m || !kernels) return TCB_ERR_NULL;
  *kernels = 0;
  if (!m->graph) return TCB_ERR_UNSUPPORTED;
  size_t n = 0;
  cudaError_t e = cudaGraphGetNodes(m->graph, nullptr, &n);
  std::vector<cudaGraphNode_t> nodes(n);
  if (e == cudaSuccess && n) e = cudaGraphGetNodes(m->graph, nodes.data(), &n);
  for (size_t i = 0; i < n && e == cudaSuccess; i++) {
    cudaGraphNodeType t;
    if ((e = cudaGraphNodeGetType(nodes[i], &t)) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++*kernels;
  }
  return e == cudaSuccess ? TCB_OK : fail(m, e);
}

int tcb_llama_buffers(tcb_llama *m, int64_t **tokens, float **logits) {
  if (!m || !tokens || !logits) return TCB_ERR_NULL;
  *tokens = m->hist;
  *logits = m->logits;
  return TCB_OK;
}

}  // extern "C"
