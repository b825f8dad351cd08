/*
 * tcb_oracle.h - CPU restatement of TR's quantized-weight matvec path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the shipped library links this code;
 * it is the checker that tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg compare the CUDA path against.
 *
 * Parity is pinned: tests/test_oracle.py checks tcbo_dequant against
 * the golden FNV-1a hashes of TR's TestDequantMatchesLlamaCpp
 * (internal/compute/tensor/quant_test.go:55-87) and the hand-computed blocks
 * of TestDequantKnownValues (quant_test.go:89-137).  The int8-activation
 * path has no stored reference outputs in TR (its tests are equalities
 * between TR's own Go and AVX2 kernels), so its absolute results are
 * restated line by line from cpu_quant_q8.go and cross-checked by the
 * relational properties those tests assert.
 *
 * Format codes are GGUF tensor type ids (internal/compute/gguf/types.go:12-16).
 */
#ifndef TCB_ORACLE_H
#define TCB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { TCBO_Q4_0 = 2, TCBO_Q8_0 = 8, TCBO_Q4_K = 12, TCBO_Q6_K = 14 };

/* elements and bytes per block (tensor/quant.go:23-47); 0 for unknown */
int tcbo_block_elems(int fmt);
int tcbo_block_bytes(int fmt);

/* IEEE half -> float, NaN payload kept (tensor/cpu_dtype.go:126-145) */
float tcbo_f16_to_f32(uint16_t h);

/* dequantize nblocks consecutive blocks (tensor/quant.go:139-221), with the
 * x86 NaN rule of gpu/kernel_quant.go:13-17 made explicit */
void tcbo_dequant(int fmt, const uint8_t *raw, size_t nblocks, float *y);

/* TR's dotF32 order: AVX2 sdot32 over the 32-multiple prefix
 * (tensor/cpu_gemv_amd64.s:65-106), scalar dot32 for the rest
 * (tensor/cpu_gemv.go:66-85) */
float tcbo_dot_f32(const float *x, const float *y, size_t n);

/* float path, one weight row: x . dequant(w) in dotF32 order
 * (tensor/cpu_quant.go:38-44; cpu_quant_amd64.go:284-297) */
float tcbo_quant_dot(int fmt, const float *x, const uint8_t *wrow, int K);

/* float path: c[m,n] += sum_k a[m,k] dequant(w)[n,k]
 * (tensor/cpu_quant.go:47-160).  Rows m are computed with the one-row
 * quantDot order (TR's M>1 path is its SGEMM microkernel order; the two
 * differ by reassociation only). nthreads<=1 runs serially. */
void tcbo_qgemm_float(int fmt, int M, int N, int K, const float *a,
                      const uint8_t *w, float *c, int nthreads);

/* activation quantisation (tensor/cpu_quant_q8.go:39-68); blk = 32 or 256.
 * q: K int8, d: K/blk floats, bs: K/16 int16 */
void tcbo_quantize_q8(const float *x, int K, int blk, int8_t *q, float *d,
                      int16_t *bs);

/* quantised-activation dot for one weight row (cpu_quant_q8.go:74-116,
 * :378-407; Q8_0 x Q8 follows dotQ4Q8Go's fold, TR has no Q8_0 int path) */
float tcbo_dot_act8(int fmt, int K, const uint8_t *wrow, const int8_t *q,
                    const float *d, const int16_t *bs);

/* int8-activation path with TR's per-row non-finite fallback to the float
 * path (cpu_quant_q8.go:125-259) */
void tcbo_qgemm_act8(int fmt, int M, int N, int K, const float *a,
                     const uint8_t *w, float *c, int nthreads);

/* rows of a quantised [V, D] table dequantised (tensor/cpu_quant.go:163-171) */
void tcbo_embedding(int fmt, const uint8_t *raw, int D, const int64_t *idx,
                    int nidx, float *out);

/* first block with a NaN/Inf fp16 scale, -1 if none (tensor/quant.go:108-133) */
long tcbo_check_scales(int fmt, const uint8_t *raw, size_t nbytes);

/* zero blocks: Q4_0 codes 0x88, others all 0 (tensor/quant.go:416-427) */
void tcbo_zero_raw(int fmt, uint8_t *raw, size_t nblocks);

/* TR's seeded test blocks: LCG bytes, NaN/Inf scales pulled finite
 * (tensor/quant_test.go:20-45) */
void tcbo_random_quant(int fmt, uint32_t seed, size_t nblocks, uint8_t *raw);

/* FNV-1a 64 over the float32 bit patterns, little endian */
/* pin the row-parallel workers, one per allowed CPU (timed baseline) */
void tcbo_set_pinning(int on);

uint64_t tcbo_fnv1a_f32(const float *y, size_t n);

#ifdef __cplusplus
}
#endif
#endif
