/*
 * tcb.h - C ABI of the B200 (sm_100a) quantized-tensor path of TR
 * (sekerahmet/TCB): GGUF block-quantized matvec/matmul, dequantisation,
 * embedding rows and verbatim block upload.
 *
 * Every entry point here replaces one call of TR's tensor.Backend quant
 * branch (internal/compute/gpu/...) and is what a cgo/purego binding in
 * TR's gpu package binds.  Conventions:
 *  - device pointers are plain addresses; a stream is a cudaStream_t passed
 *    as void* (NULL = the legacy default stream);
 *  - w is the [N, K] block store of a quantized tensor, rows of K/blk
 *    blocks laid out exactly as in the GGUF file (tensor/quant.go:14-29);
 *  - dtypes use GGUF type ids (internal/compute/gguf/types.go:12-16);
 *  - every call returns a tcb_status; nothing panics, nothing is freed that
 *    the caller owns.  Scratch memory is owned by the context.
 *  - results do not depend on the GPU's SM count or on launch timing: no
 *    float atomics, fixed reduction order (TR spec 15.22a).
 */
#ifndef TCB_H
#define TCB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum tcb_status {
  TCB_OK = 0,
  TCB_ERR_NULL = 1,        /* a required pointer is NULL */
  TCB_ERR_DTYPE = 2,       /* weight or activation/output type not supported */
  TCB_ERR_SHAPE = 3,       /* K not a multiple of the block, negative size, ... */
  TCB_ERR_ALIGN = 4,       /* offset not on a block boundary */
  TCB_ERR_CUDA = 5,        /* a CUDA runtime call failed (see tcb_last_cuda_error) */
  TCB_ERR_NOMEM = 6,       /* scratch allocation failed */
  TCB_ERR_TIMEOUT = 7,     /* a bounded device-side wait gave up */
  TCB_ERR_UNSUPPORTED = 8, /* combination not provided (e.g. Q8_0 act8 off) */
  TCB_ERR_BOUNDS = 9,      /* an index outside the table */
  TCB_ERR_SCALE = 10,      /* a NaN/Inf block scale (tensor/quant.go:108-128) */
  TCB_ERR_TOO_LARGE = 11   /* the problem does not fit the fixed static scratch */
} tcb_status;

/* weight block types (GGUF ids) */
enum { TCB_Q4_0 = 2, TCB_Q8_0 = 8, TCB_Q4_K = 12, TCB_Q6_K = 14 };
/* activation / output element types (GGUF ids) */
enum { TCB_F32 = 0, TCB_F16 = 1, TCB_BF16 = 30 };

typedef struct tcb_ctx tcb_ctx;

/* Bind to a CUDA device (the primary context, shared with TR's purego
 * driver).  Replaces the lazy backend init of gpu/cuda.go:134-166,241-290. */
int tcb_ctx_create(int device, tcb_ctx **out);
int tcb_ctx_destroy(tcb_ctx *ctx);

/* Message for a status code; never NULL. */
const char *tcb_strerror(int status);
/* The last CUDA error string seen by this context (for TCB_ERR_CUDA). */
const char *tcb_last_cuda_error(tcb_ctx *ctx);

/* The context's device error word: TCB_OK, or the status a kernel recorded
 * when one of its bounded device-side waits gave up (TCB_ERR_TIMEOUT), so a
 * result computed past such a wait is never taken for a good one.  Waits for
 * all work on the device first; clear = 1 resets the word.  TR panics with a
 * coded message where a driver call fails (gpu/gpu.go, the H4xxx codes); the
 * shim's kernels report through this word instead. */
int tcb_device_error(tcb_ctx *ctx, int *status, int clear);

/* elements and bytes of one block; 0,0 for an unknown type
 * (tensor.DType.QuantBlock, tensor/quant.go:35-47) */
int tcb_block_shape(int wtype, int *elems, int *bytes);

/* c[m, n] (+)= sum_k x[m, k] * dequant(w)[n, k]  for m < M, n < N.
 * Replaces gpu/backend_quant.go:43-65 (quantGemm, reached from
 * Backend.Gemm / GemmSet through gemmOuter, backend_gemm.go:132-158).
 *   w       device, [N, K] blocks, K a multiple of the block
 *   x       device, M rows of K elements, row stride ldx elements, xdtype
 *           F32, BF16 or F16 (converted to f32 inside the kernel)
 *   c       device, M rows of N elements, row stride ldc, cdtype F32, BF16
 *           or F16: computed in f32, rounded once
 *   accumulate  1 = Backend.Gemm (C +=), 0 = GemmSet (C =; old C unread)
 * K == 0 is the empty sum (C unchanged, or zeroed when accumulate == 0). */
int tcb_qgemm(tcb_ctx *ctx, int wtype, int M, int N, int K, const void *w,
              const void *x, int xdtype, long ldx, void *c, int cdtype,
              long ldc, int accumulate, void *stream);

/* tcb_qgemm over host buffers: x and c in host memory (w on the device, as
 * uploaded by tcb_quant_upload).  TR's CPU backend runs quantGemm over host
 * slices (tensor/cpu_quant.go:47-160, the same (M, N, K, a, b, c, over)
 * arguments); this entry lets such a caller run the product on the GPU
 * without managing device buffers.  The results are tcb_qgemm's, bit for bit.
 *   - pinned x (page-locked or registered) is copied to the device by a kernel
 *     that reads host memory, and the product starts behind it without a
 *     copy-engine hand-off; pageable x goes through cudaMemcpyAsync (which
 *     then returns only once x has been read);
 *   - pinned c is written by the product in place, over the host link;
 *     pageable c is computed in a device buffer and copied back (the call
 *     then returns after the copy);
 *   - device pointers are used in place.
 * With pinned buffers the call is asynchronous on stream: read c after the
 * stream synchronises.  The device copies live in the context and are shared
 * by its calls: order calls on one context on one stream. */
int tcb_qgemm_host(tcb_ctx *ctx, int wtype, int M, int N, int K,
                   const void *w, const void *x, int xdtype, long ldx,
                   void *c, int cdtype, long ldc, int accumulate,
                   void *stream);

/* The int8-activation product of TR's TR_quantized_activations block:
 * every finite row of x is quantised per weight block (quantizeQ8,
 * tensor/cpu_quant_q8.go:39-68), dotted in integers per block and folded
 * in block order bit-exactly as TR's CPU kernels do
 * (cpu_quant_q8.go:74-116,378-407); a row holding NaN/Inf takes the float
 * path (cpu_quant_q8.go:157-174).  Replaces ActQuantGemmer.GemmActQuant
 * (tensor/matmul.go:59-61, CPU-only in TR).  Q8_0 weights are an extension
 * (TR refuses them, H6723) with dotQ4Q8Go's fold.  Same arguments as
 * tcb_qgemm; TR's method accumulates, pass accumulate = 1 for it. */
int tcb_qgemm_act8(tcb_ctx *ctx, int wtype, int M, int N, int K,
                   const void *w, const void *x, int xdtype, long ldx,
                   void *c, int cdtype, long ldc, int accumulate,
                   void *stream);

/* out[i] = dequant(w)[i] for i < n: the first n elements of the block
 * store at w (n a multiple of the block), bit-identical to TR's CPU dequant
 * for every fp16 scale pattern including NaN and Inf (x86 NaN rule).
 * odtype F32, BF16 or F16 (rounded from f32 as TR's Cast does).
 * Replaces QuantOpener.OpenQuant (tensor/quant.go:103-105,
 * gpu/backend_quant.go:117-134). */
int tcb_qdequant(tcb_ctx *ctx, int wtype, const void *w, long n, void *out,
                 int odtype, void *stream);

/* out[i, :] = dequant(w)[idx[i], :]  for a [V, D] table on the device;
 * idx is a HOST array of nidx row numbers (TR passes a Go []int) and out a
 * device [nidx, D] f32 array.  An index outside [0, V) is refused
 * (TCB_ERR_BOUNDS) before anything is launched.  Replaces
 * Backend.Embedding with quantized w (tensor/limits.go:15-45,
 * gpu/backend_row.go:186). */
int tcb_qembed(tcb_ctx *ctx, int wtype, const void *w, long V, int D,
               const int64_t *idx, int nidx, float *out, void *stream);

/* Verbatim block upload/download (FromRaw / ToRaw, gpu/typed.go:24-55):
 * the bytes cross unchanged.  tcb_quant_upload refuses a block whose
 * fp16 scale is NaN/Inf (CheckQuantScales, tensor/quant.go:108-128) and
 * reports its index in *bad_block (-1 when all are finite). */
int tcb_quant_upload(tcb_ctx *ctx, int wtype, const void *host, size_t nbytes,
                     void *dev, long *bad_block, void *stream);
int tcb_quant_download(tcb_ctx *ctx, const void *dev, size_t nbytes,
                       void *host, void *stream);

/* Zero blocks on the device: Q4_0 codes 0x88, every other byte 0
 * (QuantZeroRaw, tensor/quant.go:416-427; gpu/backend_memory.go:131-152). */
int tcb_quant_zero(tcb_ctx *ctx, int wtype, void *dev, long nblocks,
                   void *stream);

/* host-side scale check (CheckQuantScales); *bad_block = -1 if clean */
int tcb_check_scales(int wtype, const void *host, size_t nbytes,
                     long *bad_block);

/* ---- Llama-shaped decoder, batch 1 (the callers either side of the path) ----
 *
 * A decode step of TR's GPT (lib/layers.tr: GPT.single_step 658-666, block
 * residuals 348-389, RMSNorm 68-79, rotary table and apply_rotary 85-107,
 * grouped-query causal attention 126-215, merged SwiGLU 224-276) over
 * quantized weights,
 * with an fp16 KV cache.  Every launch of a step runs on the caller's stream
 * and the step can be captured once into a CUDA graph: the current token,
 * the position and the prompt live on the device, so a prompt and the
 * greedy continuation are the same graph replayed, with no host round trip.
 * Weights are device block stores ([rows, K] GGUF blocks); the engine keeps
 * the pointers (the caller owns and keeps the memory). */
typedef struct tcb_llama tcb_llama;

typedef struct tcb_llama_config {
  int n_layers, d_model, n_heads, n_kv_heads, head_dim, ffn_dim, vocab;
  int max_ctx;        /* KV-cache positions (prompt + generated) */
  float eps;          /* RMSNorm epsilon */
  float rope_theta;   /* rotary frequency base */
  /* tensor parallelism (0 or 1: none).  Rank r holds query heads
   * [r H/tp, (r+1) H/tp) with their KV heads, gate/up rows [r ffn/tp, ...)
   * of each half, the matching K-columns of o and down, and vocabulary rows
   * [r vocab/tp, ...) of the head; the embedding table, the norms and the
   * residual are replicated.  One all-reduce follows o and down, and an
   * all-gather of the local greedy candidates picks the token. */
  int tp_size, tp_rank;
} tcb_llama_config;

typedef struct tcb_llama_weights {
  const void *tok_emb;  int tok_emb_type;  /* [vocab, d] blocks */
  const float *final_norm;                  /* [d] */
  const void *head;     int head_type;      /* [vocab, d] blocks */
  /* arrays of n_layers pointers */
  const float *const *attn_norm;            /* [d] */
  const float *const *ffn_norm;             /* [d] */
  const void *const *qkv;  int qkv_type;    /* [(H + 2*KVH)*hd, d]: q rows, k rows, v rows */
  const void *const *o;    int o_type;      /* [d, H*hd] */
  const void *const *gate_up; int gate_up_type; /* [2*ffn, d]: gate rows, then up rows */
  const void *const *down; int down_type;   /* [d, ffn] */
  /* Optional per-layer block types ([n_layers][5]: the q and k rows, the v
   * rows, o, gate_up, down), overriding the class types above; NULL for
   * none.  A layer's qkv tensor is then its q and k rows in the first type
   * followed by its v rows in the second (llama.cpp's Q4_K_M files give some
   * layers' v and down Q6_K blocks, the others Q4_K). */
  const int *layer_types;
} tcb_llama_weights;

int tcb_llama_create(tcb_ctx *ctx, const tcb_llama_config *cfg, const tcb_llama_weights *w, tcb_llama **out);
int tcb_llama_destroy(tcb_llama *m);
/* Start a sequence: copies the n prompt token ids (host, n >= 1) to the
 * device and sets position 0 with prompt[0] as the current token.  Steps
 * 0..n-2 then feed the prompt; later steps feed their own greedy token. */
int tcb_llama_start(tcb_llama *m, const int64_t *prompt, int n, void *stream);
/* Feed prompt[0..n-2] (n given to tcb_llama_start, which must come directly
 * before) through the model as row batches of up to 2048 positions: the
 * quantized products on the tensor cores (tcb_qgemm), causal attention over
 * the cache, the K/V of every position appended.  Leaves the engine where
 * n-1 prompt steps would have left it (position n-1, current token
 * prompt[n-1]); the next tcb_llama_step feeds the last prompt token and
 * takes the first greedy token.  TR's generate runs the whole prompt
 * through the model in one call the same way (lib/layers.tr 735-740).
 * Tensor parallelism sums the residual rows with NCCL.  Returns
 * TCB_ERR_UNSUPPORTED when a step has already run since the start. */
int tcb_llama_prefill(tcb_llama *m, void *stream);
/* Rows per pass of tcb_llama_prefill (rows >= 1; 0 restores the default
 * 2048).  Fewer rows need smaller row buffers; a prompt longer than rows + 1
 * positions then takes several passes with the same result (the tests use
 * it to cover pass boundaries).  TR's generate has no such setting. */
int tcb_llama_set_prefill_rows(tcb_llama *m, int rows);
/* The prompt pass of several sequences at once (TR's generate over a batch
 * of prompts): count engines made from the same weights and shapes, each
 * started with its own prompt (tcb_llama_start), are fed as one set of rows
 * through the products, with rotary, the cache append and causal attention
 * per sequence; each engine is then left as tcb_llama_prefill leaves it.
 * The rows of all sequences go through in one pass (row buffers of the first
 * engine, sized for them).  TCB_ERR_SHAPE when the engines differ in model,
 * TCB_ERR_UNSUPPORTED when one has stepped since its start or appears twice. */
int tcb_llama_prefill_batch(tcb_llama *const *engines, int count, void *stream);
/* One step: embed the current token, run every layer at the current
 * position (appending its K/V), score the vocabulary, take the greedy
 * token (first maximum), store it at tokens[pos + 1], advance.  Replays the
 * captured graph when tcb_llama_capture has made one. */
int tcb_llama_step(tcb_llama *m, void *stream);
/* Capture one step into a CUDA graph (on a stream of the engine's own,
 * after the caller's stream has drained); tcb_llama_step replays it on the
 * caller's stream from then on. */
int tcb_llama_capture(tcb_llama *m, void *stream);
/* Kernel launches in one captured step (the kernel nodes of the graph
 * tcb_llama_capture made); TCB_ERR_UNSUPPORTED before a capture. */
int tcb_llama_step_kernels(tcb_llama *m, int *kernels);
/* Device pointers of the token history (int64 [max_ctx]) and the logits of
 * the last step (float [vocab], this rank's vocabulary rows). */
int tcb_llama_buffers(tcb_llama *m, int64_t **tokens, float **logits);
/* Tensor parallelism over NCCL (libnccl.so.2, loaded at run time; the copy
 * the process has already loaded is reused).  Rank 0 makes an id, every
 * rank passes the same 128 bytes to tcb_llama_tp_init (before the first
 * step or capture), with its device current. */
int tcb_nccl_unique_id(unsigned char *id128);
int tcb_llama_tp_init(tcb_llama *m, const unsigned char *id128);
/* All-reduce of the residual over NVLink peer memory in place of NCCL's
 * (the step's collective after o and after down, TR's row-parallel
 * sublayers, layers.tr 348-389): each rank makes its exchange buffer and
 * exports a 64-byte CUDA IPC handle of it, the caller gathers all ranks'
 * handles in rank order (tp_size * 64 bytes) and passes them to
 * tcb_llama_peer_init, before the first step or capture.  Without it the
 * step uses NCCL.  A batch (tcb_llama_batch_create) of up to 16 engines led
 * by this one, created after the set-up, sums its residual rows the same
 * way.  The greedy pick's all-gather stays on NCCL. */
int tcb_llama_peer_handle(tcb_llama *m, unsigned char *handle64);
int tcb_llama_peer_init(tcb_llama *m, const unsigned char *handles);

/* Self-test of the peer all-reduce's bounded wait, on one device: runs the
 * all-reduce kernel once as rank `rank` of `tp` with every rank's exchange
 * buffer allocated locally, so for tp > 1 the other ranks' values never
 * arrive and the wait gives up after `polls` polls, leaving
 * TCB_ERR_TIMEOUT in the device error word (tcb_device_error); with tp = 1
 * the rank's own values complete the wait.  Synchronises the stream; the
 * context stays usable.  No counterpart in TR. */
int tcb_peer_ar_selftest(tcb_ctx *ctx, int tp, int rank, int d_model, unsigned polls, void *stream);

/* Greedy decode of several sequences together (TR's generate over a batch
 * of prompts, lib/layers.tr 712-770: one GPT.single_step per generated
 * position for every row of the batch).  The count engines (at most
 * TCB_LLAMA_MAX_BATCH) are made from the same weights and shapes and
 * started with their own prompts (tcb_llama_start, optionally
 * tcb_llama_prefill_batch); the batch keeps pointers to them, each keeps
 * its own K/V cache, position and token history (tcb_llama_buffers).  A
 * step feeds every sequence its current token: each product runs once over
 * the count rows (tcb_qgemm: up to 8 rows of x per matvec launch, the
 * weights streamed once for them), attention runs per sequence in one
 * launch, and every sequence takes its own greedy token.  Under tensor
 * parallelism the residual rows are summed by NCCL (tcb_llama_tp_init on
 * the first engine) and the candidates of all sequences are gathered in
 * one all-gather.  Returns TCB_ERR_SHAPE when the engines differ in model
 * or count is out of range, TCB_ERR_UNSUPPORTED when an engine is given
 * twice. */
#define TCB_LLAMA_MAX_BATCH 64
typedef struct tcb_llama_batch tcb_llama_batch;
int tcb_llama_batch_create(tcb_llama *const *engines, int count, tcb_llama_batch **out);
int tcb_llama_batch_destroy(tcb_llama_batch *b);
/* One step of every sequence (the captured graph once
 * tcb_llama_batch_capture has made one).  TCB_ERR_BOUNDS when a sequence has
 * no cache position left. */
int tcb_llama_batch_step(tcb_llama_batch *b, void *stream);
/* Capture one batch step into a CUDA graph (as tcb_llama_capture).  Run one
 * eager step first: it sizes the scratch of the products. */
int tcb_llama_batch_capture(tcb_llama_batch *b, void *stream);
/* Device pointer of the last step's logits, float [count][vocab] (this
 * rank's vocabulary rows). */
int tcb_llama_batch_logits(tcb_llama_batch *b, float **logits);

/* Size of the device array that tcb_qgemm_act8_static works in. */
#define TCB_STATIC_SCRATCH_BYTES (4u << 20)

/* tcb_qgemm_act8 for callers that must not allocate device memory.
 *
 * No counterpart in TR: TR's int8-activation product runs on the CPU.
 * This entry point exists for hosts that reserve all device memory up
 * front or must never enter the CUDA allocator on this path (for example
 * an embedding runtime with a fixed memory plan, or a caller on a
 * latency-critical thread that must not take the allocator's locks).  It
 * takes no context and calls no cudaMalloc, cudaFree or other allocating
 * routine: the quantised activations live in one file-scope device array
 * of TCB_STATIC_SCRATCH_BYTES that every GPU loading libtcb holds until the
 * process exits.
 *   - It runs on the calling thread's current device.  Every call looks up
 *     the array's device address (cudaGetSymbolAddress), so a device reset
 *     between calls is safe; the first call on a device may load the
 *     module, so make it before any stream capture.
 *   - It runs the portable quantise and dot kernels (about 64 us per
 *     activation row at 4096 x 4096, against 9.4 us for one row through
 *     tcb_qgemm_act8), since the faster kernels need per-call scratch.
 *   - Problems needing more than TCB_STATIC_SCRATCH_BYTES of scratch
 *     (about 1.28 bytes per element of x, M*K in all) are refused with
 *     TCB_ERR_TOO_LARGE before anything is launched.
 *   - Every call shares the one array: calls whose work overlaps on the GPU
 *     (different streams, or different host threads without ordering)
 *     race and may return wrong results.  Order them on one stream.
 *   - The array keeps the last call's contents; each call writes every
 *     scratch byte it reads before reading it.
 * Results are bit-identical to tcb_qgemm_act8 (same arguments, same
 * int8-activation semantics, NaN/Inf rows on the float path). */
int tcb_qgemm_act8_static(int wtype, int M, int N, int K, const void *w,
                          const void *x, int xdtype, long ldx, void *c,
                          int cdtype, long ldc, int accumulate, void *stream);

#ifdef __cplusplus
}
#endif
#endif
