/*
 * cngpt_cuda.h - extensions of libcngpt_cuda beyond the reference's C API.
 *
 * The drop-in entry points keep the reference's names and signatures
 * (cngpt/ops.h, cngpt/model.h, cngpt/fast.h). The reference has no GPU, no
 * error channel, no precision modes, no KV cache and no collectives, so the
 * calls below have no counterpart in it; each comment names the reference
 * behaviour it extends.
 */
#ifndef CNGPT_CUDA_H
#define CNGPT_CUDA_H

#include <stddef.h>

#include "cngpt/model.h"
#include "cngpt/fast.h"
#include "cngpt/ops.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status ------------------------------------------------------------
 * The reference reports failure by return value -1 / NULL / 0.0f and stderr
 * (src/model.c:179-188, 452-455). Every call here also records a status. */
#define CNGPT_OK              0
#define CNGPT_ERR_CUDA        1  /* a CUDA runtime call failed */
#define CNGPT_ERR_ARG         2  /* invalid shape, pointer or alignment */
#define CNGPT_ERR_ALLOC       3  /* device allocation failed */
#define CNGPT_ERR_DEVICE_WAIT 4  /* a bounded device-side wait gave up */
#define CNGPT_ERR_NCCL        5  /* a collective failed */
#define CNGPT_ERR_STATE       6  /* wrong call order or unknown model */

int         cngpt_cuda_last_status(void);   /* status of the last failing call */
const char *cngpt_cuda_last_message(void);
void        cngpt_cuda_clear_status(void);
/* synchronise the library stream and read the device error words */
int         cngpt_cuda_check(void);

/* ---- configuration ------------------------------------------------------ */
#define CNGPT_PREC_TF32   0  /* one tcgen05 kind::tf32 pass (~1e-3 relative) */
#define CNGPT_PREC_3XTF32 1  /* hi*hi + hi*lo + lo*hi split (fp32-level); default */
#define CNGPT_PREC_FP32   2  /* CUDA-core fp32 FMA kernels (reference-exact math) */
int   cngpt_cuda_set_precision(int mode);
int   cngpt_cuda_get_precision(void);
/* cudaStream_t for every following call; NULL = the legacy default stream */
int   cngpt_cuda_set_stream(void *stream);
void *cngpt_cuda_get_stream(void);
/* arenas allocated after this call use cudaMallocManaged (host-dereferenceable) */
int   cngpt_cuda_set_managed(int on);
/* number of kernels this library has launched so far */
unsigned long long cngpt_cuda_launch_count(void);
/* limit of every bounded device-side wait (mbarrier phases in the GEMM and
 * attention kernels, peer flags of the tensor-parallel exchange), in
 * nanoseconds of %globaltimer; 0 restores the default of 2 s. A wait that
 * runs out records its site, ends its kernel without writing the output it
 * waited for, and the next cngpt_cuda_check returns CNGPT_ERR_DEVICE_WAIT.
 * Synchronises the device first. */
int   cngpt_cuda_set_wait_limit_ns(unsigned long long ns);

/* ---- GEMM with fused epilogue --------------------------------------------
 * out[M,N] = alpha * op(A)[M,K] op(B)[N,K]^T, then the epilogue:
 *   CNGPT_EPI_STORE     D = acc + bias
 *   CNGPT_EPI_ACCUM     D = D + acc (+ bias)
 *   CNGPT_EPI_GELU      t = acc + bias; D = t (if D); D2 = gelu(t)
 *   CNGPT_EPI_RESID     t = acc + bias; D = t (if D); D2 = R + t
 *   CNGPT_EPI_GELU_BWD  D = acc * gelu'(G)
 * a_mn: A stored [K][lda] instead of [M][lda]; b_mn: B stored [K][ldb]
 * instead of [N][ldb]. All pointers are device pointers. This is the kernel
 * behind linear_fwd / linear_bwd_dx / linear_bwd_dw (src/ops.c:109-149). */
#define CNGPT_EPI_STORE    0
#define CNGPT_EPI_ACCUM    1
#define CNGPT_EPI_GELU     2
#define CNGPT_EPI_RESID    3
#define CNGPT_EPI_GELU_BWD 4
int cngpt_cuda_gemm(const float *A, long lda, int a_mn, const float *B, long ldb, int b_mn,
                    int M, int N, int K, int epi_mode, float alpha,
                    float *D, long ldd, const float *bias, float *D2, long ldd2,
                    const float *R, long ldr, const float *G, long ldg);

/* ---- fused attention (src/model.c:514-563, 742-822) -----------------------
 * qkv [B,T,3C] device; out [B,T,C]; lse [B*H*T] (may be NULL). */
int cngpt_cuda_attention_fwd(const float *qkv, float *out, float *lse,
                             int B, int T, int C, int H);
int cngpt_cuda_attention_bwd(const float *qkv, const float *out, const float *dout,
                             const float *lse, float *dqkv, int B, int T, int C, int H);

/* ---- LayerNorm backward without device allocation ---------------------------
 * No counterpart in the reference. Same result as layernorm_bwd (cngpt/ops.h)
 * on device or managed pointers, but it allocates nothing: the dw/db partial
 * sums go to a fixed 2 MiB array inside the library (every GPU that loads the
 * library holds it until the process exits), for callers that cannot let a
 * library call cudaMalloc - it synchronises the device, and it fails when the
 * caller has already reserved the GPU's memory for its own pool.
 *  - T * C up to about 33.5 million (ceil(T/128) * 2 * C <= 524288 floats);
 *    larger shapes return CNGPT_ERR_ARG with a message, as do host pointers.
 *  - The first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress); make that first call before any stream capture.
 *  - All calls share the one array: calls that overlap on the GPU (different
 *    streams, or several host threads) race on it and must be serialised.
 *    Nothing in it needs clearing - each call writes every element it reads. */
int cngpt_cuda_layernorm_bwd_noalloc(const float *dout, const float *x, const float *w,
                                     const float *mean, const float *rstd,
                                     float *dx, float *dw, float *db, int T, int C);

/* ---- training ------------------------------------------------------------
 * One full step of the reference's train loop (src/cngpt.c:154-163):
 * zero_grad, forward, backward, [DP allreduce], AdamW with clipping.
 * tokens/targets may be host or device int[B*T]. loss_out (host) may be
 * NULL, in which case nothing synchronises and the loss stays on the device
 * (read it with cngpt_cuda_last_loss). */
int cngpt_cuda_train_step(GPT *m, const int *tokens, const int *targets, int B, int T,
                          float lr, float beta1, float beta2, float eps, float wd,
                          float grad_clip, float *loss_out);
int cngpt_cuda_last_loss(GPT *m, float *loss_out);

/* Decode steps of up to 8 sequences (head size 64) as one cooperative launch
 * per token - every layer, the LM head and the greedy pick, phases separated
 * by bounded grid barriers - instead of a chain of five kernels per layer.
 * Off by default (also CNGPT_CUDA_DECODE_STEP_KERNEL=1): on B200 it does not
 * yet beat the kernel chain. Same tokens either way up to fp32 rounding. */
int cngpt_cuda_set_decode_step_kernel(int on);

/* ---- training batches, uploaded one step ahead -----------------------------
 * The reference's DataLoader (src/dataloader.c:62-82) fills host int arrays
 * inputs[b*T+t] = data[pos + b*T + t], targets[b*T+t] = data[pos + b*T + t + 1]
 * from an mmap'd uint16 token file, then advances pos by B*T and rewinds to 0
 * when pos + B*T + 1 would pass the end. The loader produces the same batch
 * sequence in device memory: each call returns the device inputs / targets of
 * the current batch (the library stream waits for their upload) and starts
 * uploading the next batch through a pinned buffer on a copy stream, so the
 * upload overlaps the step that consumes the current one. The returned
 * pointers stay valid until the call after next. `data` (host, e.g. the
 * DataLoader's mmap) must outlive the loader. */
typedef struct cngpt_cuda_loader cngpt_cuda_loader;
int    cngpt_cuda_loader_create(cngpt_cuda_loader **out, const unsigned short *data, size_t n_tokens,
                                int B, int T);
int    cngpt_cuda_loader_next(cngpt_cuda_loader *dl, const int **inputs, const int **targets);
int    cngpt_cuda_loader_reset(cngpt_cuda_loader *dl);                     /* dataloader_reset */
size_t cngpt_cuda_loader_num_batches(const cngpt_cuda_loader *dl);        /* dataloader_num_batches */
void   cngpt_cuda_loader_free(cngpt_cuda_loader *dl);

/* parameter / gradient / optimizer state transfer (n_params floats) */
int cngpt_cuda_params_to_host(GPT *m, float *dst);
int cngpt_cuda_params_from_host(GPT *m, const float *src);
int cngpt_cuda_grads_to_host(GPT *m, float *dst);
int cngpt_cuda_copy(void *dst, const void *src, size_t bytes); /* any direction, synchronous */

/* ---- training checkpoints -------------------------------------------------
 * The reference saves only the parameters (gpt_save, src/model.c:177-231)
 * and restarts AdamW from zero moments. save_checkpoint writes gpt_save's
 * file followed by an optimizer trailer (step count, first and second
 * moments), so any gpt_load still reads it as a model file; load_checkpoint
 * restores parameters, moments and step (a file without the trailer loads
 * with fresh optimizer state). A model with no arena is created from the
 * file's configuration; otherwise the configurations must match. */
int cngpt_cuda_save_checkpoint(GPT *m, const char *path);
int cngpt_cuda_load_checkpoint(GPT *m, const char *path);

/* ---- greedy decode with a KV cache ---------------------------------------
 * The reference recomputes the whole prefix per token (src/model.c:991-1016);
 * this keeps K and V per layer and runs one row per sequence per step. The
 * greedy token is the argmax of the last-position logits, lowest index on
 * ties (sample_top_k with top_k = 1, src/model.c:945-985).
 * prompt: host or device int[B*T]; out_tokens: host int[B*n_new].
 * T + n_new must not exceed block_size. */
int cngpt_cuda_generate(GPT *m, FastCtx *f, const int *prompt, int B, int T, int n_new,
                        int *out_tokens);

/* ---- data-parallel training over NCCL -------------------------------------
 * One process per GPU. Rank 0 creates the id and shares it out of band. After
 * dp_init, cngpt_cuda_train_step averages the gradient arena over the ranks
 * (the gradient of the mean loss over the global batch) in per-layer buckets:
 * each layer's gradients are averaged on a separate stream as soon as the
 * backward has finished that layer, while it continues with the layers below;
 * the embeddings (wte, wpe) go last. Its loss_out is the mean loss over the
 * global batch. cngpt_cuda_dp_allreduce_grads averages the whole arena at
 * once, for callers that drive gpt_backward themselves. A second dp_init
 * replaces the first one's communicator. */
int cngpt_cuda_dp_unique_id(unsigned char id[128]);
int cngpt_cuda_dp_init(GPT *m, const unsigned char id[128], int world, int rank);
int cngpt_cuda_dp_allreduce_grads(GPT *m);
int cngpt_cuda_dp_free(GPT *m);

/* ---- tensor-parallel inference over NCCL -----------------------------------
 * The reference runs src/fast.c:227-333 on one CPU; these split the same
 * forward over `world` processes, one GPU each, in the Megatron way: QKV by
 * heads (the first n_head % world ranks take one head more), c_proj by the
 * matching input columns, mlp_fc / mlp_proj by 4-column units of the hidden
 * width, the LM head by blocks of ceil(vocab / world) rows of the tied wte.
 * Every rank holds the full model (same weights on every rank: initialise
 * them from the same seed, or load the same file) and gets the id from
 * cngpt_cuda_dp_unique_id on rank 0. Each block ends in two sums of the
 * ranks' partial [rows, n_embd] residual streams: ncclAllReduce for the
 * prefill; for decode batches up to 8 rows the row-split GEMVs push their
 * partials into every rank's receive buffer (CUDA IPC peer memory over
 * NVLink, mapped at tp_init; CNGPT_CUDA_TP_NCCL_ONLY=1 keeps NCCL). The
 * greedy token is merged from every rank's (max, lowest index) pair. All
 * ranks make the same calls in order.
 * plan (host only, no GPU): h0, nh, f0, nf, v0, nv, vpad of `rank`. */
int cngpt_cuda_tp_plan(int n_head, int n_embd, int vocab, int world, int rank, int plan[7]);
int cngpt_cuda_tp_init(GPT *m, const unsigned char id[128], int world, int rank);
/* final-position logits of every sequence, gathered: host float[B * vocab]
 * (may be NULL to skip the gather) - what gpt_forward_fast returns */
int cngpt_cuda_tp_forward_last(GPT *m, const int *tokens, int B, int T, float *logits_out);
/* cngpt_cuda_generate split over the ranks; out_tokens (host) on every rank */
int cngpt_cuda_tp_generate(GPT *m, const int *prompt, int B, int T, int n_new, int *out_tokens);
/* how tp_generate decodes: 1 split over the ranks as above; 2 replicated -
 * every rank runs the whole one-GPU decode (cngpt_cuda_generate) on its full
 * copy of the model, no exchange, identical tokens on every rank; 0 (default)
 * replicated at batch 1, where the split step's two exchanges per layer cost
 * more than the weight stream it divides, split at larger batches */
int cngpt_cuda_tp_set_decode_mode(GPT *m, int mode);
int cngpt_cuda_tp_free(GPT *m);

/* ---- self-test hooks -------------------------------------------------------
 * One launch of the tensor-parallel decode exchange's reduce kernel on one
 * GPU, over a receive buffer of world 1 that holds partial [rows, C] (device;
 * rows <= 8, C <= 2048) for exchange 1. publish = 1 raises the buffer's flag
 * to that exchange: x [rows, C] becomes the partial and stats [rows][2] its
 * LayerNorm mean / rstd. publish = 0 leaves the flag unraised, so the wait runs
 * out after the wait limit: x and stats are left untouched and the call
 * returns CNGPT_ERR_DEVICE_WAIT (site 201). Allocates and frees its buffer. */
int cngpt_cuda_selftest_tp_reduce(float *x, const float *partial, int rows, int C, int publish, float *stats);

#ifdef __cplusplus
}
#endif
#endif /* CNGPT_CUDA_H */
