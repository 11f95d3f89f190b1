// kernels.h - launchers for the non-GEMM device kernels (internal).
#pragma once

#include <cuda_runtime.h>
#include <cstddef>

namespace cg {

int layernorm_fwd(const float *x, long ldx, const float *w, const float *b, float *out, long ldo,
                  float *mean, float *rstd, int T, int C, cudaStream_t s);
size_t layernorm_bwd_scratch_bytes(int T, int C);
int layernorm_bwd(const float *dout, const float *x, const float *w, const float *mean,
                  const float *rstd, float *dx, float *dw, float *db, int T, int C, float *scratch,
                  cudaStream_t s);
// same with dw/db partials over chunks of rows_per_chunk rows (the form
// above uses 128; the training step uses finer chunks for more parallelism)
size_t layernorm_bwd_scratch_bytes(int T, int C, int rows_per_chunk);
int layernorm_bwd(const float *dout, const float *x, const float *w, const float *mean, const float *rstd,
                  float *dx, float *dw, float *db, int T, int C, float *scratch, cudaStream_t s,
                  int rows_per_chunk);
constexpr int kLnBwdTrainRows = 32;
// LayerNorm backward in one pass over the rows with dw / db and, when cs is
// given, cs += column sums of the updated dx (the bias gradient of the linear
// layer that produced the LayerNorm input's gradient); C % 128 == 0,
// C <= 1024, 16-byte aligned rows (layernorm_bwd_fused_ok)
bool layernorm_bwd_fused_ok(int C, const void *dout, const void *x, const void *w, const void *dx);
size_t layernorm_bwd_fused_scratch_bytes(int T, int C);
int layernorm_bwd_fused(const float *dout, const float *x, const float *w, const float *mean, const float *rstd,
                        float *dx, float *dw, float *db, float *cs, int T, int C, float *scratch, cudaStream_t s);
int gelu_fwd(const float *x, float *out, long n, cudaStream_t s);
int gelu_bwd(const float *dout, const float *x, float *dx, long n, cudaStream_t s);
int softmax_rows(float *x, int rows, int cols, cudaStream_t s);
int causal_mask(float *scores, int T, cudaStream_t s);
int cross_entropy_rows(const float *logits, long ldl, const int *targets, float *probs, long ldp,
                       float *dlogits, long ldd, float scale, float *rowterm, int rows, int V,
                       cudaStream_t s);
int cross_entropy_loss(const float *rowterm, int rows, float *loss, cudaStream_t s);
// second half of the fused LM-head + cross-entropy: merges the GEMM
// epilogue's per-64-column (max, sum exp) pairs part[rows][ce_ld] into each
// row's log-sum-exp, writes the NLL terms to rowterm and overwrites the
// logits rows (pitch ldd, ldd % 4 == 0) with scale * (softmax - onehot)
int cross_entropy_fused(float *rows_io, long ldd, const float2 *part, int ce_ld, const int *targets, float scale,
                        float *rowterm, int rows, int V, cudaStream_t s);
int cross_entropy_bwd(float *dlogits, const float *probs, const int *targets, float scale, int rows,
                      int V, cudaStream_t s);
int axpy1(float *dst, const float *src, long n, cudaStream_t s);
int add3(float *dst, const float *a, const float *b, long n, cudaStream_t s);
int scale(float *x, long n, const float *dev_factor, float factor, cudaStream_t s);
int mask_mul(float *x, const unsigned char *mask, long n, float sc, cudaStream_t s);
size_t norm_scratch_bytes();
int grad_norm(const float *g, long n, double *scratch, float *norm, float *clip_factor, float clip,
              cudaStream_t s);
int embed_fwd(const int *tok, const float *wte, const float *wpe, float *out, int BT, int T, int C,
              int pos0, cudaStream_t s);
int embed_bwd(const int *tok, const float *dx, float *dwte, float *dwpe, int B, int T, int C,
              cudaStream_t s);
int adamw(float *p, float *g, float *m, float *v, const unsigned char *decay, long n,
          const float *clip_factor, float lr, float b1, float b2, float eps, float wd, float bc1,
          float bc2, cudaStream_t s);
size_t colsum_scratch_bytes(int M, int N);
int colsum_add(const float *y, long ldy, int M, int N, float *db, float *scratch, cudaStream_t s);
int ce_grad(const float *probs, long ldp, const int *targets, float sc, float *dl, long ldd, int rows,
            int V, cudaStream_t s);
int kv_append(const float *qkv, float *kc, float *vc, int B, int T, long Tmax, int pos0, int C,
              cudaStream_t s);
int gather_last(const float *src, float *dst, int B, int T, int C, cudaStream_t s);
int argmax_rows(const float *x, long ldx, int rows, int V, int *out, float *outval, cudaStream_t s);
// decode-step variants reading positions from device counters (ctr[0] =
// position of the incoming token, ctr[1] = step index)
int embed_fwd_at(const int *tok, const float *wte, const float *wpe, float *out, int B, int C,
                 const int *pos_dev, cudaStream_t s);
int kv_append_at(const float *qkv, float *kc, float *vc, int B, long Tmax, int C, const int *pos_dev,
                 cudaStream_t s);
int argmax_log(const float *x, long ldx, int rows, int V, int *cur, int *log, const int *step_dev,
               cudaStream_t s);
int decode_advance(int *ctr, cudaStream_t s);
// greedy keys: key = (order-preserving bits of the value) << 32 | ~column, so
// the largest key is the largest value with the lowest column
int argmax_keys(const float *x, long ldx, int rows, int V, unsigned long long *keys, cudaStream_t s);
// keys[m] -> token column: next[m], log[*step * rows + m] (log optional) and
// the (value bits, column) pair pair[m], pair[rows + m] (optional); clears
// the keys; then, when ctr is given, advances the decode counters
int greedy_finalize(unsigned long long *keys, int rows, int *next, int *log, const int *step, int *pair,
                    int *ctr, cudaStream_t s);

// ---------------------------------------------------------------- attention
// Causal self-attention over packed qkv rows [B, T, 3C] (head h: columns
// h*hs, C+h*hs, 2C+h*hs), output merged heads out[B, T, C] at column h*hs.
// lse [B*H*T] (row log-sum-exp of the scaled scores) is saved for backward
// when non-null.
int attention_fwd(const float *qkv, float *out, float *lse, int B, int T, int C, int H,
                  cudaStream_t s);
// TF32 tcgen05 version (head size 64): ERR_ARG without launching anything
// when the shapes or alignment do not fit
int attention_fwd_tc(const float *qkv, float *out, float *lse, int B, int T, int C, int H, cudaStream_t s);
// TF32 tcgen05 backward (head size 64), D = rowsum(dO * O) already computed;
// ERR_ARG without launching when the shapes or alignment do not fit
int attention_bwd_tc(const float *qkv, const float *dout, const float *lse, const float *D, float *dqkv, int B,
                     int T, int C, int H, cudaStream_t s);
// dqkv [B, T, 3C] is overwritten with dQ, dK, dV. dout/out are [B, T, C].
size_t attention_bwd_scratch_bytes(int B, int T, int H);
int attention_bwd(const float *qkv, const float *out, const float *dout, const float *lse,
                  float *dqkv, float *scratch, int B, int T, int C, int H, cudaStream_t s);
// Rows [q0, T) only (fast path: the last layer needs only row T-1); output
// rows are written at out + ((b*T + t) * C).
int attention_fwd_rows(const float *qkv, float *out, int B, int T, int C, int H, int q0,
                       cudaStream_t s);
// Single-query decode attention over a KV cache: q [B, C] (head h at h*hs),
// kcache/vcache [B, Tmax, C], attends positions [0, len). out [B, C].
// part: attention_decode_scratch_floats(B, H, Tmax) floats for the split-
// context kernel (head size 64), zero-filled once after allocation (its tail
// holds per-head tickets that every call leaves at zero); NULL selects the
// one-block-per-head kernel.
size_t attention_decode_scratch_floats(int B, int H, long Tmax);
int attention_decode(const float *q, long ldq, const float *kcache, const float *vcache, long Tmax,
                     int len, float *out, int B, int C, int H, float *part, cudaStream_t s);
// same, with the attended length (position + 1) read from a device counter
int attention_decode_at(const float *q, long ldq, const float *kcache, const float *vcache, long Tmax,
                        const int *pos_dev, float *out, int B, int C, int H, float *part,
                        cudaStream_t s);

}  // namespace cg
