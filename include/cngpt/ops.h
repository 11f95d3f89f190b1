/*
 * ops.h - tensor primitives of libcngpt_cuda (drop-in for the reference's
 * src/ops.h:19-107; same names, argument meaning, C linkage).
 *
 * All matrices are row-major fp32; weights are [out, in]. Pointers may be
 * device, managed or plain host memory: host buffers are staged through the
 * device and copied back before the call returns, so the reference's own
 * unit tests (stack arrays) run unchanged. Calls on device pointers are
 * enqueued on the library stream (cngpt_cuda_set_stream, default the legacy
 * default stream) and are ordered with later copies on that stream.
 * Failures are reported through cngpt_cuda_last_status() (the reference API
 * has no error channel).
 */
#ifndef CNGPT_OPS_H
#define CNGPT_OPS_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Y[M,N] = X[M,K] W[N,K]^T + b[N]; b may be NULL.        ref src/ops.h:19 */
void linear_fwd(const float *X, const float *W, const float *b,
                float *Y, int M, int K, int N);
/* dX[M,K] += dY[M,N] W[N,K]                               ref src/ops.h:23 */
void linear_bwd_dx(const float *dY, const float *W,
                   float *dX, int M, int K, int N);
/* dW[N,K] += dY^T X ; db[N] += column sums of dY (db may be NULL)
 *                                                         ref src/ops.h:28 */
void linear_bwd_dw(const float *dY, const float *X,
                   float *dW, float *db, int M, int K, int N);
/* scores[b] = (1/sqrt(hs)) Q[b] K[b]^T for b < B          ref src/ops.h:35 */
void attn_scores(const float *Q, const float *K, float *scores,
                 int B, int T, int hs);
/* out[b] = scores[b] V[b]                                 ref src/ops.h:39 */
void attn_values(const float *scores, const float *V, float *out,
                 int B, int T, int hs);
/* LayerNorm, eps 1e-5; mean/rstd [T] saved              ref src/ops.h:47 */
void layernorm_fwd(const float *x, const float *w, const float *b,
                   float *out, float *mean, float *rstd, int T, int C);
/* dx += ..., dw += ..., db += ...                         ref src/ops.h:51 */
void layernorm_bwd(const float *dout, const float *x, const float *w,
                   const float *mean, const float *rstd,
                   float *dx, float *dw, float *db, int T, int C);
/* tanh GELU; gelu_bwd accumulates into dx                 ref src/ops.h:59-60 */
void gelu_fwd(const float *x, float *out, int n);
void gelu_bwd(const float *dout, const float *x, float *dx, int n);
/* row softmax in place                                    ref src/ops.h:66 */
void softmax_inplace(float *x, int rows, int cols);
/* scores[i, j > i] = -1e9                                 ref src/ops.h:72 */
void causal_mask(float *scores, int T);
/* probs = softmax(logits); *loss_out = mean NLL           ref src/ops.h:80 */
void cross_entropy_fwd(const float *logits, const int *targets,
                       float *probs_out, float *loss_out,
                       int B, int T, int V);
/* dlogits += scale (probs - onehot(targets))              ref src/ops.h:85 */
void cross_entropy_bwd(float *dlogits, const float *probs,
                       const int *targets,
                       float scale, int B, int T, int V);
/* dst += src                                              ref src/ops.h:92 */
void residual_add(float *dst, const float *src, int n);
/* dropout with the host rand() stream (mask drawn exactly as the reference)
 *                                                         ref src/ops.h:98-99 */
void dropout_fwd(float *x, unsigned char *mask, int n, float p);
void dropout_bwd(float *dx, const unsigned char *mask, int n, float p);
/* ||grads||_2                                             ref src/ops.h:104 */
float global_grad_norm(const float *grads, int n);
/* grads *= scale                                          ref src/ops.h:107 */
void scale_grads(float *grads, int n, float scale);

#ifdef __cplusplus
}
#endif
#endif /* CNGPT_OPS_H */
