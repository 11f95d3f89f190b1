/*
 * cngpt_oracle.h - CPU restatement of the reference's GEMM hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the parity checker for libcngpt_cuda:
 * only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg may
 * load it, and never as the thing measured or shipped.
 *
 * Every function restates one function of the reference (moebiusV/cngpt,
 * release 0.1.0) in plain C11 with fp32 arithmetic; the citation next to each
 * declaration is the reference file:line it follows. The restatement is
 * pinned against the reference itself (oracle/_ref/libcngpt_ref.so, built by
 * oracle/Makefile from the reference's own sources) by tests/test_oracle.py
 * and by the golden fixtures under tests/golden/.
 */
#ifndef CNGPT_ORACLE_H
#define CNGPT_ORACLE_H
#ifdef __cplusplus
extern "C" {
#endif

/* ---- ops (src/ops.h:19-107) ------------------------------------------- */
void  orc_linear_fwd(const float *X, const float *W, const float *b, float *Y,
                     int M, int K, int N);                       /* src/ops.c:109 */
void  orc_linear_bwd_dx(const float *dY, const float *W, float *dX,
                        int M, int K, int N);                    /* src/ops.c:125 */
void  orc_linear_bwd_dw(const float *dY, const float *X, float *dW, float *db,
                        int M, int K, int N);                    /* src/ops.c:135 */
void  orc_attn_scores(const float *Q, const float *K, float *scores,
                      int B, int T, int hs);                     /* src/ops.c:155 */
void  orc_attn_values(const float *scores, const float *V, float *out,
                      int B, int T, int hs);                     /* src/ops.c:172 */
void  orc_layernorm_fwd(const float *x, const float *w, const float *b,
                        float *out, float *mean, float *rstd, int T, int C); /* src/ops.c:191 */
void  orc_layernorm_bwd(const float *dout, const float *x, const float *w,
                        const float *mean, const float *rstd,
                        float *dx, float *dw, float *db, int T, int C);      /* src/ops.c:250 */
void  orc_gelu_fwd(const float *x, float *out, int n);           /* src/ops.c:357 */
void  orc_gelu_bwd(const float *dout, const float *x, float *dx, int n); /* src/ops.c:382 */
void  orc_softmax_inplace(float *x, int rows, int cols);         /* src/ops.c:424 */
void  orc_causal_mask(float *scores, int T);                     /* src/ops.c:488 */
void  orc_cross_entropy_fwd(const float *logits, const int *targets,
                            float *probs, float *loss, int B, int T, int V); /* src/ops.c:499 */
void  orc_cross_entropy_bwd(float *dlogits, const float *probs, const int *targets,
                            float scale, int B, int T, int V);   /* src/ops.c:576 */
void  orc_residual_add(float *dst, const float *src, int n);     /* src/ops.c:594 */
float orc_global_grad_norm(const float *g, int n);               /* src/ops.c:631 */
void  orc_scale_grads(float *g, int n, float s);                 /* src/ops.c:636 */

/* ---- model (src/model.h:143-194) -------------------------------------- */
typedef struct {
    int n_layer, n_head, n_embd, vocab_size, block_size;
} orc_config;

long  orc_num_params(const orc_config *c);                       /* src/model.c:20 */
/* glibc rand() stream, Marsaglia polar normals (src/model.c:275-331). The caller
 * seeds (or does not seed) the stream exactly as the reference driver would. */
void  orc_init_weights(const orc_config *c, float *params);
void  orc_decay_mask(const orc_config *c, unsigned char *decay); /* src/model.c:148-172 */

/* gpt_forward (src/model.c:442-625). logits [B*T*V] and probs [B*T*V] may be NULL.
 * Returns the mean cross-entropy (0 when targets == NULL). */
float orc_forward(const orc_config *c, const float *params, const int *tokens,
                  const int *targets, int B, int T, float *logits, float *probs);

/* gpt_forward + gpt_backward (src/model.c:634-873); gradients ACCUMULATE into
 * grads (the reference's grad arena semantics). Returns the loss. */
float orc_forward_backward(const orc_config *c, const float *params, const int *tokens,
                           const int *targets, int B, int T, float *grads);

/* gpt_adamw (src/model.c:888-921): one step, *step is incremented. */
void  orc_adamw(float *params, float *grads, float *m, float *v,
                const unsigned char *decay, long n, int *step, float lr,
                float beta1, float beta2, float eps, float wd, float grad_clip);

/* gpt_forward_fast (src/fast.c:227-333): last-position logits [B*V]. */
void  orc_forward_last(const orc_config *c, const float *params, const int *tokens,
                       int B, int T, float *logits_last);

#ifdef __cplusplus
}
#endif
#endif
