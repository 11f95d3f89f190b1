/*
 * fast.h - inference forward of libcngpt_cuda (drop-in for the reference's
 * src/fast.h:35-60; FastCtx is byte-identical).
 *
 * gpt_forward_fast returns the final-position logits [B, V] of each
 * sequence in a buffer owned by the context (device memory, or managed in
 * managed mode), valid until the next call; NULL on failure. Attention is
 * the fused causal kernel (no T x T scores; FastCtx.scores stays NULL), the
 * last layer runs only the final row of each sequence past attention, and
 * the LM head runs for those rows only, as in src/fast.c:287-329.
 */
#ifndef CNGPT_FAST_H
#define CNGPT_FAST_H

#include "model.h"

typedef struct {
    int    B, T;
    float *x;
    float *ln;
    float *qkv;
    float *scores;
    float *aout;
    float *hid;
    float *mean, *rstd;
    float *logits;
} FastCtx;

#ifdef __cplusplus
extern "C" {
#endif

void fast_init(FastCtx *f);                   /* ref src/fast.h:48 */
void fast_free(FastCtx *f);                   /* ref src/fast.h:49 */
/* CPU thread count in the reference; accepted and ignored here (one device
 * per process)                                  ref src/fast.h:55 */
void fast_set_threads(int n);
/* ref src/fast.h:60 */
const float *gpt_forward_fast(GPT *m, FastCtx *f, const int *tokens, int B, int T);

#ifdef __cplusplus
}
#endif
#endif /* CNGPT_FAST_H */
