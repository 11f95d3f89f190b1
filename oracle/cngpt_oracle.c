/*
 * cngpt_oracle.c - CPU restatement of the reference's GEMM hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see cngpt_oracle.h). Plain loops over fp32
 * data; every matrix product (the reference's cblas_sgemm calls) sums along K
 * in a double accumulator and rounds once, so the oracle's own rounding error
 * stays well below the fp32 noise of the implementations it checks.
 * Parallelised over output rows with OpenMP so GPT-2-sized checks finish.
 */
#include "cngpt_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

/* C[M,N] = alpha * op(A) op(B) + beta * C, row-major.
 * op(A) is [M,K]: A is [M,K] (ta=0) or [K,M] (ta=1); op(B) is [K,N]: B is
 * [K,N] (tb=0) or [N,K] (tb=1). The reference's four sgemm forms
 * (src/ops.c:113,129,139, src/model.c:535-803) are all instances. */
static void mm(int M, int N, int K, float alpha,
               const float *A, int lda, int ta,
               const float *B, int ldb, int tb,
               float beta, float *C, int ldc)
{
    #pragma omp parallel for schedule(static) if ((long)M * N * K > 32768)
    for (int i = 0; i < M; i++) {
        for (int j = 0; j < N; j++) {
            double acc = 0.0;
            for (int k = 0; k < K; k++) {
                double a = ta ? A[(size_t)k * lda + i] : A[(size_t)i * lda + k];
                double b = tb ? B[(size_t)j * ldb + k] : B[(size_t)k * ldb + j];
                acc += a * b;
            }
            float *c = C + (size_t)i * ldc + j;
            *c = (beta == 0.0f) ? (float)(alpha * acc) : (float)(alpha * acc + (double)beta * *c);
        }
    }
}

/* ---------------------------------------------------------------- ops */

void orc_linear_fwd(const float *X, const float *W, const float *b, float *Y,
                    int M, int K, int N)
{
    /* Y = X W^T (beta 0), then + b per row (src/ops.c:113-122) */
    mm(M, N, K, 1.0f, X, K, 0, W, K, 1, 0.0f, Y, N);
    if (b)
        for (int i = 0; i < M; i++)
            for (int j = 0; j < N; j++) Y[(size_t)i * N + j] += b[j];
}

void orc_linear_bwd_dx(const float *dY, const float *W, float *dX, int M, int K, int N)
{
    /* dX += dY W (src/ops.c:129-132) */
    mm(M, K, N, 1.0f, dY, N, 0, W, K, 0, 1.0f, dX, K);
}

void orc_linear_bwd_dw(const float *dY, const float *X, float *dW, float *db,
                       int M, int K, int N)
{
    /* dW += dY^T X ; db += column sums of dY, row by row (src/ops.c:139-148) */
    mm(N, K, M, 1.0f, dY, N, 1, X, K, 0, 1.0f, dW, K);
    if (db)
        for (int i = 0; i < M; i++)
            for (int j = 0; j < N; j++) db[j] += dY[(size_t)i * N + j];
}

void orc_attn_scores(const float *Q, const float *K, float *scores, int B, int T, int hs)
{
    /* per batch entry: S = (1/sqrt(hs)) Q K^T (src/ops.c:158-169) */
    float scale = 1.0f / sqrtf((float)hs);
    for (int b = 0; b < B; b++)
        mm(T, T, hs, scale, Q + (size_t)b * T * hs, hs, 0, K + (size_t)b * T * hs, hs, 1,
           0.0f, scores + (size_t)b * T * T, T);
}

void orc_attn_values(const float *scores, const float *V, float *out, int B, int T, int hs)
{
    /* per batch entry: O = S V (src/ops.c:175-184) */
    for (int b = 0; b < B; b++)
        mm(T, hs, T, 1.0f, scores + (size_t)b * T * T, T, 0, V + (size_t)b * T * hs, hs, 0,
           0.0f, out + (size_t)b * T * hs, hs);
}

void orc_layernorm_fwd(const float *x, const float *w, const float *b,
                       float *out, float *mean, float *rstd, int T, int C)
{
    /* eps 1e-5, biased variance, rstd = 1/sqrt(var+eps) (src/ops.c:231-247) */
    #pragma omp parallel for schedule(static) if (T >= 64)
    for (int t = 0; t < T; t++) {
        const float *xr = x + (size_t)t * C;
        float m = 0.0f;
        for (int c = 0; c < C; c++) m += xr[c];
        m /= (float)C;
        float v = 0.0f;
        for (int c = 0; c < C; c++) { float d = xr[c] - m; v += d * d; }
        float rs = 1.0f / sqrtf(v / (float)C + 1e-5f);
        mean[t] = m;
        rstd[t] = rs;
        for (int c = 0; c < C; c++)
            out[(size_t)t * C + c] = (xr[c] - m) * rs * w[c] + b[c];
    }
}

void orc_layernorm_bwd(const float *dout, const float *x, const float *w,
                       const float *mean, const float *rstd,
                       float *dx, float *dw, float *db, int T, int C)
{
    /* dx += rstd (dn - mean(dn) - xhat mean(dn xhat)); dw += dout xhat;
     * db += dout (src/ops.c:305-329) */
    for (int t = 0; t < T; t++) {
        const float *dr = dout + (size_t)t * C, *xr = x + (size_t)t * C;
        float m = mean[t], rs = rstd[t], s1 = 0.0f, s2 = 0.0f;
        for (int c = 0; c < C; c++) {
            float xh = (xr[c] - m) * rs, dn = dr[c] * w[c];
            s1 += dn;
            s2 += dn * xh;
        }
        s1 /= (float)C;
        s2 /= (float)C;
        for (int c = 0; c < C; c++) {
            float xh = (xr[c] - m) * rs, dn = dr[c] * w[c];
            dx[(size_t)t * C + c] += rs * (dn - s1 - xh * s2);
            dw[c] += dr[c] * xh;
            db[c] += dr[c];
        }
    }
}

#define ORC_GELU_K 0.7978845608028654f /* sqrt(2/pi), src/ops.c:337 */
#define ORC_GELU_C 0.044715f           /* src/ops.c:338 */

void orc_gelu_fwd(const float *x, float *out, int n)
{
    /* 0.5 x (1 + tanh(k (x + c x^3))) (src/ops.c:340-345) */
    #pragma omp parallel for schedule(static) if (n >= 65536)
    for (int i = 0; i < n; i++) {
        float v = x[i];
        out[i] = 0.5f * v * (1.0f + tanhf(ORC_GELU_K * (v + ORC_GELU_C * v * v * v)));
    }
}

void orc_gelu_bwd(const float *dout, const float *x, float *dx, int n)
{
    /* dx += dout * gelu'(x) (src/ops.c:347-355, 412-416) */
    #pragma omp parallel for schedule(static) if (n >= 65536)
    for (int i = 0; i < n; i++) {
        float v = x[i];
        float th = tanhf(ORC_GELU_K * (v + ORC_GELU_C * v * v * v));
        float g = 0.5f * (1.0f + th) +
                  0.5f * v * (1.0f - th * th) * ORC_GELU_K * (1.0f + 3.0f * ORC_GELU_C * v * v);
        dx[i] += dout[i] * g;
    }
}

void orc_softmax_inplace(float *x, int rows, int cols)
{
    /* max-subtracted, exp, normalise by 1/sum (src/ops.c:464-480) */
    for (int r = 0; r < rows; r++) {
        float *row = x + (size_t)r * cols, mx = -FLT_MAX, s = 0.0f;
        for (int c = 0; c < cols; c++) if (row[c] > mx) mx = row[c];
        for (int c = 0; c < cols; c++) { row[c] = expf(row[c] - mx); s += row[c]; }
        float inv = 1.0f / s;
        for (int c = 0; c < cols; c++) row[c] *= inv;
    }
}

void orc_causal_mask(float *scores, int T)
{
    /* j > i  ->  -1e9 (src/ops.c:490-492) */
    for (int i = 0; i < T; i++)
        for (int j = i + 1; j < T; j++) scores[(size_t)i * T + j] = -1e9f;
}

void orc_cross_entropy_fwd(const float *logits, const int *targets, float *probs,
                           float *loss, int B, int T, int V)
{
    /* per row: softmax into probs, loss -= (l[tgt]-max) - log(sum); mean over
     * B*T rows, accumulated in one float in row order (src/ops.c:551-573) */
    int BT = B * T;
    float *rowloss = malloc((size_t)BT * sizeof(float));
    #pragma omp parallel for schedule(static) if ((long)BT * V >= 65536)
    for (int r = 0; r < BT; r++) {
        const float *lg = logits + (size_t)r * V;
        float *pr = probs + (size_t)r * V, mx = -FLT_MAX, s = 0.0f;
        for (int v = 0; v < V; v++) if (lg[v] > mx) mx = lg[v];
        for (int v = 0; v < V; v++) { pr[v] = expf(lg[v] - mx); s += pr[v]; }
        float inv = 1.0f / s;
        for (int v = 0; v < V; v++) pr[v] *= inv;
        rowloss[r] = (lg[targets[r]] - mx) - logf(s);
    }
    float acc = 0.0f;
    for (int r = 0; r < BT; r++) acc -= rowloss[r];
    free(rowloss);
    *loss = acc / (float)BT;
}

void orc_cross_entropy_bwd(float *dlogits, const float *probs, const int *targets,
                           float scale, int B, int T, int V)
{
    /* dlogits += scale (probs - onehot) (src/ops.c:581-587) */
    int BT = B * T;
    #pragma omp parallel for schedule(static) if ((long)BT * V >= 65536)
    for (int r = 0; r < BT; r++)
        for (int v = 0; v < V; v++)
            dlogits[(size_t)r * V + v] +=
                scale * (probs[(size_t)r * V + v] - (v == targets[r] ? 1.0f : 0.0f));
}

void orc_residual_add(float *dst, const float *src, int n)
{
    for (int i = 0; i < n; i++) dst[i] += src[i]; /* src/ops.c:596 */
}

float orc_global_grad_norm(const float *g, int n)
{
    /* ||g||_2 (src/ops.c:633); accumulated in double here, as BLAS nrm2
     * implementations scale to avoid overflow */
    double s = 0.0;
    for (int i = 0; i < n; i++) s += (double)g[i] * (double)g[i];
    return (float)sqrt(s);
}

void orc_scale_grads(float *g, int n, float s)
{
    for (int i = 0; i < n; i++) g[i] *= s; /* src/ops.c:638 */
}

/* -------------------------------------------------------------- model */

long orc_num_params(const orc_config *c)
{
    long C = c->n_embd, V = c->vocab_size, T = c->block_size, L = c->n_layer;
    return V * C + T * C + L * (12 * C * C + 13 * C) + 2 * C; /* src/model.c:20-48 */
}

/* parameter views in the reference's flat order (src/model.c:54-83) */
typedef struct {
    const float *wte, *wpe, *lnfw, *lnfb;
    const float *ln1w, *ln1b, *attw, *attb, *prjw, *prjb, *ln2w, *ln2b, *fcw, *fcb, *mpw, *mpb;
} view_t;

static long layer_size(long C) { return 12 * C * C + 13 * C; }

static void view_layer(const orc_config *c, const float *p, int l, view_t *v)
{
    long C = c->n_embd;
    const float *q = p + (long)c->vocab_size * C + (long)c->block_size * C + l * layer_size(C);
    v->ln1w = q; q += C;   v->ln1b = q; q += C;
    v->attw = q; q += 3 * C * C; v->attb = q; q += 3 * C;
    v->prjw = q; q += C * C;     v->prjb = q; q += C;
    v->ln2w = q; q += C;   v->ln2b = q; q += C;
    v->fcw = q;  q += 4 * C * C; v->fcb = q; q += 4 * C;
    v->mpw = q;  q += 4 * C * C; v->mpb = q;
}

static void view_global(const orc_config *c, const float *p, view_t *v)
{
    long C = c->n_embd;
    v->wte = p;
    v->wpe = p + (long)c->vocab_size * C;
    v->lnfw = p + (long)c->vocab_size * C + (long)c->block_size * C + c->n_layer * layer_size(C);
    v->lnfb = v->lnfw + C;
}

/* Marsaglia polar normal from rand() (src/model.c:275-284) */
static float orc_randn(void)
{
    float u, v, s;
    do {
        u = (float)rand() / (float)RAND_MAX * 2.0f - 1.0f;
        v = (float)rand() / (float)RAND_MAX * 2.0f - 1.0f;
        s = u * u + v * v;
    } while (s >= 1.0f || s == 0.0f);
    return u * sqrtf(-2.0f * logf(s) / s);
}

void orc_init_weights(const orc_config *c, float *p)
{
    /* same draw order as src/model.c:292-331: wte, wpe, then per layer
     * c_attn_w, c_proj_w (residual std), mlp_fc_w, mlp_proj_w (residual std) */
    long C = c->n_embd;
    float std = 0.02f, rstd = 0.02f / sqrtf(2.0f * (float)c->n_layer);
    float *q = p;
    for (long i = 0; i < (long)c->vocab_size * C; i++) *q++ = orc_randn() * std;
    for (long i = 0; i < (long)c->block_size * C; i++) *q++ = orc_randn() * std;
    for (int l = 0; l < c->n_layer; l++) {
        for (long i = 0; i < C; i++) *q++ = 1.0f;
        for (long i = 0; i < C; i++) *q++ = 0.0f;
        for (long i = 0; i < 3 * C * C; i++) *q++ = orc_randn() * std;
        for (long i = 0; i < 3 * C; i++) *q++ = 0.0f;
        for (long i = 0; i < C * C; i++) *q++ = orc_randn() * rstd;
        for (long i = 0; i < C; i++) *q++ = 0.0f;
        for (long i = 0; i < C; i++) *q++ = 1.0f;
        for (long i = 0; i < C; i++) *q++ = 0.0f;
        for (long i = 0; i < 4 * C * C; i++) *q++ = orc_randn() * std;
        for (long i = 0; i < 4 * C; i++) *q++ = 0.0f;
        for (long i = 0; i < 4 * C * C; i++) *q++ = orc_randn() * rstd;
        for (long i = 0; i < C; i++) *q++ = 0.0f;
    }
    for (long i = 0; i < C; i++) *q++ = 1.0f;
    for (long i = 0; i < C; i++) *q++ = 0.0f;
}

void orc_decay_mask(const orc_config *c, unsigned char *d)
{
    /* 2-D tensors (wte, wpe, the four weight matrices) decay; vectors do not
     * (src/model.c:148-172) */
    long C = c->n_embd;
    memset(d, 1, (size_t)((long)c->vocab_size * C + (long)c->block_size * C));
    d += (long)c->vocab_size * C + (long)c->block_size * C;
    for (int l = 0; l < c->n_layer; l++) {
        memset(d, 0, 2 * C);        d += 2 * C;
        memset(d, 1, 3 * C * C);    d += 3 * C * C;
        memset(d, 0, 3 * C);        d += 3 * C;
        memset(d, 1, C * C);        d += C * C;
        memset(d, 0, 3 * C);        d += 3 * C;
        memset(d, 1, 4 * C * C);    d += 4 * C * C;
        memset(d, 0, 4 * C);        d += 4 * C;
        memset(d, 1, 4 * C * C);    d += 4 * C * C;
        memset(d, 0, C);            d += C;
    }
    memset(d, 0, 2 * C);
}

/* saved forward state, the reference's activation arena minus dropout masks
 * (src/model.c:333-436) */
typedef struct {
    float *emb, *ln1, *m1, *r1, *qkv, *probs, *aout, *proj, *res1, *ln2, *m2, *r2,
          *fc, *gelu, *mp, *res2, *lnf, *mf, *rf, *logits, *pr;
} acts_t;

static float *xalloc(size_t n) { return calloc(n ? n : 1, sizeof(float)); }

static void acts_alloc(acts_t *a, const orc_config *c, int B, int T)
{
    size_t L = c->n_layer, C = c->n_embd, H = c->n_head, N = (size_t)B * T;
    a->emb = xalloc(N * C);
    a->ln1 = xalloc(L * N * C);  a->m1 = xalloc(L * N); a->r1 = xalloc(L * N);
    a->qkv = xalloc(L * N * 3 * C);
    a->probs = xalloc(L * B * H * T * T);
    a->aout = xalloc(L * N * C); a->proj = xalloc(L * N * C); a->res1 = xalloc(L * N * C);
    a->ln2 = xalloc(L * N * C);  a->m2 = xalloc(L * N); a->r2 = xalloc(L * N);
    a->fc = xalloc(L * N * 4 * C); a->gelu = xalloc(L * N * 4 * C);
    a->mp = xalloc(L * N * C);   a->res2 = xalloc(L * N * C);
    a->lnf = xalloc(N * C); a->mf = xalloc(N); a->rf = xalloc(N);
    a->logits = xalloc(N * c->vocab_size); a->pr = xalloc(N * c->vocab_size);
}

static void acts_free(acts_t *a)
{
    float **f = (float **)a;
    for (size_t i = 0; i < sizeof(*a) / sizeof(float *); i++) free(f[i]);
}

/* one causal attention head over packed qkv rows (src/model.c:514-563) */
static void attn_head(const float *qkv, float *probs, float *aout,
                      int T, int C, int hs, int h)
{
    float scale = 1.0f / sqrtf((float)hs);
    for (int i = 0; i < T; i++) {
        float *p = probs + (size_t)i * T;
        const float *q = qkv + (size_t)i * 3 * C + h * hs;
        for (int j = 0; j < T; j++) {
            const float *k = qkv + (size_t)j * 3 * C + C + h * hs;
            double acc = 0.0;
            for (int d = 0; d < hs; d++) acc += (double)q[d] * k[d];
            p[j] = (float)(scale * acc);
        }
    }
    orc_causal_mask(probs, T);
    orc_softmax_inplace(probs, T, T);
    for (int i = 0; i < T; i++)
        for (int d = 0; d < hs; d++) {
            double acc = 0.0;
            for (int j = 0; j < T; j++)
                acc += (double)probs[(size_t)i * T + j] * qkv[(size_t)j * 3 * C + 2 * C + h * hs + d];
            aout[(size_t)i * C + h * hs + d] = (float)acc;
        }
}

static float forward_impl(const orc_config *c, const float *params, const int *tok,
                          const int *tgt, int B, int T, acts_t *a)
{
    int L = c->n_layer, C = c->n_embd, H = c->n_head, V = c->vocab_size, hs = C / H;
    size_t N = (size_t)B * T;
    view_t g, w;
    view_global(c, params, &g);
    for (size_t i = 0; i < N; i++)                    /* src/model.c:460-470 */
        for (int k = 0; k < C; k++)
            a->emb[i * C + k] = g.wte[(size_t)tok[i] * C + k] + g.wpe[(i % T) * C + k];
    const float *x = a->emb;
    for (int l = 0; l < L; l++) {
        view_layer(c, params, l, &w);
        float *ln1 = a->ln1 + l * N * C, *qkv = a->qkv + l * N * 3 * C;
        float *aout = a->aout + l * N * C, *proj = a->proj + l * N * C;
        float *res1 = a->res1 + l * N * C, *ln2 = a->ln2 + l * N * C;
        float *fc = a->fc + l * N * 4 * C, *ge = a->gelu + l * N * 4 * C;
        float *mp = a->mp + l * N * C, *res2 = a->res2 + l * N * C;
        orc_layernorm_fwd(x, w.ln1w, w.ln1b, ln1, a->m1 + l * N, a->r1 + l * N, (int)N, C);
        orc_linear_fwd(ln1, w.attw, w.attb, qkv, (int)N, C, 3 * C);
        #pragma omp parallel for schedule(static)
        for (int bh = 0; bh < B * H; bh++) {
            int b = bh / H, h = bh % H;
            attn_head(qkv + (size_t)b * T * 3 * C,
                      a->probs + ((size_t)l * B * H + bh) * T * T,
                      aout + (size_t)b * T * C, T, C, hs, h);
        }
        orc_linear_fwd(aout, w.prjw, w.prjb, proj, (int)N, C, C);
        for (size_t i = 0; i < N * C; i++) res1[i] = x[i] + proj[i];   /* src/model.c:570-571 */
        orc_layernorm_fwd(res1, w.ln2w, w.ln2b, ln2, a->m2 + l * N, a->r2 + l * N, (int)N, C);
        orc_linear_fwd(ln2, w.fcw, w.fcb, fc, (int)N, C, 4 * C);
        orc_gelu_fwd(fc, ge, (int)(N * 4 * C));
        orc_linear_fwd(ge, w.mpw, w.mpb, mp, (int)N, 4 * C, C);
        for (size_t i = 0; i < N * C; i++) res2[i] = res1[i] + mp[i];   /* src/model.c:595-596 */
        x = res2;
    }
    orc_layernorm_fwd(x, g.lnfw, g.lnfb, a->lnf, a->mf, a->rf, (int)N, C);
    orc_linear_fwd(a->lnf, g.wte, NULL, a->logits, (int)N, C, V);     /* tied head, src/model.c:613 */
    if (!tgt) return 0.0f;
    float loss;
    orc_cross_entropy_fwd(a->logits, tgt, a->pr, &loss, B, T, V);
    return loss;
}

float orc_forward(const orc_config *c, const float *params, const int *tok,
                  const int *tgt, int B, int T, float *logits, float *probs)
{
    acts_t a;
    acts_alloc(&a, c, B, T);
    float loss = forward_impl(c, params, tok, tgt, B, T, &a);
    size_t n = (size_t)B * T * c->vocab_size;
    if (logits) memcpy(logits, a.logits, n * sizeof(float));
    if (probs) memcpy(probs, a.pr, n * sizeof(float));
    acts_free(&a);
    return loss;
}

/* gradient views share the parameter layout */
static float *gl(const orc_config *c, float *grads, int l)
{
    long C = c->n_embd;
    return grads + (long)c->vocab_size * C + (long)c->block_size * C + l * layer_size(C);
}

float orc_forward_backward(const orc_config *c, const float *params, const int *tok,
                           const int *tgt, int B, int T, float *grads)
{
    int L = c->n_layer, C = c->n_embd, H = c->n_head, V = c->vocab_size, hs = C / H;
    size_t N = (size_t)B * T;
    acts_t a;
    acts_alloc(&a, c, B, T);
    float loss = forward_impl(c, params, tok, tgt, B, T, &a);
    view_t g;
    view_global(c, params, &g);
    float *dlog = xalloc(N * V), *dlnf = xalloc(N * C), *dx = xalloc(N * C);
    float *dres1 = xalloc(N * C), *dln2 = xalloc(N * C), *dfc = xalloc(N * 4 * C);
    float *dge = xalloc(N * 4 * C), *dln1 = xalloc(N * C), *dqkv = xalloc(N * 3 * C);
    float *dao = xalloc(N * C);
    float *g_wte = grads, *g_wpe = grads + (long)V * C;
    float *g_lnf = gl(c, grads, L);
    /* src/model.c:665-685 */
    orc_cross_entropy_bwd(dlog, a.pr, tgt, 1.0f / (float)N, B, T, V);
    orc_linear_bwd_dx(dlog, g.wte, dlnf, (int)N, C, V);
    orc_linear_bwd_dw(dlog, a.lnf, g_wte, NULL, (int)N, C, V);
    orc_layernorm_bwd(dlnf, L > 0 ? a.res2 + (L - 1) * N * C : a.emb, g.lnfw, a.mf, a.rf,
                      dx, g_lnf, g_lnf + C, (int)N, C);
    float sc = 1.0f / sqrtf((float)hs);
    for (int l = L - 1; l >= 0; l--) {                 /* src/model.c:691-842 */
        view_t w;
        view_layer(c, params, l, &w);
        float *gw = gl(c, grads, l);
        float *g_ln1w = gw, *g_ln1b = gw + C, *g_attw = gw + 2 * C;
        float *g_attb = g_attw + 3 * C * C, *g_prjw = g_attb + 3 * C, *g_prjb = g_prjw + C * C;
        float *g_ln2w = g_prjb + C, *g_ln2b = g_ln2w + C, *g_fcw = g_ln2b + C;
        float *g_fcb = g_fcw + 4 * C * C, *g_mpw = g_fcb + 4 * C, *g_mpb = g_mpw + 4 * C * C;
        const float *x_in = l == 0 ? a.emb : a.res2 + (l - 1) * N * C;
        memcpy(dres1, dx, N * C * sizeof(float));
        memset(dge, 0, N * 4 * C * sizeof(float));
        orc_linear_bwd_dx(dx, w.mpw, dge, (int)N, 4 * C, C);
        orc_linear_bwd_dw(dx, a.gelu + l * N * 4 * C, g_mpw, g_mpb, (int)N, 4 * C, C);
        memset(dfc, 0, N * 4 * C * sizeof(float));
        orc_gelu_bwd(dge, a.fc + l * N * 4 * C, dfc, (int)(N * 4 * C));
        memset(dln2, 0, N * C * sizeof(float));
        orc_linear_bwd_dx(dfc, w.fcw, dln2, (int)N, C, 4 * C);
        orc_linear_bwd_dw(dfc, a.ln2 + l * N * C, g_fcw, g_fcb, (int)N, C, 4 * C);
        orc_layernorm_bwd(dln2, a.res1 + l * N * C, w.ln2w, a.m2 + l * N, a.r2 + l * N,
                          dres1, g_ln2w, g_ln2b, (int)N, C);
        memset(dao, 0, N * C * sizeof(float));
        orc_linear_bwd_dx(dres1, w.prjw, dao, (int)N, C, C);
        orc_linear_bwd_dw(dres1, a.aout + l * N * C, g_prjw, g_prjb, (int)N, C, C);
        memset(dqkv, 0, N * 3 * C * sizeof(float));
        const float *qkv = a.qkv + l * N * 3 * C;
        #pragma omp parallel for schedule(static)
        for (int bh = 0; bh < B * H; bh++) {           /* src/model.c:749-821 */
            int b = bh / H, h = bh % H;
            const float *P = a.probs + ((size_t)l * B * H + bh) * T * T;
            const float *q0 = qkv + (size_t)b * T * 3 * C;
            float *dq0 = dqkv + (size_t)b * T * 3 * C;
            const float *do0 = dao + (size_t)b * T * C;
            float *dp = malloc((size_t)T * T * sizeof(float));
            for (int i = 0; i < T; i++)                 /* dP = dO V^T */
                for (int j = 0; j < T; j++) {
                    double acc = 0.0;
                    for (int d = 0; d < hs; d++)
                        acc += (double)do0[(size_t)i * C + h * hs + d] * q0[(size_t)j * 3 * C + 2 * C + h * hs + d];
                    dp[(size_t)i * T + j] = (float)acc;
                }
            for (int j = 0; j < T; j++)                 /* dV = P^T dO */
                for (int d = 0; d < hs; d++) {
                    double acc = 0.0;
                    for (int i = 0; i < T; i++)
                        acc += (double)P[(size_t)i * T + j] * do0[(size_t)i * C + h * hs + d];
                    dq0[(size_t)j * 3 * C + 2 * C + h * hs + d] += (float)acc;
                }
            for (int i = 0; i < T; i++) {               /* dS = P (dP - sum P dP), lower triangle */
                float dot = 0.0f;
                for (int j = 0; j <= i; j++) dot += P[(size_t)i * T + j] * dp[(size_t)i * T + j];
                for (int j = 0; j <= i; j++)
                    dp[(size_t)i * T + j] = P[(size_t)i * T + j] * (dp[(size_t)i * T + j] - dot);
                for (int j = i + 1; j < T; j++) dp[(size_t)i * T + j] = 0.0f;
            }
            for (int i = 0; i < T; i++)                 /* dQ = sc dS K */
                for (int d = 0; d < hs; d++) {
                    double acc = 0.0;
                    for (int j = 0; j < T; j++)
                        acc += (double)dp[(size_t)i * T + j] * q0[(size_t)j * 3 * C + C + h * hs + d];
                    dq0[(size_t)i * 3 * C + h * hs + d] += (float)(sc * acc);
                }
            for (int j = 0; j < T; j++)                 /* dK = sc dS^T Q */
                for (int d = 0; d < hs; d++) {
                    double acc = 0.0;
                    for (int i = 0; i < T; i++)
                        acc += (double)dp[(size_t)i * T + j] * q0[(size_t)i * 3 * C + h * hs + d];
                    dq0[(size_t)j * 3 * C + C + h * hs + d] += (float)(sc * acc);
                }
            free(dp);
        }
        memset(dln1, 0, N * C * sizeof(float));
        orc_linear_bwd_dx(dqkv, w.attw, dln1, (int)N, C, 3 * C);
        orc_linear_bwd_dw(dqkv, a.ln1 + l * N * C, g_attw, g_attb, (int)N, C, 3 * C);
        memset(dx, 0, N * C * sizeof(float));
        orc_layernorm_bwd(dln1, x_in, w.ln1w, a.m1 + l * N, a.r1 + l * N, dx, g_ln1w, g_ln1b, (int)N, C);
        orc_residual_add(dx, dres1, (int)(N * C));
    }
    for (size_t i = 0; i < N; i++)                      /* src/model.c:853-867 */
        for (int k = 0; k < C; k++) g_wpe[(i % T) * C + k] += dx[i * C + k];
    for (size_t i = 0; i < N; i++)
        for (int k = 0; k < C; k++) g_wte[(size_t)tok[i] * C + k] += dx[i * C + k];
    free(dlog); free(dlnf); free(dx); free(dres1); free(dln2);
    free(dfc); free(dge); free(dln1); free(dqkv); free(dao);
    acts_free(&a);
    return loss;
}

void orc_adamw(float *p, float *g, float *m, float *v, const unsigned char *decay,
               long n, int *step, float lr, float b1, float b2, float eps, float wd,
               float clip)
{
    /* src/model.c:891-920 */
    *step += 1;
    if (clip > 0.0f) {
        float norm = orc_global_grad_norm(g, (int)n);
        if (norm > clip) orc_scale_grads(g, (int)n, clip / norm);
    }
    float bc1 = 1.0f - powf(b1, (float)*step), bc2 = 1.0f - powf(b2, (float)*step);
    for (long i = 0; i < n; i++) {
        m[i] = b1 * m[i] + (1.0f - b1) * g[i];
        v[i] = b2 * v[i] + (1.0f - b2) * g[i] * g[i];
        float mh = m[i] / bc1, vh = v[i] / bc2;
        float ewd = decay[i] ? wd : 0.0f;
        p[i] = p[i] * (1.0f - lr * ewd) - lr * mh / (sqrtf(vh) + eps);
    }
}

void orc_forward_last(const orc_config *c, const float *params, const int *tok,
                      int B, int T, float *out)
{
    /* gpt_forward_fast returns the final position of each sequence
     * (src/fast.c:300-329); that equals gpt_forward's row T-1 */
    size_t V = c->vocab_size;
    float *logits = malloc((size_t)B * T * V * sizeof(float));
    orc_forward(c, params, tok, NULL, B, T, logits, NULL);
    for (int b = 0; b < B; b++)
        memcpy(out + b * V, logits + ((size_t)b * T + T - 1) * V, V * sizeof(float));
    free(logits);
}
