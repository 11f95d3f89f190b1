// model_abi.cu - the C entry points of cngpt/model.h on the device.
//
// Same names, arguments, arena layouts and return conventions as the
// reference's src/model.c; the arithmetic runs in this library's kernels:
//
//   forward  (src/model.c:442-625): embedding, per layer LN1 -> QKV GEMM(+bias)
//            -> fused causal attention (saves row LSE) -> c_proj GEMM with the
//            residual add fused (writes attn_proj and res1) -> LN2 -> fc GEMM
//            with bias+GELU fused (writes mlp_fc_out and mlp_gelu) -> proj GEMM
//            with the residual fused (mlp_proj_out, res2); LN_f; tied LM head;
//            cross-entropy writing probs, the row NLL terms and (for the
//            backward) dlogits in one pass.
//   backward (src/model.c:634-873): LM-head dX/dW GEMMs, LN_f backward, per
//            layer: mlp_proj dX GEMM with GELU-backward fused, dW GEMMs
//            accumulating into the gradient arena plus deterministic bias
//            column sums, LayerNorm backward accumulating straight into the
//            running residual gradient, fused attention backward, embedding
//            scatter in position order.
//   AdamW    (src/model.c:888-921): device grad norm -> clip factor -> one
//            fused update pass.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "abi_common.h"
#include "kernels.h"
#include "model_ctx.h"

extern "C" {
#include "cngpt_cuda.h"
}

namespace cg {

namespace {
std::mutex g_mu;
std::unordered_map<const GPT *, ModelCtx *> g_models;
std::unordered_map<const FastCtx *, FastDev *> g_fast;
}  // namespace

ModelCtx *model_ctx(const GPT *m) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_models.find(m);
    if (it == g_models.end()) {
        set_last_error(ERR_STATE, "model %p was not initialised by gpt_init/gpt_load", (const void *)m);
        return nullptr;
    }
    return it->second;
}

FastDev *fast_dev(const FastCtx *f, bool create) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_fast.find(f);
    if (it != g_fast.end()) return it->second;
    if (!create) return nullptr;
    FastDev *d = new FastDev();
    g_fast[f] = d;
    return d;
}

void fast_forget(const FastCtx *f) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_fast.find(f);
    if (it != g_fast.end()) {
        delete it->second;
        g_fast.erase(it);
    }
}

int dev_alloc(void **p, size_t bytes, bool managed) {
    *p = nullptr;
    if (bytes == 0) bytes = 16;
    cudaError_t e = managed ? cudaMallocManaged(p, bytes) : cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        *p = nullptr;
        set_last_error(ERR_ALLOC, "device allocation of %zu bytes failed: %s", bytes,
                       cudaGetErrorString(e));
        return ERR_ALLOC;
    }
    return OK;
}

void dev_free(void *p) {
    if (p) cudaFree(p);
}

int stage_tokens(const int *src, size_t n, int **buf, size_t *cap, const int **out, cudaStream_t s) {
    if (!src) {
        *out = nullptr;
        return OK;
    }
    if (mem_kind(src) != MEM_HOST) {
        *out = src;
        return OK;
    }
    if (n > *cap) {
        dev_free(*buf);
        *buf = nullptr;
        *cap = 0;
        CG_TRY(dev_alloc((void **)buf, n * sizeof(int), false));
        *cap = n;
    }
    CG_CUDA(cudaMemcpyAsync(*buf, src, n * sizeof(int), cudaMemcpyHostToDevice, s));
    *out = *buf;
    return OK;
}

namespace {

long layer_floats(long C) { return 12 * C * C + 13 * C; }

// pointer views in the reference's flat order (src/model.c:54-83)
void assign_weights(GPTWeights *w, float *buf, const GPTConfig *cfg) {
    const long C = cfg->n_embd, V = cfg->vocab_size, T = cfg->block_size;
    float *p = buf;
    w->wte = p; p += V * C;
    w->wpe = p; p += T * C;
    for (int l = 0; l < cfg->n_layer; l++) {
        w->ln1_w[l] = p; p += C;
        w->ln1_b[l] = p; p += C;
        w->c_attn_w[l] = p; p += 3 * C * C;
        w->c_attn_b[l] = p; p += 3 * C;
        w->c_proj_w[l] = p; p += C * C;
        w->c_proj_b[l] = p; p += C;
        w->ln2_w[l] = p; p += C;
        w->ln2_b[l] = p; p += C;
        w->mlp_fc_w[l] = p; p += 4 * C * C;
        w->mlp_fc_b[l] = p; p += 4 * C;
        w->mlp_proj_w[l] = p; p += C * 4 * C;
        w->mlp_proj_b[l] = p; p += C;
    }
    w->ln_f_w = p; p += C;
    w->ln_f_b = p;
}

int alloc_weight_ptrs(GPTWeights *w, int L) {
    float ***f[] = {&w->ln1_w, &w->ln1_b, &w->c_attn_w, &w->c_attn_b, &w->c_proj_w, &w->c_proj_b,
                    &w->ln2_w, &w->ln2_b, &w->mlp_fc_w, &w->mlp_fc_b, &w->mlp_proj_w, &w->mlp_proj_b};
    for (auto pp : f) {
        *pp = (float **)calloc((size_t)(L > 0 ? L : 1), sizeof(float *));
        if (!*pp) return -1;
    }
    return 0;
}

void free_weight_ptrs(GPTWeights *w) {
    free(w->ln1_w); free(w->ln1_b); free(w->c_attn_w); free(w->c_attn_b);
    free(w->c_proj_w); free(w->c_proj_b); free(w->ln2_w); free(w->ln2_b);
    free(w->mlp_fc_w); free(w->mlp_fc_b); free(w->mlp_proj_w); free(w->mlp_proj_b);
}

void free_act_ptrs(GPTActivations *a) {
    float **f[] = {a->ln1_out, a->ln1_mean, a->ln1_rstd, a->qkv, a->attn_scores, a->attn_probs,
                   a->attn_out, a->attn_proj, a->res1, a->ln2_out, a->ln2_mean, a->ln2_rstd,
                   a->mlp_fc_out, a->mlp_gelu, a->mlp_proj_out, a->res2};
    for (auto p : f) free(p);
    free(a->res1_mask);
    free(a->res2_mask);
}

// Marsaglia polar normal from the C library rand() stream; the draw order
// and arithmetic follow src/model.c:275-290 so the weights equal the
// reference's bit for bit for the same stream.
float polar_randn() {
    float u, v, s;
    do {
        u = (float)rand() / (float)RAND_MAX * 2.0f - 1.0f;
        v = (float)rand() / (float)RAND_MAX * 2.0f - 1.0f;
        s = u * u + v * v;
    } while (s >= 1.0f || s == 0.0f);
    return u * sqrtf(-2.0f * logf(s) / s);
}

void sync_if_managed(ModelCtx *c) {
    if (c->managed) cudaStreamSynchronize(g_stream);
}

// byte offset of the fused cross-entropy partials in the model's scratch,
// after the BT row terms
size_t ce_part_offset(size_t BT) { return (BT * sizeof(float) + 255) & ~(size_t)255; }

// extras sized for B*T rows
int ensure_extras(GPT *m, ModelCtx *c, int B, int T) {
    const size_t BT = (size_t)B * T;
    const long C = m->cfg.n_embd, V = m->cfg.vocab_size, H = m->cfg.n_head;
    if (BT <= c->extra_BT && c->dlogits) return OK;
    cudaStreamSynchronize(g_stream);
    float **bufs[] = {&c->dlogits, &c->d_x, &c->d_ln, &c->d_mlp, &c->d_ao, &c->d_qkv, &c->scratch};
    for (auto b : bufs) {
        dev_free(*b);
        *b = nullptr;
    }
    dev_free(c->tok);
    dev_free(c->tgt);
    c->tok = c->tgt = nullptr;
    c->extra_BT = 0;
    c->ldlog = (V + 3) & ~3L;
    CG_TRY(dev_alloc((void **)&c->dlogits, BT * c->ldlog * sizeof(float), false));
    CG_TRY(dev_alloc((void **)&c->d_x, BT * C * sizeof(float), false));
    CG_TRY(dev_alloc((void **)&c->d_ln, BT * C * sizeof(float), false));
    CG_TRY(dev_alloc((void **)&c->d_mlp, BT * 4 * C * sizeof(float), false));
    CG_TRY(dev_alloc((void **)&c->d_ao, BT * C * sizeof(float), false));
    CG_TRY(dev_alloc((void **)&c->d_qkv, BT * 3 * C * sizeof(float), false));
    size_t sb = layernorm_bwd_scratch_bytes((int)BT, (int)C, kLnBwdTrainRows);
    sb = std::max(sb, colsum_scratch_bytes((int)BT, (int)(4 * C)));
    sb = std::max(sb, layernorm_bwd_fused_scratch_bytes((int)BT, (int)C));
    sb = std::max(sb, attention_bwd_scratch_bytes(B, T, (int)H));
    sb = std::max(sb, BT * sizeof(float));  // CE row terms
    // fused LM-head + cross-entropy: row terms, then the per-64-column
    // (max, sum exp) pairs of every row
    sb = std::max(sb, ce_part_offset(BT) + BT * (size_t)((V + 63) / 64) * sizeof(float2));
    sb = std::max(sb, norm_scratch_bytes());
    c->scratch_bytes = sb;
    CG_TRY(dev_alloc((void **)&c->scratch, sb, false));
    CG_TRY(dev_alloc((void **)&c->tok, BT * sizeof(int), false));
    CG_TRY(dev_alloc((void **)&c->tgt, BT * sizeof(int), false));
    c->extra_BT = BT;
    return OK;
}

}  // namespace

int resize_acts(GPT *m, ModelCtx *c, int B, int T) {
    const size_t C = m->cfg.n_embd, V = m->cfg.vocab_size, L = m->cfg.n_layer, H = m->cfg.n_head;
    const size_t BT = (size_t)B * T;
    // totals exactly as src/model.c:341-371
    const size_t per_layer = BT * C + BT + BT + BT * 3 * C + (size_t)B * H * T * T * 2 + BT * C * 3 +
                             BT * C + BT + BT + BT * 4 * C * 2 + BT * C + BT * C;
    const size_t total = BT * C + per_layer * L + BT * C + BT + BT + BT * V + BT * V;
    const size_t mask_total = BT * C + BT * C * L * 2;
    if (total > c->act_cap || mask_total > c->mask_cap) {
        cudaStreamSynchronize(g_stream);
        dev_free(m->act_buf);
        dev_free(m->mask_buf);
        m->act_buf = nullptr;
        m->mask_buf = nullptr;
        c->act_cap = c->mask_cap = 0;
        CG_TRY(dev_alloc((void **)&m->act_buf, total * sizeof(float), c->managed));
        CG_TRY(dev_alloc((void **)&m->mask_buf, mask_total, c->managed));
        c->act_cap = total;
        c->mask_cap = mask_total;
    }
    GPTActivations *a = &m->acts;
    if (!a->ln1_out) {
        float ***f[] = {&a->ln1_out, &a->ln1_mean, &a->ln1_rstd, &a->qkv, &a->attn_scores,
                        &a->attn_probs, &a->attn_out, &a->attn_proj, &a->res1, &a->ln2_out,
                        &a->ln2_mean, &a->ln2_rstd, &a->mlp_fc_out, &a->mlp_gelu, &a->mlp_proj_out,
                        &a->res2};
        for (auto pp : f) *pp = (float **)calloc(L ? L : 1, sizeof(float *));
        a->res1_mask = (unsigned char **)calloc(L ? L : 1, sizeof(unsigned char *));
        a->res2_mask = (unsigned char **)calloc(L ? L : 1, sizeof(unsigned char *));
        if (!a->ln1_out || !a->res2 || !a->res2_mask) {
            set_last_error(ERR_ALLOC, "host pointer arrays");
            return ERR_ALLOC;
        }
    }
    // pointer assignment exactly as src/model.c:402-433
    float *p = m->act_buf;
    unsigned char *mp = m->mask_buf;
    a->emb = p; p += BT * C;
    a->emb_mask = mp; mp += BT * C;
    for (size_t l = 0; l < L; l++) {
        a->ln1_out[l] = p; p += BT * C;
        a->ln1_mean[l] = p; p += BT;
        a->ln1_rstd[l] = p; p += BT;
        a->qkv[l] = p; p += BT * 3 * C;
        a->attn_scores[l] = p; p += (size_t)B * H * T * T;
        a->attn_probs[l] = p; p += (size_t)B * H * T * T;
        a->attn_out[l] = p; p += BT * C;
        a->attn_proj[l] = p; p += BT * C;
        a->res1[l] = p; p += BT * C;
        a->ln2_out[l] = p; p += BT * C;
        a->ln2_mean[l] = p; p += BT;
        a->ln2_rstd[l] = p; p += BT;
        a->mlp_fc_out[l] = p; p += BT * 4 * C;
        a->mlp_gelu[l] = p; p += BT * 4 * C;
        a->mlp_proj_out[l] = p; p += BT * C;
        a->res2[l] = p; p += BT * C;
        a->res1_mask[l] = mp; mp += BT * C;
        a->res2_mask[l] = mp; mp += BT * C;
    }
    a->ln_f_out = p; p += BT * C;
    a->ln_f_mean = p; p += BT;
    a->ln_f_rstd = p; p += BT;
    a->logits = p; p += BT * V;
    a->probs = p;
    c->B = B;
    c->T = T;
    return ensure_extras(m, c, B, T);
}

// ------------------------------------------------------------ forward
// fused_ce (training step): the LM-head GEMM writes the logits straight into
// the dlogits buffer and forms each row's softmax statistics in its epilogue;
// one pass then turns the rows into dlogits in place. The arena's logits and
// probs slots are not written. Otherwise logits and probs land in the arena
// as in the reference.
int forward(GPT *m, ModelCtx *c, const int *tokens, const int *targets, int B, int T, bool want_grad,
            cudaStream_t s, bool fused_ce = false) {
    const int C = m->cfg.n_embd, V = m->cfg.vocab_size, L = m->cfg.n_layer, H = m->cfg.n_head;
    const int BT = B * T;
    if (B <= 0 || T <= 0 || T > m->cfg.block_size || H <= 0 || C % H != 0) {
        set_last_error(ERR_ARG, "gpt_forward: bad shape B=%d T=%d (block %d) C=%d H=%d", B, T,
                       m->cfg.block_size, C, H);
        return ERR_ARG;
    }
    CG_TRY(resize_acts(m, c, B, T));
    const int *tok = nullptr, *tgt = nullptr;
    size_t cap = c->extra_BT;
    CG_TRY(stage_tokens(tokens, BT, &c->tok, &cap, &tok, s));
    CG_TRY(stage_tokens(targets, BT, &c->tgt, &cap, &tgt, s));
    const bool training = targets && m->cfg.dropout > 0.0f;
    GPTActivations *a = &m->acts;
    GPTWeights *w = &m->params;
    CG_TRY(embed_fwd(tok, w->wte, w->wpe, a->emb, BT, T, C, 0, s));
    if (training) dropout_fwd(a->emb, a->emb_mask, BT * C, m->cfg.dropout);
    const float *x = a->emb;
    for (int l = 0; l < L; l++) {
        CG_TRY(layernorm_fwd(x, C, w->ln1_w[l], w->ln1_b[l], a->ln1_out[l], C, a->ln1_mean[l],
                             a->ln1_rstd[l], BT, C, s));
        GemmEpi e;
        e.mode = EPI_STORE;
        e.D = a->qkv[l];
        e.ldd = 3 * C;
        e.bias = w->c_attn_b[l];
        CG_TRY(gemm(a->ln1_out[l], C, false, w->c_attn_w[l], C, false, BT, 3 * C, C, e, s));
        CG_TRY(attention_fwd(a->qkv[l], a->attn_out[l], a->attn_scores[l], B, T, C, H, s));
        e = GemmEpi();
        e.mode = EPI_RESID;
        e.D = a->attn_proj[l];
        e.ldd = C;
        e.bias = w->c_proj_b[l];
        e.D2 = a->res1[l];
        e.ldd2 = C;
        e.R = x;
        e.ldr = C;
        CG_TRY(gemm(a->attn_out[l], C, false, w->c_proj_w[l], C, false, BT, C, C, e, s));
        if (training) dropout_fwd(a->res1[l], a->res1_mask[l], BT * C, m->cfg.dropout);
        CG_TRY(layernorm_fwd(a->res1[l], C, w->ln2_w[l], w->ln2_b[l], a->ln2_out[l], C,
                             a->ln2_mean[l], a->ln2_rstd[l], BT, C, s));
        e = GemmEpi();
        e.mode = EPI_GELU;
        e.D = a->mlp_fc_out[l];
        e.ldd = 4 * C;
        e.bias = w->mlp_fc_b[l];
        e.D2 = a->mlp_gelu[l];
        e.ldd2 = 4 * C;
        CG_TRY(gemm(a->ln2_out[l], C, false, w->mlp_fc_w[l], C, false, BT, 4 * C, C, e, s));
        e = GemmEpi();
        e.mode = EPI_RESID;
        e.D = a->mlp_proj_out[l];
        e.ldd = C;
        e.bias = w->mlp_proj_b[l];
        e.D2 = a->res2[l];
        e.ldd2 = C;
        e.R = a->res1[l];
        e.ldr = C;
        CG_TRY(gemm(a->mlp_gelu[l], 4 * C, false, w->mlp_proj_w[l], 4 * C, false, BT, C, 4 * C, e, s));
        if (training) dropout_fwd(a->res2[l], a->res2_mask[l], BT * C, m->cfg.dropout);
        x = a->res2[l];
    }
    CG_TRY(layernorm_fwd(x, C, w->ln_f_w, w->ln_f_b, a->ln_f_out, C, a->ln_f_mean, a->ln_f_rstd, BT,
                         C, s));
    c->dlogits_valid = false;
    c->fwd_targets = targets;
    float *rowterm = c->scratch;
    if (fused_ce && targets && want_grad) {
        // src/model.c:612-623 and 644-665 in two kernels: logits with row
        // statistics, then loss terms and dlogits
        float2 *part = (float2 *)((char *)c->scratch + ce_part_offset(BT));
        GemmEpi e;
        e.mode = EPI_STORE;
        e.D = c->dlogits;
        e.ldd = c->ldlog;
        e.ce_part = part;
        e.ce_ld = (V + 63) / 64;
        CG_TRY(gemm(a->ln_f_out, C, false, w->wte, C, false, BT, V, C, e, s));
        CG_TRY(cross_entropy_fused(c->dlogits, c->ldlog, part, e.ce_ld, tgt, 1.0f / (float)BT, rowterm, BT, V, s));
        CG_TRY(cross_entropy_loss(rowterm, BT, &c->dev_scalars[0], s));
        c->dlogits_valid = true;
        return OK;
    }
    GemmEpi e;
    e.mode = EPI_STORE;
    e.D = a->logits;
    e.ldd = V;
    CG_TRY(gemm(a->ln_f_out, C, false, w->wte, C, false, BT, V, C, e, s));
    if (!targets) return OK;
    CG_TRY(cross_entropy_rows(a->logits, V, tgt, a->probs, V, want_grad ? c->dlogits : nullptr,
                              c->ldlog, 1.0f / (float)BT, rowterm, BT, V, s));
    CG_TRY(cross_entropy_loss(rowterm, BT, &c->dev_scalars[0], s));
    c->dlogits_valid = want_grad;
    return OK;
}

// ------------------------------------------------------------ backward
// Data-parallel gradient buckets (world > 1, from the training step): each
// layer's gradient range is final once its iteration of the backward loop has
// run (src/model.c:691-842; the ranges are contiguous, src/model.c:66-79), so
// it is averaged over the ranks on the communication stream while the
// backward continues below it. The last layer's bucket also takes ln_f (final
// after the LN_f backward, and next in the arena); wte and wpe, which the
// embedding backward completes last, form the final bucket.
int grad_bucket(GPT *m, ModelCtx *c, size_t off, size_t n, cudaStream_t s) {
    CG_CUDA(cudaEventRecord(c->ev_ready, s));
    CG_CUDA(cudaStreamWaitEvent(c->comm_stream, c->ev_ready, 0));
    return dp_allreduce(c, m->grad_buf + off, n, c->comm_stream);
}

int backward(GPT *m, ModelCtx *c, const int *tokens, const int *targets, int B, int T, cudaStream_t s,
             bool dp_buckets = false) {
    const int C = m->cfg.n_embd, V = m->cfg.vocab_size, L = m->cfg.n_layer, H = m->cfg.n_head;
    const int BT = B * T;
    if (B != c->B || T != c->T || !m->act_buf) {
        set_last_error(ERR_STATE, "gpt_backward: shape (%d,%d) does not match the last forward (%d,%d)",
                       B, T, c->B, c->T);
        return ERR_STATE;
    }
    const int *tok = nullptr, *tgt = nullptr;
    size_t cap = c->extra_BT;
    CG_TRY(stage_tokens(tokens, BT, &c->tok, &cap, &tok, s));
    GPTActivations *a = &m->acts;
    GPTWeights *w = &m->params, *g = &m->grads;
    // dlogits = (probs - onehot) / BT, unless the forward already produced it
    // for these same targets (src/model.c:665)
    if (!(c->dlogits_valid && targets == c->fwd_targets)) {
        CG_TRY(stage_tokens(targets, BT, &c->tgt, &cap, &tgt, s));
        if (!tgt) {
            set_last_error(ERR_ARG, "gpt_backward: targets required");
            return ERR_ARG;
        }
        CG_TRY(ce_grad(a->probs, V, tgt, 1.0f / (float)BT, c->dlogits, c->ldlog, BT, V, s));
    }
    float *scr = c->scratch;
    // Without dropout the LayerNorm backward passes fold in the column sums
    // that follow them: dw / db, and the bias gradient of the projection
    // whose output gradient the updated residual gradient is (mlp_proj after
    // LN_f / LN1 of the layer above, c_proj after LN2). Dropout masks d_x
    // between the two, so with dropout the separate passes run.
    const bool fuse_ln = m->cfg.dropout <= 0.0f && C % 128 == 0 && C <= 1024;
    auto ln_bwd = [&](const float *x_in, const float *lw, const float *mean, const float *rstd, float *gw, float *gb,
                      float *bias_grad) -> int {
        if (fuse_ln && layernorm_bwd_fused_ok(C, c->d_ln, x_in, lw, c->d_x))
            return layernorm_bwd_fused(c->d_ln, x_in, lw, mean, rstd, c->d_x, gw, gb, bias_grad, BT, C, scr, s);
        CG_TRY(layernorm_bwd(c->d_ln, x_in, lw, mean, rstd, c->d_x, gw, gb, BT, C, scr, s, kLnBwdTrainRows));
        // unaligned rows: the bias column sum as its own pass, at the same point
        return fuse_ln && bias_grad ? colsum_add(c->d_x, C, BT, C, bias_grad, scr, s) : OK;
    };
    // LM head (src/model.c:672-674): d_ln_f = dlogits wte ; d_wte += dlogits^T ln_f_out
    GemmEpi e;
    e.mode = EPI_STORE;
    e.D = c->d_ln;
    e.ldd = C;
    CG_TRY(gemm(c->dlogits, c->ldlog, false, w->wte, C, true, BT, C, V, e, s));
    e = GemmEpi();
    e.mode = EPI_ACCUM;
    e.D = g->wte;
    e.ldd = C;
    CG_TRY(gemm(c->dlogits, c->ldlog, true, a->ln_f_out, C, true, V, C, BT, e, s));
    // LN_f (src/model.c:680-685): d_x = 0 + LN_f backward
    CG_CUDA(cudaMemsetAsync(c->d_x, 0, (size_t)BT * C * sizeof(float), s));
    CG_TRY(ln_bwd(L > 0 ? a->res2[L - 1] : a->emb, w->ln_f_w, a->ln_f_mean, a->ln_f_rstd, g->ln_f_w, g->ln_f_b,
                  L > 0 ? g->mlp_proj_b[L - 1] : nullptr));
    for (int l = L - 1; l >= 0; l--) {
        const float *x_in = (l == 0) ? a->emb : a->res2[l - 1];
        if (m->cfg.dropout > 0.0f) dropout_bwd(c->d_x, a->res2_mask[l], BT * C, m->cfg.dropout);
        // mlp_proj dX with the GELU backward fused: d_mlp = (d_x W) * gelu'(fc_out)
        e = GemmEpi();
        e.mode = EPI_GELU_BWD;
        e.D = c->d_mlp;
        e.ldd = 4 * C;
        e.G = a->mlp_fc_out[l];
        e.ldg = 4 * C;
        CG_TRY(gemm(c->d_x, C, false, w->mlp_proj_w[l], 4 * C, true, BT, 4 * C, C, e, s));
        e = GemmEpi();
        e.mode = EPI_ACCUM;
        e.D = g->mlp_proj_w[l];
        e.ldd = 4 * C;
        CG_TRY(gemm(c->d_x, C, true, a->mlp_gelu[l], 4 * C, true, C, 4 * C, BT, e, s));
        if (!fuse_ln) CG_TRY(colsum_add(c->d_x, C, BT, C, g->mlp_proj_b[l], scr, s));
        // fc (src/model.c:716-720)
        e = GemmEpi();
        e.mode = EPI_STORE;
        e.D = c->d_ln;
        e.ldd = C;
        CG_TRY(gemm(c->d_mlp, 4 * C, false, w->mlp_fc_w[l], C, true, BT, C, 4 * C, e, s));
        e = GemmEpi();
        e.mode = EPI_ACCUM;
        e.D = g->mlp_fc_w[l];
        e.ldd = C;
        CG_TRY(gemm(c->d_mlp, 4 * C, true, a->ln2_out[l], C, true, 4 * C, C, BT, e, s));
        CG_TRY(colsum_add(c->d_mlp, 4 * C, BT, 4 * C, g->mlp_fc_b[l], scr, s));
        // LN2 accumulates into the residual gradient: d_x becomes d_res1
        CG_TRY(ln_bwd(a->res1[l], w->ln2_w[l], a->ln2_mean[l], a->ln2_rstd[l], g->ln2_w[l], g->ln2_b[l],
                      g->c_proj_b[l]));
        if (m->cfg.dropout > 0.0f) dropout_bwd(c->d_x, a->res1_mask[l], BT * C, m->cfg.dropout);
        // c_proj (src/model.c:736-740)
        e = GemmEpi();
        e.mode = EPI_STORE;
        e.D = c->d_ao;
        e.ldd = C;
        CG_TRY(gemm(c->d_x, C, false, w->c_proj_w[l], C, true, BT, C, C, e, s));
        e = GemmEpi();
        e.mode = EPI_ACCUM;
        e.D = g->c_proj_w[l];
        e.ldd = C;
        CG_TRY(gemm(c->d_x, C, true, a->attn_out[l], C, true, C, C, BT, e, s));
        if (!fuse_ln) CG_TRY(colsum_add(c->d_x, C, BT, C, g->c_proj_b[l], scr, s));
        // attention (src/model.c:742-822)
        CG_TRY(attention_bwd(a->qkv[l], a->attn_out[l], c->d_ao, a->attn_scores[l], c->d_qkv, scr, B,
                             T, C, H, s));
        // c_attn (src/model.c:825-829)
        e = GemmEpi();
        e.mode = EPI_STORE;
        e.D = c->d_ln;
        e.ldd = C;
        CG_TRY(gemm(c->d_qkv, 3 * C, false, w->c_attn_w[l], C, true, BT, C, 3 * C, e, s));
        e = GemmEpi();
        e.mode = EPI_ACCUM;
        e.D = g->c_attn_w[l];
        e.ldd = C;
        CG_TRY(gemm(c->d_qkv, 3 * C, true, a->ln1_out[l], C, true, 3 * C, C, BT, e, s));
        CG_TRY(colsum_add(c->d_qkv, 3 * C, BT, 3 * C, g->c_attn_b[l], scr, s));
        // LN1 accumulates into d_x (= d_res1 + LN1 backward, src/model.c:833-840)
        CG_TRY(ln_bwd(x_in, w->ln1_w[l], a->ln1_mean[l], a->ln1_rstd[l], g->ln1_w[l], g->ln1_b[l],
                      l > 0 ? g->mlp_proj_b[l - 1] : nullptr));
        if (dp_buckets) {
            const size_t off = (size_t)(g->ln1_w[l] - m->grad_buf);
            const size_t n = l == L - 1 ? (size_t)m->n_params - off : (size_t)layer_floats(C);
            CG_TRY(grad_bucket(m, c, off, n, s));
        }
    }
    if (m->cfg.dropout > 0.0f) dropout_bwd(c->d_x, a->emb_mask, BT * C, m->cfg.dropout);
    // embeddings (src/model.c:852-867)
    CG_TRY(embed_bwd(tok, c->d_x, g->wte, g->wpe, B, T, C, s));
    if (dp_buckets) {
        const size_t n_emb = (size_t)(g->ln1_w && L > 0 ? g->ln1_w[0] - m->grad_buf : m->n_params);
        CG_TRY(grad_bucket(m, c, 0, n_emb, s));
        // the optimizer waits for every bucket
        CG_CUDA(cudaEventRecord(c->ev_done, c->comm_stream));
        CG_CUDA(cudaStreamWaitEvent(s, c->ev_done, 0));
    }
    return OK;
}

int adamw_step(GPT *m, ModelCtx *c, float lr, float b1, float b2, float eps, float wd, float clip,
               cudaStream_t s) {
    m->step++;
    float *clip_factor = nullptr;
    if (clip > 0.0f) {
        CG_TRY(grad_norm(m->grad_buf, m->n_params, c->norm_scratch, &c->dev_scalars[1],
                         &c->dev_scalars[2], clip, s));
        clip_factor = &c->dev_scalars[2];
    }
    const float bc1 = 1.0f - powf(b1, (float)m->step);
    const float bc2 = 1.0f - powf(b2, (float)m->step);
    return adamw(m->param_buf, m->grad_buf, m->m_buf, m->v_buf, m->decay_buf, m->n_params, clip_factor,
                 lr, b1, b2, eps, wd, bc1, bc2, s);
}

}  // namespace cg

using namespace cg;

// ============================================================ model.h

extern "C" int gpt_num_params(const GPTConfig *cfg) {
    const long C = cfg->n_embd, V = cfg->vocab_size, T = cfg->block_size, L = cfg->n_layer;
    return (int)(V * C + T * C + L * layer_floats(C) + 2 * C);  // src/model.c:20-48
}

extern "C" int gpt_init(GPT *m, GPTConfig cfg) {
    memset(m, 0, sizeof(*m));
    m->cfg = cfg;
    const int L = cfg.n_layer;
    if (alloc_weight_ptrs(&m->params, L) != 0 || alloc_weight_ptrs(&m->grads, L) != 0) return -1;
    m->n_params = gpt_num_params(&cfg);
    ModelCtx *c = new ModelCtx();
    c->cfg = cfg;
    c->managed = g_managed;
    const size_t n = (size_t)m->n_params;
    if (dev_alloc((void **)&m->param_buf, n * 4, c->managed) || dev_alloc((void **)&m->grad_buf, n * 4, c->managed) ||
        dev_alloc((void **)&m->m_buf, n * 4, c->managed) || dev_alloc((void **)&m->v_buf, n * 4, c->managed) ||
        dev_alloc((void **)&m->decay_buf, n, c->managed) ||
        dev_alloc((void **)&c->dev_scalars, 16 * sizeof(float), false) ||
        dev_alloc((void **)&c->norm_scratch, norm_scratch_bytes(), false) ||
        cudaMallocHost((void **)&c->host_loss, sizeof(float)) != cudaSuccess) {
        delete c;
        return -1;
    }
    cudaMemsetAsync(m->param_buf, 0, n * 4, g_stream);
    cudaMemsetAsync(m->grad_buf, 0, n * 4, g_stream);
    cudaMemsetAsync(m->m_buf, 0, n * 4, g_stream);
    cudaMemsetAsync(m->v_buf, 0, n * 4, g_stream);
    cudaMemsetAsync(c->dev_scalars, 0, 16 * sizeof(float), g_stream);
    assign_weights(&m->params, m->param_buf, &cfg);
    assign_weights(&m->grads, m->grad_buf, &cfg);
    // decay mask: 2-D tensors decay, vectors do not (src/model.c:148-172)
    {
        const size_t C = cfg.n_embd, V = cfg.vocab_size, T = cfg.block_size;
        std::vector<uint8_t> d(n, 0);
        uint8_t *q = d.data();
        memset(q, 1, V * C + T * C);
        q += V * C + T * C;
        for (int l = 0; l < L; l++) {
            q += 2 * C;
            memset(q, 1, 3 * C * C); q += 3 * C * C + 3 * C;
            memset(q, 1, C * C);     q += C * C + 3 * C;
            memset(q, 1, 4 * C * C); q += 4 * C * C + 4 * C;
            memset(q, 1, 4 * C * C); q += 4 * C * C + C;
        }
        if (cudaMemcpy(m->decay_buf, d.data(), n, cudaMemcpyHostToDevice) != cudaSuccess) {
            set_last_error(ERR_CUDA, "decay mask upload");
            delete c;
            return -1;
        }
    }
    {
        std::lock_guard<std::mutex> lk(g_mu);
        g_models[m] = c;
    }
    if (cudaStreamSynchronize(g_stream) != cudaSuccess) return -1;
    return 0;
}

extern "C" void gpt_init_weights(GPT *m) {
    ModelCtx *c = model_ctx(m);
    if (!c) return;
    const long C = m->cfg.n_embd, V = m->cfg.vocab_size, L = m->cfg.n_layer;
    const float std = 0.02f, rstd = 0.02f / sqrtf(2.0f * (float)L);
    std::vector<float> h((size_t)m->n_params);
    float *q = h.data();
    // order of draws as src/model.c:301-330
    for (long i = 0; i < V * C; i++) *q++ = polar_randn() * std;
    for (long i = 0; i < (long)m->cfg.block_size * C; i++) *q++ = polar_randn() * std;
    for (long l = 0; l < L; l++) {
        for (long i = 0; i < C; i++) *q++ = 1.0f;
        for (long i = 0; i < C; i++) *q++ = 0.0f;
        for (long i = 0; i < 3 * C * C; i++) *q++ = polar_randn() * std;
        for (long i = 0; i < 3 * C; i++) *q++ = 0.0f;
        for (long i = 0; i < C * C; i++) *q++ = polar_randn() * rstd;
        for (long i = 0; i < C; i++) *q++ = 0.0f;
        for (long i = 0; i < C; i++) *q++ = 1.0f;
        for (long i = 0; i < C; i++) *q++ = 0.0f;
        for (long i = 0; i < 4 * C * C; i++) *q++ = polar_randn() * std;
        for (long i = 0; i < 4 * C; i++) *q++ = 0.0f;
        for (long i = 0; i < 4 * C * C; i++) *q++ = polar_randn() * rstd;
        for (long i = 0; i < C; i++) *q++ = 0.0f;
    }
    for (long i = 0; i < C; i++) *q++ = 1.0f;
    for (long i = 0; i < C; i++) *q++ = 0.0f;
    if (cudaMemcpy(m->param_buf, h.data(), h.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)
        set_last_error(ERR_CUDA, "gpt_init_weights upload failed");
}

extern "C" int gpt_load(GPT *m, const char *path) {
    FILE *f = fopen(path, "rb");
    if (!f) {
        perror(path);
        return -1;
    }
    GPTHeader hdr;
    if (fread(&hdr, sizeof(hdr), 1, f) != 1) {
        fprintf(stderr, "gpt_load: short header\n");
        fclose(f);
        return -1;
    }
    if (hdr.magic != CNGPT_MAGIC) {
        fprintf(stderr, "gpt_load: bad magic 0x%X\n", hdr.magic);
        fclose(f);
        return -1;
    }
    if (m->param_buf == NULL) {
        GPTConfig cfg = {hdr.n_layer, hdr.n_head, hdr.n_embd, hdr.vocab_size, hdr.block_size, 0.0f};
        if (gpt_init(m, cfg) != 0) {
            fclose(f);
            return -1;
        }
    }
    std::vector<float> h((size_t)m->n_params);
    if (fread(h.data(), sizeof(float), h.size(), f) != h.size()) {
        fprintf(stderr, "gpt_load: short param data\n");
        fclose(f);
        return -1;
    }
    fclose(f);
    if (cudaMemcpy(m->param_buf, h.data(), h.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        set_last_error(ERR_CUDA, "gpt_load upload failed");
        return -1;
    }
    return 0;
}

extern "C" int gpt_save(GPT *m, const char *path) {
    std::vector<float> h((size_t)m->n_params);
    cudaStreamSynchronize(g_stream);
    if (cudaMemcpy(h.data(), m->param_buf, h.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        set_last_error(ERR_CUDA, "gpt_save download failed");
        return -1;
    }
    FILE *f = fopen(path, "wb");
    if (!f) {
        perror(path);
        return -1;
    }
    GPTHeader hdr = {CNGPT_MAGIC, CNGPT_VERSION, m->cfg.n_layer, m->cfg.n_head, m->cfg.n_embd,
                     m->cfg.vocab_size, m->cfg.block_size};
    fwrite(&hdr, sizeof(hdr), 1, f);
    fwrite(h.data(), sizeof(float), h.size(), f);
    fclose(f);
    return 0;
}

// ------------------------------------------------------- training checkpoints
// gpt_save's file (header + parameters, readable by any gpt_load) followed by
// an optimizer trailer the reference never writes: magic, AdamW step count,
// then the first and second moments (n_params floats each).
namespace {
constexpr uint32_t kOptMagic = 0x4F50544Du;  // "MTPO"

int write_all(FILE *f, const void *p, size_t bytes) { return fwrite(p, 1, bytes, f) == bytes ? 0 : -1; }
int read_all(FILE *f, void *p, size_t bytes) { return fread(p, 1, bytes, f) == bytes ? 0 : -1; }
}  // namespace

extern "C" int cngpt_cuda_save_checkpoint(GPT *m, const char *path) {
    if (!model_ctx(m)) return ERR_STATE;
    const size_t n = (size_t)m->n_params;
    std::vector<float> h(n);
    cudaStreamSynchronize(g_stream);
    FILE *f = fopen(path, "wb");
    if (!f) {
        set_last_error(ERR_ARG, "save_checkpoint: cannot open %s", path);
        return ERR_ARG;
    }
    GPTHeader hdr = {CNGPT_MAGIC, CNGPT_VERSION, m->cfg.n_layer, m->cfg.n_head, m->cfg.n_embd,
                     m->cfg.vocab_size, m->cfg.block_size};
    int st = write_all(f, &hdr, sizeof(hdr));
    const float *bufs[3] = {m->param_buf, m->m_buf, m->v_buf};
    for (int i = 0; i < 3 && st == 0; ++i) {
        if (i == 1) {
            const uint32_t magic = kOptMagic;
            const int32_t step = m->step;
            st = write_all(f, &magic, 4) | write_all(f, &step, 4);
        }
        if (cudaMemcpy(h.data(), bufs[i], n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
            fclose(f);
            set_last_error(ERR_CUDA, "save_checkpoint: download failed");
            return ERR_CUDA;
        }
        if (st == 0) st = write_all(f, h.data(), n * 4);
    }
    if (fclose(f) != 0 || st != 0) {
        set_last_error(ERR_ARG, "save_checkpoint: writing %s failed", path);
        return ERR_ARG;
    }
    return OK;
}

// The whole file is read and checked on the host before anything reaches the
// device, so a truncated or foreign file leaves the model as it was.
extern "C" int cngpt_cuda_load_checkpoint(GPT *m, const char *path) {
    FILE *f = fopen(path, "rb");
    if (!f) {
        set_last_error(ERR_ARG, "load_checkpoint: cannot open %s", path);
        return ERR_ARG;
    }
    GPTHeader hdr;
    if (read_all(f, &hdr, sizeof(hdr)) != 0 || hdr.magic != CNGPT_MAGIC) {
        fclose(f);
        set_last_error(ERR_ARG, "load_checkpoint: %s is not a cngpt model file", path);
        return ERR_ARG;
    }
    if (m->param_buf && (hdr.n_layer != m->cfg.n_layer || hdr.n_head != m->cfg.n_head ||
                         hdr.n_embd != m->cfg.n_embd || hdr.vocab_size != m->cfg.vocab_size ||
                         hdr.block_size != m->cfg.block_size)) {
        fclose(f);
        set_last_error(ERR_ARG, "load_checkpoint: %s holds a different configuration", path);
        return ERR_ARG;
    }
    GPTConfig cfg = {hdr.n_layer, hdr.n_head, hdr.n_embd, hdr.vocab_size, hdr.block_size, 0.0f};
    if (hdr.n_layer < 0 || hdr.n_head <= 0 || hdr.n_embd <= 0 || hdr.vocab_size <= 0 || hdr.block_size <= 0) {
        fclose(f);
        set_last_error(ERR_ARG, "load_checkpoint: %s has an invalid configuration", path);
        return ERR_ARG;
    }
    const size_t n = (size_t)gpt_num_params(&cfg);
    std::vector<float> params(n), mom1, mom2;
    uint32_t magic = 0;
    int32_t step = 0;
    bool ok = read_all(f, params.data(), n * 4) == 0;
    bool has_opt = false;
    if (ok && read_all(f, &magic, 4) == 0) {
        // a trailer that starts must be complete
        has_opt = magic == kOptMagic;
        if (has_opt) {
            mom1.resize(n);
            mom2.resize(n);
            ok = read_all(f, &step, 4) == 0 && read_all(f, mom1.data(), n * 4) == 0 &&
                 read_all(f, mom2.data(), n * 4) == 0;
        }
    }
    fclose(f);
    if (!ok) {
        set_last_error(ERR_ARG, "load_checkpoint: %s is truncated", path);
        return ERR_ARG;
    }
    if (!m->param_buf && gpt_init(m, cfg) != 0) return ERR_ALLOC;
    CG_CUDA(cudaStreamSynchronize(g_stream));
    CG_CUDA(cudaMemcpy(m->param_buf, params.data(), n * 4, cudaMemcpyHostToDevice));
    if (has_opt) {
        CG_CUDA(cudaMemcpy(m->m_buf, mom1.data(), n * 4, cudaMemcpyHostToDevice));
        CG_CUDA(cudaMemcpy(m->v_buf, mom2.data(), n * 4, cudaMemcpyHostToDevice));
        m->step = step;
    } else {  // a plain gpt_save file: fresh optimizer state
        CG_CUDA(cudaMemset(m->m_buf, 0, n * 4));
        CG_CUDA(cudaMemset(m->v_buf, 0, n * 4));
        m->step = 0;
    }
    return OK;
}

extern "C" int cngpt_cuda_dp_free(GPT *m);

extern "C" void gpt_free(GPT *m) {
    ModelCtx *c = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        auto it = g_models.find(m);
        if (it != g_models.end()) c = it->second;
    }
    cudaStreamSynchronize(g_stream);
    if (c && (c->nccl_comm || c->comm_stream)) cngpt_cuda_dp_free(m);
    tp_release(m);
    dev_free(m->param_buf);
    dev_free(m->grad_buf);
    dev_free(m->m_buf);
    dev_free(m->v_buf);
    dev_free(m->decay_buf);
    dev_free(m->act_buf);
    dev_free(m->mask_buf);
    free_weight_ptrs(&m->params);
    free_weight_ptrs(&m->grads);
    if (m->acts.ln1_out) free_act_ptrs(&m->acts);
    if (c) {
        float *bufs[] = {c->dlogits, c->d_x, c->d_ln, c->d_mlp, c->d_ao, c->d_qkv, c->scratch,
                         c->dev_scalars};
        for (auto b : bufs) dev_free(b);
        dev_free(c->norm_scratch);
        dev_free(c->tok);
        dev_free(c->tgt);
        if (c->host_loss) cudaFreeHost(c->host_loss);
        std::lock_guard<std::mutex> lk(g_mu);
        g_models.erase(m);
        delete c;
    }
    memset(m, 0, sizeof(*m));
}

extern "C" int gpt_resize_acts(GPT *m, int B, int T) {
    ModelCtx *c = model_ctx(m);
    if (!c) return -1;
    return resize_acts(m, c, B, T) == OK ? 0 : -1;
}

extern "C" float gpt_forward(GPT *m, const int *tokens, const int *targets, int B, int T) {
    ModelCtx *c = model_ctx(m);
    if (!c) return 0.0f;
    if (forward(m, c, tokens, targets, B, T, true, g_stream) != OK) {
        fprintf(stderr, "gpt_forward: %s\n", last_message());
        return 0.0f;
    }
    if (!targets) {
        sync_if_managed(c);
        return 0.0f;
    }
    if (cudaMemcpyAsync(c->host_loss, &c->dev_scalars[0], sizeof(float), cudaMemcpyDeviceToHost,
                        g_stream) != cudaSuccess ||
        cudaStreamSynchronize(g_stream) != cudaSuccess) {
        set_last_error(ERR_CUDA, "gpt_forward: loss readback failed");
        return 0.0f;
    }
    return *c->host_loss;
}

extern "C" void gpt_backward(GPT *m, const int *tokens, const int *targets, int B, int T) {
    ModelCtx *c = model_ctx(m);
    if (!c) return;
    if (backward(m, c, tokens, targets, B, T, g_stream) != OK) {
        fprintf(stderr, "gpt_backward: %s\n", last_message());
        return;
    }
    sync_if_managed(c);
}

extern "C" void gpt_zero_grad(GPT *m) {
    ModelCtx *c = model_ctx(m);
    if (!c) return;
    cudaMemsetAsync(m->grad_buf, 0, (size_t)m->n_params * sizeof(float), g_stream);
    sync_if_managed(c);
}

extern "C" void gpt_adamw(GPT *m, float lr, float beta1, float beta2, float eps, float wd,
                          float grad_clip) {
    ModelCtx *c = model_ctx(m);
    if (!c) return;
    if (adamw_step(m, c, lr, beta1, beta2, eps, wd, grad_clip, g_stream) != OK) {
        fprintf(stderr, "gpt_adamw: %s\n", last_message());
        return;
    }
    sync_if_managed(c);
}

// ============================================================ cngpt_cuda.h (model)

extern "C" int cngpt_cuda_train_step(GPT *m, const int *tokens, const int *targets, int B, int T,
                                     float lr, float beta1, float beta2, float eps, float wd,
                                     float grad_clip, float *loss_out) {
    ModelCtx *c = model_ctx(m);
    if (!c) return ERR_STATE;
    if (!targets) {
        set_last_error(ERR_ARG, "train_step: targets required");
        return ERR_ARG;
    }
    cudaStream_t s = g_stream;
    const bool dp = c->world > 1 && c->nccl_comm;
    CG_CUDA(cudaMemsetAsync(m->grad_buf, 0, (size_t)m->n_params * sizeof(float), s));
    CG_TRY(forward(m, c, tokens, targets, B, T, true, s, true));
    if (dp) {
        // the reported loss is the mean over the global batch (every rank has B*T rows)
        CG_CUDA(cudaEventRecord(c->ev_ready, s));
        CG_CUDA(cudaStreamWaitEvent(c->comm_stream, c->ev_ready, 0));
        CG_TRY(dp_allreduce(c, &c->dev_scalars[0], 1, c->comm_stream));
    }
    CG_TRY(backward(m, c, tokens, targets, B, T, s, dp));
    CG_TRY(adamw_step(m, c, lr, beta1, beta2, eps, wd, grad_clip, s));
    if (loss_out) {
        CG_CUDA(cudaMemcpyAsync(c->host_loss, &c->dev_scalars[0], sizeof(float), cudaMemcpyDeviceToHost, s));
        CG_CUDA(cudaStreamSynchronize(s));
        *loss_out = *c->host_loss;
    }
    return OK;
}

extern "C" int cngpt_cuda_last_loss(GPT *m, float *loss_out) {
    ModelCtx *c = model_ctx(m);
    if (!c) return ERR_STATE;
    CG_CUDA(cudaMemcpyAsync(c->host_loss, &c->dev_scalars[0], sizeof(float), cudaMemcpyDeviceToHost,
                            g_stream));
    CG_CUDA(cudaStreamSynchronize(g_stream));
    *loss_out = *c->host_loss;
    return OK;
}

extern "C" int cngpt_cuda_params_to_host(GPT *m, float *dst) {
    CG_CUDA(cudaStreamSynchronize(g_stream));
    CG_CUDA(cudaMemcpy(dst, m->param_buf, (size_t)m->n_params * 4, cudaMemcpyDefault));
    return OK;
}

extern "C" int cngpt_cuda_params_from_host(GPT *m, const float *src) {
    CG_CUDA(cudaStreamSynchronize(g_stream));
    CG_CUDA(cudaMemcpy(m->param_buf, src, (size_t)m->n_params * 4, cudaMemcpyDefault));
    return OK;
}

extern "C" int cngpt_cuda_grads_to_host(GPT *m, float *dst) {
    CG_CUDA(cudaStreamSynchronize(g_stream));
    CG_CUDA(cudaMemcpy(dst, m->grad_buf, (size_t)m->n_params * 4, cudaMemcpyDefault));
    return OK;
}
