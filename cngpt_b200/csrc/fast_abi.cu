// fast_abi.cu - cngpt/fast.h on the device, plus greedy decode with a KV cache.
//
// gpt_forward_fast follows src/fast.c:227-333: scratch sized once per (B, T)
// and reused, attention straight from the packed qkv rows, the last layer
// continued past attention for the final position of each sequence only,
// residual adds folded into the projection epilogues (x += ...), GELU fused
// into the fc epilogue, and the LM head for the final positions only.
//
// cngpt_cuda_generate adds what the reference does not have (it recomputes
// the whole prefix for every token, src/model.c:1001-1015): the prefill
// stores K and V of every layer, then each step runs one row per sequence
// through the stack with single-query attention over the cache, and takes the
// argmax of the last-position logits (lowest index on ties).
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "abi_common.h"
#include "decode_mk.h"
#include "kernels.h"
#include "model_ctx.h"

extern "C" {
#include "cngpt_cuda.h"
}

namespace cg {
void fast_forget(const FastCtx *f);

namespace {

void drop_graph(FastDev *d) {
    if (d->step_graph) cudaGraphExecDestroy(d->step_graph);
    d->step_graph = nullptr;
    d->graph_params = nullptr;
}

int fast_resize(FastCtx *f, FastDev *d, const GPT *m, int B, int T, bool managed) {
    if (f->x && f->B == B && f->T == T) return OK;
    cudaStreamSynchronize(g_stream);
    if (d->cap_stream) cudaStreamSynchronize(d->cap_stream);
    drop_graph(d);  // the captured step holds the scratch addresses
    float **bufs[] = {&f->x, &f->ln, &f->qkv, &f->aout, &f->hid, &f->mean, &f->rstd, &f->logits,
                      &d->xl, &d->al};
    for (auto b : bufs) {
        dev_free(*b);
        *b = nullptr;
    }
    f->scores = nullptr;  // the fused attention never forms T x T scores
    const size_t C = m->cfg.n_embd, V = m->cfg.vocab_size, N = (size_t)B * T;
    CG_TRY(dev_alloc((void **)&f->x, N * C * 4, managed));
    CG_TRY(dev_alloc((void **)&f->ln, N * C * 4, managed));
    CG_TRY(dev_alloc((void **)&f->qkv, N * 3 * C * 4, managed));
    CG_TRY(dev_alloc((void **)&f->aout, N * C * 4, managed));
    CG_TRY(dev_alloc((void **)&f->hid, N * 4 * C * 4, managed));
    CG_TRY(dev_alloc((void **)&f->mean, N * 4, managed));
    CG_TRY(dev_alloc((void **)&f->rstd, N * 4, managed));
    CG_TRY(dev_alloc((void **)&f->logits, (size_t)B * V * 4, managed));
    CG_TRY(dev_alloc((void **)&d->xl, (size_t)B * C * 4, false));
    CG_TRY(dev_alloc((void **)&d->al, (size_t)B * C * 4, false));
    f->B = B;
    f->T = T;
    return OK;
}

GemmEpi epi_store(float *D, long ldd, const float *bias) {
    GemmEpi e;
    e.mode = EPI_STORE;
    e.D = D;
    e.ldd = ldd;
    e.bias = bias;
    return e;
}

// x += A W^T + b  (src/fast.c:314-315, 322-323 with accumulate = 1)
GemmEpi epi_resid_inplace(float *x, long ld, const float *bias) {
    GemmEpi e;
    e.mode = EPI_RESID;
    e.bias = bias;
    e.D2 = x;
    e.ldd2 = ld;
    e.R = x;
    e.ldr = ld;
    return e;
}

GemmEpi epi_gelu_only(float *out, long ld, const float *bias) {
    GemmEpi e;
    e.mode = EPI_GELU;
    e.bias = bias;
    e.D2 = out;
    e.ldd2 = ld;
    return e;
}

// One transformer block for `rows` rows of x (post-attention part).
int block_tail(const GPT *m, int l, FastCtx *f, float *x, const float *aout, int rows, cudaStream_t s) {
    const int C = m->cfg.n_embd;
    const GPTWeights *w = &m->params;
    CG_TRY(gemm(aout, C, false, w->c_proj_w[l], C, false, rows, C, C,
                epi_resid_inplace(x, C, w->c_proj_b[l]), s));
    CG_TRY(layernorm_fwd(x, C, w->ln2_w[l], w->ln2_b[l], f->ln, C, f->mean, f->rstd, rows, C, s));
    CG_TRY(gemm(f->ln, C, false, w->mlp_fc_w[l], C, false, rows, 4 * C, C,
                epi_gelu_only(f->hid, 4 * C, w->mlp_fc_b[l]), s));
    CG_TRY(gemm(f->hid, 4 * C, false, w->mlp_proj_w[l], 4 * C, false, rows, C, 4 * C,
                epi_resid_inplace(x, C, w->mlp_proj_b[l]), s));
    return OK;
}

// Full-prefix forward; if kv is given, K/V of every layer are stored at
// positions [0, T). Leaves the final-position logits in f->logits.
int fast_forward(const GPT *m, FastCtx *f, FastDev *d, const int *tok, int B, int T, bool store_kv,
                 cudaStream_t s) {
    const int C = m->cfg.n_embd, V = m->cfg.vocab_size, L = m->cfg.n_layer, H = m->cfg.n_head;
    const int BT = B * T;
    const GPTWeights *w = &m->params;
    CG_TRY(embed_fwd(tok, w->wte, w->wpe, f->x, BT, T, C, 0, s));
    for (int l = 0; l < L; l++) {
        const bool last = (l == L - 1);
        CG_TRY(layernorm_fwd(f->x, C, w->ln1_w[l], w->ln1_b[l], f->ln, C, f->mean, f->rstd, BT, C, s));
        CG_TRY(gemm(f->ln, C, false, w->c_attn_w[l], C, false, BT, 3 * C, C,
                    epi_store(f->qkv, 3 * C, w->c_attn_b[l]), s));
        if (store_kv) {
            const size_t per = (size_t)d->kv_B * d->kv_T * C;
            CG_TRY(kv_append(f->qkv, d->kc + l * per, d->vc + l * per, B, T, d->kv_T, 0, C, s));
        }
        if (!last) {
            CG_TRY(attention_fwd(f->qkv, f->aout, nullptr, B, T, C, H, s));
            CG_TRY(block_tail(m, l, f, f->x, f->aout, BT, s));
        } else {
            // only the final query row of each sequence (src/fast.c:287-311)
            CG_TRY(attention_fwd_rows(f->qkv, f->aout, B, T, C, H, T - 1, s));
            CG_TRY(gather_last(f->aout, d->al, B, T, C, s));
            CG_TRY(gather_last(f->x, d->xl, B, T, C, s));
            CG_TRY(block_tail(m, l, f, d->xl, d->al, B, s));
        }
    }
    const float *xf = L > 0 ? d->xl : f->x;
    if (L == 0) {
        CG_TRY(gather_last(f->x, d->xl, B, T, C, s));
        xf = d->xl;
    }
    CG_TRY(layernorm_fwd(xf, C, w->ln_f_w, w->ln_f_b, f->ln, C, f->mean, f->rstd, B, C, s));
    CG_TRY(gemm(f->ln, C, false, w->wte, C, false, B, V, C, epi_store(f->logits, V, nullptr), s));
    return OK;
}

// One decode step for B sequences: the incoming tokens d->next[B] sit at
// position ctr[0]; K/V are appended there, the greedy token of the step is
// written to d->next and to d->gen[ctr[1]], then both counters advance. All
// positions are read on the device, so one captured graph replays every step.
int decode_step(const GPT *m, FastCtx *f, FastDev *d, int B, cudaStream_t s) {
    const int C = m->cfg.n_embd, V = m->cfg.vocab_size, L = m->cfg.n_layer, H = m->cfg.n_head;
    const GPTWeights *w = &m->params;
    if (d->mk_bar && mk_decode_ok(B, C, H, d->kv_T)) {
        // the whole step as one cooperative launch (decode_mk.cu)
        MkArgs a;
        a.params = m->param_buf;
        a.wte = w->wte;
        a.wpe = w->wpe;
        a.L = L;
        a.C = C;
        a.H = H;
        a.V = V;
        a.block = m->cfg.block_size;
        a.B = B;
        a.Tmax = d->kv_T;
        a.scale = 1.0f / sqrtf((float)(C / H));
        a.x = d->xl;
        a.qkv = f->qkv;
        a.att = d->al;
        a.hid = f->hid;
        a.logits = f->logits;
        a.ldlog = V;
        a.kc = d->kc;
        a.vc = d->vc;
        a.part = d->dec_part;
        a.tickets = (int *)(d->dec_part + mk_part_floats(B, H, d->kv_T));
        a.S = (int)((d->kv_T + 63) / 64);
        a.next = d->next;
        a.gen = d->gen;
        a.ctr = d->ctr;
        a.am_key = d->am_key;
        a.bar = d->mk_bar;
        a.abort = (int *)(d->mk_bar + 1);
        a.fast_act = 0;  // accurate tanh, as the GEMV decode path
        a.trace = d->mk_trace;
        return decode_step_mk(a, s);
    }
    float *x = d->xl;
    CG_TRY(embed_fwd_at(d->next, w->wte, w->wpe, x, B, C, d->ctr, s));
    const size_t per = (size_t)d->kv_B * d->kv_T * C;
    // LayerNorm statistics of the residual stream come from the last block of
    // the GEMV that produced it (stats[0]: after c_proj, stats[1]: after
    // mlp_proj); layer 0's come from the embedding inside the first GEMV
    const bool st = B <= 8;
    float *st_attn = d->ln_stats, *st_mlp = d->ln_stats + 16;
    auto resid = [&](float *xx, const float *bias, float *stats, int *ticket) {
        GemmEpi e = epi_resid_inplace(xx, C, bias);
        if (st) {
            e.ln_stats_out = stats;
            e.ln_ticket = ticket;
        }
        return e;
    };
    for (int l = 0; l < L; l++) {
        // LN1 fused into the qkv GEMV, whose epilogue also appends K and V
        GemmEpi eq = epi_store(f->qkv, 3 * C, w->c_attn_b[l]);
        eq.kc = d->kc + l * per;
        eq.vc = d->vc + l * per;
        eq.kv_ld = (long)d->kv_T * C;
        eq.kv_pos = d->ctr;
        eq.kv_C = C;
        CG_TRY(gemm_ln(x, C, w->ln1_w[l], w->ln1_b[l], (st && l > 0) ? st_mlp : nullptr, f->ln,
                       w->c_attn_w[l], C, B, 3 * C, C, eq, s));
        CG_TRY(attention_decode_at(f->qkv, 3L * C, d->kc + l * per, d->vc + l * per, d->kv_T, d->ctr,
                                   d->al, B, C, H, d->dec_part, s));
        CG_TRY(gemm(d->al, C, false, w->c_proj_w[l], C, false, B, C, C,
                    resid(x, w->c_proj_b[l], st_attn, d->ln_ticket), s));
        CG_TRY(gemm_ln(x, C, w->ln2_w[l], w->ln2_b[l], st ? st_attn : nullptr, f->ln, w->mlp_fc_w[l], C, B,
                       4 * C, C, epi_gelu_only(f->hid, 4 * C, w->mlp_fc_b[l]), s));
        CG_TRY(gemm(f->hid, 4 * C, false, w->mlp_proj_w[l], 4 * C, false, B, C, 4 * C,
                    resid(x, w->mlp_proj_b[l], st_mlp, d->ln_ticket + 1), s));
    }
    // LM head with the greedy argmax folded into its epilogue
    GemmEpi eh = epi_store(f->logits, V, nullptr);
    eh.argmax_key = d->am_key;
    CG_TRY(gemm_ln(x, C, w->ln_f_w, w->ln_f_b, (st && L > 0) ? st_mlp : nullptr, f->ln, w->wte, C, B, V, C, eh, s));
    // tokens of this step -> next input and the log; counters advance
    return greedy_finalize(d->am_key, B, d->next, d->gen, d->ctr + 1, nullptr, d->ctr, s);
}

// Capture one decode step on the FastDev's own stream (reused while the model,
// batch, cache capacity, precision and output buffer are unchanged).
int capture_step(const GPT *m, FastCtx *f, FastDev *d, int B) {
    if (d->step_graph && d->graph_params == m->param_buf && d->graph_B == B && d->graph_T == d->kv_T &&
        d->graph_prec == precision() && d->graph_logits == f->logits)
        return OK;
    drop_graph(d);
    cudaGraph_t g = nullptr;
    CG_CUDA(cudaStreamBeginCapture(d->cap_stream, cudaStreamCaptureModeThreadLocal));
    const int st = decode_step(m, f, d, B, d->cap_stream);
    const cudaError_t e = cudaStreamEndCapture(d->cap_stream, &g);
    if (st != OK) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    if (e != cudaSuccess) {
        set_last_error(ERR_CUDA, "decode graph capture: %s", cudaGetErrorString(e));
        return ERR_CUDA;
    }
    const cudaError_t ei = cudaGraphInstantiate(&d->step_graph, g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) {
        d->step_graph = nullptr;
        set_last_error(ERR_CUDA, "decode graph instantiate: %s", cudaGetErrorString(ei));
        return ERR_CUDA;
    }
    d->graph_params = m->param_buf;
    d->graph_B = B;
    d->graph_T = d->kv_T;
    d->graph_prec = precision();
    d->graph_logits = f->logits;
    return OK;
}

}  // namespace
}  // namespace cg

using namespace cg;

extern "C" void fast_init(FastCtx *f) {
    fast_forget(f);
    memset(f, 0, sizeof(*f));
}

extern "C" void fast_free(FastCtx *f) {
    cudaStreamSynchronize(g_stream);
    float *bufs[] = {f->x, f->ln, f->qkv, f->aout, f->hid, f->mean, f->rstd, f->logits};
    for (auto b : bufs) dev_free(b);
    FastDev *d = fast_dev(f, false);
    if (d) {
        dev_free(d->xl);
        dev_free(d->al);
        dev_free(d->tok);
        dev_free(d->kc);
        dev_free(d->vc);
        dev_free(d->dec_part);
        dev_free(d->next);
        dev_free(d->gen);
        dev_free(d->ctr);
        dev_free(d->ln_stats);
        dev_free(d->ln_ticket);
        dev_free(d->am_key);
        dev_free(d->mk_bar);
        dev_free(d->mk_trace);
        drop_graph(d);
        if (d->ev_a) cudaEventDestroy(d->ev_a);
        if (d->ev_b) cudaEventDestroy(d->ev_b);
        if (d->cap_stream) cudaStreamDestroy(d->cap_stream);
        fast_forget(f);
    }
    memset(f, 0, sizeof(*f));
}

extern "C" void fast_set_threads(int n) { (void)n; }

extern "C" const float *gpt_forward_fast(GPT *m, FastCtx *f, const int *tokens, int B, int T) {
    ModelCtx *c = model_ctx(m);
    if (!c) return nullptr;
    if (B <= 0 || T <= 0 || T > m->cfg.block_size) {
        set_last_error(ERR_ARG, "gpt_forward_fast: bad shape B=%d T=%d", B, T);
        return nullptr;
    }
    FastDev *d = fast_dev(f, true);
    if (fast_resize(f, d, m, B, T, c->managed) != OK) return nullptr;
    const int *tok = nullptr;
    if (stage_tokens(tokens, (size_t)B * T, &d->tok, &d->tok_cap, &tok, g_stream) != OK) return nullptr;
    if (fast_forward(m, f, d, tok, B, T, false, g_stream) != OK) {
        fprintf(stderr, "gpt_forward_fast: %s\n", last_message());
        return nullptr;
    }
    if (c->managed) cudaStreamSynchronize(g_stream);
    return f->logits;
}

namespace cg {
namespace {
// Phase stamps of the last single-launch decode step, summarised on stderr:
// the embedding, each layer's five phases (mean over layers) and the LM head.
void report_trace(const unsigned long long *dev, int L) {
    std::vector<unsigned long long> t(5 * (size_t)L + 3);
    if (cudaMemcpy(t.data(), dev, t.size() * sizeof(t[0]), cudaMemcpyDeviceToHost) != cudaSuccess) return;
    double ph[5] = {0, 0, 0, 0, 0};
    for (int l = 0; l < L; ++l)
        for (int k = 0; k < 5; ++k) ph[k] += (double)(t[1 + 5 * l + k + 1] - t[1 + 5 * l + k]) / L;
    fprintf(stderr,
            "decode step trace: embed %.2f us; per layer ln1+qkv %.2f, attention %.2f, c_proj %.2f, ln2+fc %.2f, "
            "proj %.2f us; ln_f+lm_head %.2f us; total %.1f us\n",
            (t[1] - t[0]) * 1e-3, ph[0] * 1e-3, ph[1] * 1e-3, ph[2] * 1e-3, ph[3] * 1e-3, ph[4] * 1e-3,
            (t[2 + 5 * L] - t[1 + 5 * L]) * 1e-3, (t[2 + 5 * L] - t[0]) * 1e-3);
}

// Decode state of a FastCtx for B sequences, a prompt of T tokens and n_new
// generated tokens: the KV cache (capacity T + n_new positions), the decode
// counters, the per-step token log and the statistics / argmax scratch.
int kv_prepare(const GPT *m, FastCtx *f, FastDev *d, int B, int T, int n_new, bool managed, cudaStream_t s) {
    CG_TRY(fast_resize(f, d, m, B, T, managed));
    const int Tmax = T + n_new;
    const size_t C = m->cfg.n_embd, L = m->cfg.n_layer;
    if (!d->cap_stream) {
        CG_CUDA(cudaStreamCreateWithFlags(&d->cap_stream, cudaStreamNonBlocking));
        CG_CUDA(cudaEventCreateWithFlags(&d->ev_a, cudaEventDisableTiming));
        CG_CUDA(cudaEventCreateWithFlags(&d->ev_b, cudaEventDisableTiming));
        CG_TRY(dev_alloc((void **)&d->ctr, 2 * sizeof(int), false));
        CG_TRY(dev_alloc((void **)&d->ln_stats, 32 * sizeof(float), false));
        CG_TRY(dev_alloc((void **)&d->ln_ticket, 4 * sizeof(int), false));
        CG_CUDA(cudaMemsetAsync(d->ln_ticket, 0, 4 * sizeof(int), s));
        CG_TRY(dev_alloc((void **)&d->am_key, 8 * sizeof(unsigned long long), false));
        CG_CUDA(cudaMemsetAsync(d->am_key, 0, 8 * sizeof(unsigned long long), s));
        CG_TRY(dev_alloc((void **)&d->mk_bar, 2 * sizeof(unsigned long long), false));
        CG_CUDA(cudaMemsetAsync(d->mk_bar, 0, 2 * sizeof(unsigned long long), s));
        if (getenv("CNGPT_CUDA_DECODE_TRACE"))
            CG_TRY(dev_alloc((void **)&d->mk_trace, (5 * (size_t)L + 3) * sizeof(unsigned long long), false));
    }
    if (d->kv_B != B || d->kv_T < Tmax) {
        CG_CUDA(cudaStreamSynchronize(s));
        drop_graph(d);
        dev_free(d->kc);
        dev_free(d->vc);
        dev_free(d->next);
        dev_free(d->dec_part);
        d->kc = d->vc = d->dec_part = nullptr;
        d->next = nullptr;
        CG_TRY(dev_alloc((void **)&d->kc, L * B * Tmax * C * 4, false));
        CG_TRY(dev_alloc((void **)&d->vc, L * B * Tmax * C * 4, false));
        CG_TRY(dev_alloc((void **)&d->dec_part,
                         attention_decode_scratch_floats(B, m->cfg.n_head, Tmax) * 4, false));
        CG_CUDA(cudaMemsetAsync(d->dec_part, 0, attention_decode_scratch_floats(B, m->cfg.n_head, Tmax) * 4, s));
        CG_TRY(dev_alloc((void **)&d->next, (size_t)B * 4, false));
        d->kv_B = B;
        d->kv_T = Tmax;
    }
    if ((size_t)B * n_new > d->gen_cap) {
        CG_CUDA(cudaStreamSynchronize(s));
        drop_graph(d);
        dev_free(d->gen);
        d->gen = nullptr;
        CG_TRY(dev_alloc((void **)&d->gen, (size_t)B * n_new * 4, false));
        d->gen_cap = (size_t)B * n_new;
    }
    return OK;
}
}  // namespace
}  // namespace cg

extern "C" int cngpt_cuda_generate(GPT *m, FastCtx *f, const int *prompt, int B, int T, int n_new,
                                   int *out_tokens) {
    ModelCtx *c = model_ctx(m);
    if (!c) return ERR_STATE;
    if (B <= 0 || T <= 0 || n_new <= 0 || T + n_new - 1 > m->cfg.block_size) {
        set_last_error(ERR_ARG, "generate: B=%d T=%d n_new=%d exceeds block_size %d", B, T, n_new,
                       m->cfg.block_size);
        return ERR_ARG;
    }
    cudaStream_t s = g_stream;
    FastDev *d = fast_dev(f, true);
    CG_TRY(kv_prepare(m, f, d, B, T, n_new, c->managed, s));
    const size_t V = m->cfg.vocab_size;
    const int *tok = nullptr;
    CG_TRY(stage_tokens(prompt, (size_t)B * T, &d->tok, &d->tok_cap, &tok, s));
    // counters {T-1, 0}: the prefill's greedy token is logged at step 0, then
    // decode_advance moves to {T, 1} - position T for the first decode input
    const int ctr0[2] = {T - 1, 0};
    CG_CUDA(cudaMemcpyAsync(d->ctr, ctr0, sizeof(ctr0), cudaMemcpyHostToDevice, s));
    CG_TRY(fast_forward(m, f, d, tok, B, T, true, s));
    CG_TRY(argmax_log(f->logits, V, B, (int)V, d->next, d->gen, d->ctr + 1, s));
    CG_TRY(decode_advance(d->ctr, s));
    if (n_new > 1) {
        // the decode steps run on the FastDev's stream, ordered after the prefill
        CG_CUDA(cudaEventRecord(d->ev_a, s));
        CG_CUDA(cudaStreamWaitEvent(d->cap_stream, d->ev_a, 0));
        CG_TRY(decode_step(m, f, d, B, d->cap_stream));  // eager first step (warms the kernels)
        if (n_new > 2) {
            CG_TRY(capture_step(m, f, d, B));
            for (int i = 2; i < n_new; ++i) CG_CUDA(cudaGraphLaunch(d->step_graph, d->cap_stream));
        }
        CG_CUDA(cudaEventRecord(d->ev_b, d->cap_stream));
        CG_CUDA(cudaStreamWaitEvent(s, d->ev_b, 0));
    }
    std::vector<int> h((size_t)B * n_new);
    CG_CUDA(cudaMemcpyAsync(h.data(), d->gen, h.size() * 4, cudaMemcpyDeviceToHost, s));
    CG_CUDA(cudaStreamSynchronize(s));
    CG_TRY(check_device_error());
    for (int b = 0; b < B; ++b)
        for (int i = 0; i < n_new; ++i) out_tokens[(size_t)b * n_new + i] = h[(size_t)i * B + b];
    if (d->mk_trace && n_new > 1) report_trace(d->mk_trace, m->cfg.n_layer);
    return OK;
}

// ---------------------------------------------------------------- gpt_sample
// Temperature / top-k sampling with the host rand() stream, the same steps as
// src/model.c:927-989; logits come from the device fast forward (the final
// position of the cropped context, src/model.c:1001-1011).
namespace {
int sample_top_k(const float *logits, int V, float temp, int top_k) {
    std::vector<float> sc((size_t)V);
    for (int i = 0; i < V; i++) sc[i] = logits[i] / (temp > 0.0f ? temp : 1.0f);
    float mx = sc[0];
    for (int i = 1; i < V; i++)
        if (sc[i] > mx) mx = sc[i];
    float sum = 0.0f;
    for (int i = 0; i < V; i++) {
        sc[i] = expf(sc[i] - mx);
        sum += sc[i];
    }
    for (int i = 0; i < V; i++) sc[i] /= sum;
    if (top_k > 0 && top_k < V) {
        std::vector<float> cp(sc);
        for (int k = 0; k < top_k && k < V; k++)
            for (int i = k + 1; i < V; i++)
                if (cp[i] > cp[k]) std::swap(cp[i], cp[k]);
        const float threshold = cp[top_k - 1];
        float ns = 0.0f;
        for (int i = 0; i < V; i++) {
            if (sc[i] < threshold) sc[i] = 0.0f;
            ns += sc[i];
        }
        if (ns > 0.0f)
            for (int i = 0; i < V; i++) sc[i] /= ns;
    }
    const float r = (float)rand() / ((float)RAND_MAX + 1.0f);
    float cdf = 0.0f;
    int tok = V - 1;
    for (int i = 0; i < V; i++) {
        cdf += sc[i];
        if (r < cdf) {
            tok = i;
            break;
        }
    }
    return tok;
}
}  // namespace

// The reference recomputes the whole (cropped) prefix for every token
// (src/model.c:991-1016). While the context still fits block_size, nothing
// is cropped and every position keeps its embedding, so here the prompt is
// prefilled once into the KV cache and each further step runs one row
// through the cached decode step; only the sampling runs on the host, on the
// step's final-position logits, with the same rand() stream. Once the
// context would exceed block_size the reference crops it and every position
// shifts: those steps recompute the cropped prefix as the reference does.
namespace {
// tokens out[p, p + n) for p = prompt_len; returns the number produced
int sample_cached(GPT *m, FastCtx *f, int *out, int prompt_len, int n, float temp, int top_k) {
    ModelCtx *c = model_ctx(m);
    if (!c) return 0;
    cudaStream_t s = g_stream;
    FastDev *d = fast_dev(f, true);
    const int V = m->cfg.vocab_size;
    std::vector<float> lg((size_t)V);
    const int *tok = nullptr;
    if (kv_prepare(m, f, d, 1, prompt_len, n, c->managed, s) != OK ||
        stage_tokens(out, (size_t)prompt_len, &d->tok, &d->tok_cap, &tok, s) != OK ||
        fast_forward(m, f, d, tok, 1, prompt_len, true, s) != OK ||
        cudaMemcpyAsync(lg.data(), f->logits, (size_t)V * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return 0;
    for (int i = 0; i < n; ++i) {
        const int t = sample_top_k(lg.data(), V, temp, top_k);
        out[prompt_len + i] = t;
        if (i + 1 == n) return n;
        // the sampled token enters at position prompt_len + i; the step's own
        // greedy bookkeeping (token log, next id) is overwritten by the sample
        const int ctr[2] = {prompt_len + i, i + 1};
        if (cudaMemcpyAsync(d->ctr, ctr, sizeof(ctr), cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaMemcpyAsync(d->next, &out[prompt_len + i], sizeof(int), cudaMemcpyHostToDevice, s) != cudaSuccess ||
            decode_step(m, f, d, 1, s) != OK ||
            cudaMemcpyAsync(lg.data(), f->logits, (size_t)V * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess || check_device_error() != OK)
            return i + 1;
    }
    return n;
}
}  // namespace

extern "C" void gpt_sample(GPT *m, const int *prompt_tokens, int prompt_len, int *out_tokens,
                           int max_new_tokens, float temp, int top_k) {
    const int block = m->cfg.block_size, V = m->cfg.vocab_size;
    memcpy(out_tokens, prompt_tokens, (size_t)prompt_len * sizeof(int));
    FastCtx f;
    fast_init(&f);
    int i = 0;
    if (prompt_len > 0 && prompt_len <= block && max_new_tokens > 0) {
        const int n = std::min(max_new_tokens, block - prompt_len + 1);
        i = sample_cached(m, &f, out_tokens, prompt_len, n, temp, top_k);
        if (i < n) {
            fprintf(stderr, "gpt_sample: cached decode failed: %s\n", last_message());
            fast_free(&f);
            return;
        }
    }
    std::vector<float> lg((size_t)V);
    for (; i < max_new_tokens; i++) {
        const int total = prompt_len + i;
        const int start = total > block ? total - block : 0;
        const float *d = gpt_forward_fast(m, &f, out_tokens + start, 1, total - start);
        if (!d || cudaMemcpy(lg.data(), d, (size_t)V * 4, cudaMemcpyDefault) != cudaSuccess) {
            fprintf(stderr, "gpt_sample: forward failed: %s\n", last_message());
            break;
        }
        out_tokens[total] = sample_top_k(lg.data(), V, temp, top_k);
    }
    fast_free(&f);
}
