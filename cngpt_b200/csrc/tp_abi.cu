// tp_abi.cu - tensor-parallel GPT-2 inference, one process per GPU over NCCL.
//
// The reference runs inference on one CPU (src/fast.c:227-333, greedy
// decoding as in src/model.c:991-1016); this splits the same forward across
// ranks the Megatron way, with the rank's slices read straight out of the
// reference's single parameter arena:
//   QKV     column split by heads: rank r owns heads [h0, h0+nh) of q, k, v
//           (packed once into a local [3*nh*hs, C] block, the only copy);
//   c_proj  row split: columns [h0*hs, (h0+nh)*hs) of c_proj_w, read in place
//           with leading dimension C;
//   mlp_fc  column split: rows [f0, f0+nf) of mlp_fc_w, in place;
//   mlp_proj row split: columns [f0, f0+nf) of mlp_proj_w, in place (ld 4C);
//   LM head vocabulary split: rows [v0, v0+nv) of the tied wte, in place.
// Each row-split projection writes its partial sum over the rank's slice into
// the residual stream - rank 0 adds the bias and the old residual in its GEMM
// epilogue, the others store the bare partial - and one sum-allreduce of the
// [rows, C] stream then leaves x + proj(...) + b on every rank (two per
// block). LayerNorms, embeddings and attention of the local heads run
// replicated / locally. The greedy token is the max over ranks of each rank's
// (max logit, lowest index) pair, gathered with one allgather; ties between
// ranks go to the lower vocabulary index, as in the one-GPU argmax.
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "abi_common.h"
#include "common.cuh"
#include "decode_mk.h"
#include "kernels.h"
#include "model_ctx.h"

extern "C" {
#include "cngpt_cuda.h"
}

namespace cg {

CG_DEV_ERROR_ACCESSORS(tp_take_dev_error, tp_set_wait_limit)

namespace {

struct TpPlan {
    int h0 = 0, nh = 0;  // local heads
    int f0 = 0, nf = 0;  // local MLP hidden columns
    int v0 = 0, nv = 0;  // local vocabulary rows
    int vpad = 0;        // vocabulary rows per rank before the ragged last one
};

int make_plan(int H, int C, int V, int world, int rank, TpPlan *p) {
    if (H <= 0 || C <= 0 || V <= 0 || C % H != 0 || world < 1 || rank < 0 || rank >= world ||
        world > H) {
        set_last_error(ERR_ARG, "tp plan: n_head=%d n_embd=%d vocab=%d world=%d rank=%d", H, C, V, world,
                       rank);
        return ERR_ARG;
    }
    // heads: the first H % world ranks take one extra
    const int hq = H / world, hr = H % world;
    p->nh = hq + (rank < hr ? 1 : 0);
    p->h0 = rank * hq + (rank < hr ? rank : hr);
    // MLP hidden width 4C in units of 4 columns (16-byte aligned slices)
    const int units = C, uq = units / world, ur = units % world;
    p->nf = 4 * (uq + (rank < ur ? 1 : 0));
    p->f0 = 4 * (rank * uq + (rank < ur ? rank : ur));
    // vocabulary: equal blocks of ceil(V / world), the last one ragged
    p->vpad = (V + world - 1) / world;
    p->v0 = rank * p->vpad;
    p->nv = std::min(p->vpad, V - p->v0);
    if (p->nv <= 0) {
        set_last_error(ERR_ARG, "tp plan: vocab %d too small for world %d", V, world);
        return ERR_ARG;
    }
    return OK;
}

struct TpState {
    int world = 1, rank = 0;
    void *comm = nullptr;
    TpPlan p;
    int L = 0, C = 0, V = 0, H = 0, hs = 0, Cl = 0;
    long ldlog = 0;
    float *wbuf = nullptr;  // packed QKV weights [L][3Cl][C] then biases [L][3Cl]
    // activations, sized for (B, T)
    int B = 0, T = 0;
    float *x = nullptr, *ln = nullptr, *qkv = nullptr, *aout = nullptr, *hid = nullptr;
    float *mean = nullptr, *rstd = nullptr, *xl = nullptr, *al = nullptr, *logits = nullptr;
    int *pairs = nullptr, *gath = nullptr;  // [2B] local (value bits, index); [world][2B]
    float *lgath = nullptr;                 // [world][B][ldlog] full-logit gather
    int *tok = nullptr;
    size_t tok_cap = 0;
    // KV cache of the local heads [L][B][Tmax][Cl]
    float *kc = nullptr, *vc = nullptr, *dec_part = nullptr;
    int kv_B = 0, kv_T = 0;
    int *next = nullptr, *gen = nullptr, *ctr = nullptr;
    size_t gen_cap = 0;
    cudaStream_t cap_stream = nullptr;
    cudaEvent_t ev_a = nullptr, ev_b = nullptr;
    cudaGraphExec_t graph = nullptr;
    int graph_B = 0, graph_T = 0, graph_prec = -1;
    // peer memory for the decode all-reduce: this rank's receive buffer
    // (tp_buf_bytes), every rank's buffer mapped here (IPC), a device copy of
    // those pointers, the step counter that numbers the exchanges, tickets
    char *pbuf = nullptr;
    char *peer[TP_MAX_WORLD] = {};
    char **d_peers = nullptr;
    int *d_step = nullptr, *d_ticket = nullptr;
    float *d_stats = nullptr;  // [8][2] LayerNorm statistics of x after each exchange
    unsigned long long *am_key = nullptr;  // [8] greedy keys of the LM-head GEMV
    unsigned long long *mk_bar = nullptr;  // grid barrier of the single-launch decode step (world 1)
    // greedy decode split over the ranks (1), replicated on every rank (2), or
    // by batch size (0: replicated at batch 1, split above)
    int decode_mode = 0;
    FastCtx fctx{};  // the replicated decode's one-GPU state

    const float *qkv_w(int l) const { return wbuf + (size_t)l * 3 * Cl * C; }
    const float *qkv_b(int l) const { return wbuf + (size_t)L * 3 * Cl * C + (size_t)l * 3 * Cl; }
};

std::mutex g_tp_mu;
std::map<const GPT *, TpState *> g_tp;

TpState *tp_state(const GPT *m) {
    std::lock_guard<std::mutex> lk(g_tp_mu);
    auto it = g_tp.find(m);
    if (it == g_tp.end()) {
        set_last_error(ERR_STATE, "tensor parallelism not initialised for this model (tp_init)");
        return nullptr;
    }
    return it->second;
}

// greedy token over ranks: gath holds, per rank r, [B] max values (as bits)
// then [B] local indices; global index = local + r * vpad
__global__ void tp_argmax_merge_kernel(const int *__restrict__ gath, int B, int world, int vpad,
                                       int *__restrict__ next, int *__restrict__ log,
                                       const int *__restrict__ step_dev) {
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= B) return;
    float best = -INFINITY;
    int bi = INT_MAX;
    for (int r = 0; r < world; ++r) {
        const int *g = gath + (size_t)r * 2 * B;
        const float v = __int_as_float(g[b]);
        const int i = g[B + b] + r * vpad;
        if (v > best || (v == best && i < bi)) {
            best = v;
            bi = i;
        }
    }
    next[b] = bi;
    if (log) log[(size_t)(*step_dev) * B + b] = bi;
}

// x[m, :] = sum over ranks r, in rank order, of the partial row rank r pushed
// into this rank's receive slot (identical on every rank), then the LayerNorm
// statistics of x for the next LayerNorm-fused GEMV. One block per row. The
// peers' flags are awaited with a bounded spin (the wait limit, 2 s of
// %globaltimer by default); on expiry the block records DEV_ERR_TP_FLAG and
// leaves x unchanged.
__global__ void __launch_bounds__(256)
tp_reduce_kernel(char *__restrict__ buf, int world, int C, const int *__restrict__ step, int nk, int k,
                 float *__restrict__ x, float *__restrict__ stats) {
    pdl_trigger();
    pdl_wait();
    const unsigned long long ep = (unsigned long long)(*step) * nk + k + 1;
    __shared__ int ok;
    __shared__ float red[8][2];
    if (threadIdx.x == 0) ok = 1;
    __syncthreads();
    if ((int)threadIdx.x < world) {
        const unsigned long long *flag = (const unsigned long long *)buf + threadIdx.x;
        const uint64_t t0 = globaltimer_ns();
        const uint64_t limit = *(volatile unsigned long long *)&g_cngpt_wait_limit_ns;
        for (unsigned it = 0;; ++it) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
            if (v >= ep) break;
            if ((it & 255u) == 255u && globaltimer_ns() - t0 > limit) {
                record_error(DEV_ERR_TP_FLAG);
                ok = 0;
                break;
            }
        }
    }
    __syncthreads();
    if (!ok) return;
    const int m = blockIdx.x, slot = (int)(ep & 1), lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float v[8];
    float s1 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int n = threadIdx.x + i * 256;
        v[i] = 0.f;
        if (n < C) {
            float a = 0.f;
            for (int r = 0; r < world; ++r) a += __ldcg(tp_slot(buf, world, C, slot, r) + (long)m * C + n);
            v[i] = a;
            x[(long)m * C + n] = a;
            s1 += a;
        }
    }
    s1 = warp_sum(s1);
    if (lane == 0) red[warp][0] = s1;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < 8; ++w) tot += red[w][0];
    const float mean = tot / (float)C;
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int n = threadIdx.x + i * 256;
        if (n < C) s2 += (v[i] - mean) * (v[i] - mean);
    }
    s2 = warp_sum(s2);
    if (lane == 0) red[warp][1] = s2;
    __syncthreads();
    if (threadIdx.x == 0) {
        float var = 0.f;
        for (int w = 0; w < 8; ++w) var += red[w][1];
        stats[2 * m] = mean;
        stats[2 * m + 1] = 1.0f / sqrtf(var / (float)C + 1e-5f);
    }
}

__global__ void step_advance_kernel(int *step) {
    if (threadIdx.x == 0) *step += 1;
}

void drop_graph(TpState *t) {
    if (t->graph) cudaGraphExecDestroy(t->graph);
    t->graph = nullptr;
}

int allreduce(TpState *t, float *buf, size_t n, cudaStream_t s) {
    if (t->world == 1) return OK;
    return nccl_allreduce_sum(buf, n, t->comm, s);
}

GemmEpi epi_store(float *D, long ldd, const float *bias) {
    GemmEpi e;
    e.mode = EPI_STORE;
    e.D = D;
    e.ldd = ldd;
    e.bias = bias;
    return e;
}

// rank 0: x = x + acc + bias; other ranks: x = acc (their partial sums)
GemmEpi epi_partial(const TpState *t, float *x, long ld, const float *bias) {
    GemmEpi e;
    if (t->rank == 0) {
        e.mode = EPI_RESID;
        e.bias = bias;
        e.D2 = x;
        e.ldd2 = ld;
        e.R = x;
        e.ldr = ld;
    } else {
        e.mode = EPI_STORE;
        e.D = x;
        e.ldd = ld;
    }
    return e;
}

int resize(TpState *t, int B, int T) {
    if (t->x && t->B == B && t->T == T) return OK;
    cudaStreamSynchronize(g_stream);
    if (t->cap_stream) cudaStreamSynchronize(t->cap_stream);
    drop_graph(t);
    float **bufs[] = {&t->x, &t->ln, &t->qkv, &t->aout, &t->hid, &t->mean, &t->rstd, &t->xl, &t->al,
                      &t->logits, &t->lgath};
    for (auto b : bufs) {
        dev_free(*b);
        *b = nullptr;
    }
    dev_free(t->pairs);
    dev_free(t->gath);
    t->pairs = t->gath = nullptr;
    const size_t N = (size_t)B * T, C = t->C, Cl = t->Cl, W = t->world;
    CG_TRY(dev_alloc((void **)&t->x, N * C * 4, false));
    CG_TRY(dev_alloc((void **)&t->ln, N * C * 4, false));
    CG_TRY(dev_alloc((void **)&t->qkv, N * 3 * Cl * 4, false));
    CG_TRY(dev_alloc((void **)&t->aout, N * Cl * 4, false));
    CG_TRY(dev_alloc((void **)&t->hid, N * t->p.nf * 4, false));
    CG_TRY(dev_alloc((void **)&t->mean, N * 4, false));
    CG_TRY(dev_alloc((void **)&t->rstd, N * 4, false));
    CG_TRY(dev_alloc((void **)&t->xl, (size_t)B * C * 4, false));
    CG_TRY(dev_alloc((void **)&t->al, (size_t)B * Cl * 4, false));
    CG_TRY(dev_alloc((void **)&t->logits, (size_t)B * t->ldlog * 4, false));
    CG_TRY(dev_alloc((void **)&t->lgath, W * B * t->ldlog * 4, false));
    CG_TRY(dev_alloc((void **)&t->pairs, (size_t)2 * B * 4, false));
    CG_TRY(dev_alloc((void **)&t->gath, W * 2 * B * 4, false));
    t->B = B;
    t->T = T;
    return OK;
}

// post-attention part of block l for `rows` rows of x (aout: local heads)
int block_tail(const GPT *m, TpState *t, int l, float *x, const float *aout, int rows, cudaStream_t s) {
    const GPTWeights *w = &m->params;
    const int C = t->C, Cl = t->Cl, nf = t->p.nf;
    CG_TRY(gemm(aout, Cl, false, w->c_proj_w[l] + (size_t)t->p.h0 * t->hs, C, false, rows, C, Cl,
                epi_partial(t, x, C, w->c_proj_b[l]), s));
    CG_TRY(allreduce(t, x, (size_t)rows * C, s));
    CG_TRY(layernorm_fwd(x, C, w->ln2_w[l], w->ln2_b[l], t->ln, C, t->mean, t->rstd, rows, C, s));
    GemmEpi g;
    g.mode = EPI_GELU;
    g.bias = w->mlp_fc_b[l] + t->p.f0;
    g.D2 = t->hid;
    g.ldd2 = nf;
    CG_TRY(gemm(t->ln, C, false, w->mlp_fc_w[l] + (size_t)t->p.f0 * C, C, false, rows, nf, C, g, s));
    CG_TRY(gemm(t->hid, nf, false, w->mlp_proj_w[l] + t->p.f0, 4L * C, false, rows, C, nf,
                epi_partial(t, x, C, w->mlp_proj_b[l]), s));
    return allreduce(t, x, (size_t)rows * C, s);
}

// local logits of the final rows xl [B, C] -> t->logits [B, ldlog]
int lm_head(const GPT *m, TpState *t, int B, cudaStream_t s) {
    const GPTWeights *w = &m->params;
    const int C = t->C;
    CG_TRY(layernorm_fwd(t->xl, C, w->ln_f_w, w->ln_f_b, t->ln, C, t->mean, t->rstd, B, C, s));
    return gemm(t->ln, C, false, w->wte + (size_t)t->p.v0 * C, C, false, B, t->p.nv, C,
                epi_store(t->logits, t->ldlog, nullptr), s);
}

// greedy token of the local logits, merged over ranks -> t->next, t->gen[step]
// (pairs_ready: the LM-head GEMV already left the local (max, index) pairs)
int greedy(TpState *t, int B, cudaStream_t s, bool pairs_ready = false) {
    if (!pairs_ready) CG_TRY(argmax_rows(t->logits, t->ldlog, B, t->p.nv, t->pairs + B, (float *)t->pairs, s));
    const int *g = t->pairs;
    if (t->world > 1) {
        CG_TRY(nccl_allgather_words(t->pairs, t->gath, (size_t)2 * B, t->comm, s));
        g = t->gath;
    }
    tp_argmax_merge_kernel<<<(B + 127) / 128, 128, 0, s>>>(g, B, t->world, t->p.vpad, t->next, t->gen,
                                                           t->ctr + 1);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    return OK;
}

// full-prefix forward over (B, T); stores K/V of the local heads when kv
int prefill(const GPT *m, TpState *t, const int *tok, int B, int T, bool kv, cudaStream_t s) {
    const GPTWeights *w = &m->params;
    const int C = t->C, Cl = t->Cl, BT = B * T;
    CG_TRY(embed_fwd(tok, w->wte, w->wpe, t->x, BT, T, C, 0, s));
    const size_t per = (size_t)t->kv_B * t->kv_T * Cl;
    for (int l = 0; l < t->L; ++l) {
        CG_TRY(layernorm_fwd(t->x, C, w->ln1_w[l], w->ln1_b[l], t->ln, C, t->mean, t->rstd, BT, C, s));
        CG_TRY(gemm(t->ln, C, false, t->qkv_w(l), C, false, BT, 3 * Cl, C,
                    epi_store(t->qkv, 3 * Cl, t->qkv_b(l)), s));
        if (kv) CG_TRY(kv_append(t->qkv, t->kc + l * per, t->vc + l * per, B, T, t->kv_T, 0, Cl, s));
        if (l < t->L - 1) {
            CG_TRY(attention_fwd(t->qkv, t->aout, nullptr, B, T, Cl, t->p.nh, s));
            CG_TRY(block_tail(m, t, l, t->x, t->aout, BT, s));
        } else {
            CG_TRY(attention_fwd_rows(t->qkv, t->aout, B, T, Cl, t->p.nh, T - 1, s));
            CG_TRY(gather_last(t->aout, t->al, B, T, Cl, s));
            CG_TRY(gather_last(t->x, t->xl, B, T, C, s));
            CG_TRY(block_tail(m, t, l, t->xl, t->al, B, s));
        }
    }
    if (t->L == 0) CG_TRY(gather_last(t->x, t->xl, B, T, C, s));
    return lm_head(m, t, B, s);
}

// one decode step: tokens t->next at position ctr[0] (see fast_abi.cu); the
// LayerNorms are fused into the GEMVs that consume them and the qkv GEMV's
// epilogue appends K and V to the cache
int decode_step(const GPT *m, TpState *t, int B, cudaStream_t s) {
    const GPTWeights *w = &m->params;
    const int C = t->C, Cl = t->Cl, nf = t->p.nf, L = t->L;
    if (t->world == 1 && t->mk_bar && mk_decode_ok(B, C, t->H, t->kv_T)) {
        // one rank holds every head: the single-launch step over the arena (decode_mk.cu)
        MkArgs a;
        a.params = m->param_buf;
        a.wte = w->wte;
        a.wpe = w->wpe;
        a.L = L;
        a.C = C;
        a.H = t->H;
        a.V = t->V;
        a.block = m->cfg.block_size;
        a.B = B;
        a.Tmax = t->kv_T;
        a.scale = 1.0f / sqrtf((float)t->hs);
        a.x = t->xl;
        a.qkv = t->qkv;
        a.att = t->al;
        a.hid = t->hid;
        a.logits = t->logits;
        a.ldlog = t->ldlog;
        a.kc = t->kc;
        a.vc = t->vc;
        a.part = t->dec_part;
        a.tickets = (int *)(t->dec_part + mk_part_floats(B, t->H, t->kv_T));
        a.S = (int)((t->kv_T + 63) / 64);
        a.next = t->next;
        a.gen = t->gen;
        a.ctr = t->ctr;
        a.am_key = t->am_key;
        a.bar = t->mk_bar;
        a.abort = (int *)(t->mk_bar + 1);
        a.fast_act = 0;  // accurate tanh, as the GEMV decode path
        return decode_step_mk(a, s);
    }
    float *x = t->xl;
    CG_TRY(embed_fwd_at(t->next, w->wte, w->wpe, x, B, C, t->ctr, s));
    const size_t per = (size_t)t->kv_B * t->kv_T * Cl;
    // with peer memory, each row-split GEMV pushes its partial sums to every
    // rank and tp_reduce_kernel adds them (and the LayerNorm statistics for
    // the next GEMV); otherwise the partials go through ncclAllReduce
    const bool push = t->d_peers && B <= TP_MAX_ROWS;
    auto partial = [&](int k, const float *bias) {
        GemmEpi e = epi_partial(t, x, C, bias);
        if (push) {
            e.push_bufs = t->d_peers;
            e.push_world = t->world;
            e.push_rank = t->rank;
            e.push_ld = C;
            e.push_k = k;
            e.push_nk = 2 * L;
            e.push_step = t->d_step;
            e.push_ticket = t->d_ticket;
        }
        return e;
    };
    auto exchange = [&](int k) -> int {
        if (!push) return allreduce(t, x, (size_t)B * C, s);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(B);
        cfg.blockDim = dim3(256);
        cfg.stream = s;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        CG_CUDA(cudaLaunchKernelEx(&cfg, tp_reduce_kernel, t->pbuf, t->world, C, (const int *)t->d_step, 2 * L, k,
                                   x, t->d_stats));
        ++g_launch_count;
        return OK;
    };
    for (int l = 0; l < L; ++l) {
        GemmEpi eq = epi_store(t->qkv, 3 * Cl, t->qkv_b(l));
        eq.kc = t->kc + l * per;
        eq.vc = t->vc + l * per;
        eq.kv_ld = (long)t->kv_T * Cl;
        eq.kv_pos = t->ctr;
        eq.kv_C = Cl;
        CG_TRY(gemm_ln(x, C, w->ln1_w[l], w->ln1_b[l], (push && l > 0) ? t->d_stats : nullptr, t->ln,
                       t->qkv_w(l), C, B, 3 * Cl, C, eq, s));
        CG_TRY(attention_decode_at(t->qkv, 3L * Cl, t->kc + l * per, t->vc + l * per, t->kv_T, t->ctr,
                                   t->al, B, Cl, t->p.nh, t->dec_part, s));
        CG_TRY(gemm(t->al, Cl, false, w->c_proj_w[l] + (size_t)t->p.h0 * t->hs, C, false, B, C, Cl,
                    partial(2 * l, w->c_proj_b[l]), s));
        CG_TRY(exchange(2 * l));
        GemmEpi g;
        g.mode = EPI_GELU;
        g.bias = w->mlp_fc_b[l] + t->p.f0;
        g.D2 = t->hid;
        g.ldd2 = nf;
        CG_TRY(gemm_ln(x, C, w->ln2_w[l], w->ln2_b[l], push ? t->d_stats : nullptr, t->ln,
                       w->mlp_fc_w[l] + (size_t)t->p.f0 * C, C, B, nf, C, g, s));
        CG_TRY(gemm(t->hid, nf, false, w->mlp_proj_w[l] + t->p.f0, 4L * C, false, B, C, nf,
                    partial(2 * l + 1, w->mlp_proj_b[l]), s));
        CG_TRY(exchange(2 * l + 1));
    }
    GemmEpi eh = epi_store(t->logits, t->ldlog, nullptr);
    eh.argmax_key = t->am_key;
    CG_TRY(gemm_ln(x, C, w->ln_f_w, w->ln_f_b, (push && L > 0) ? t->d_stats : nullptr, t->ln,
                   w->wte + (size_t)t->p.v0 * C, C, B, t->p.nv, C, eh, s));
    CG_TRY(greedy_finalize(t->am_key, B, nullptr, nullptr, nullptr, t->pairs, nullptr, s));
    CG_TRY(greedy(t, B, s, true));
    CG_TRY(decode_advance(t->ctr, s));
    if (push) {  // the exchange numbering advances once per step
        step_advance_kernel<<<1, 32, 0, s>>>(t->d_step);
        ++g_launch_count;
        CG_CUDA(cudaGetLastError());
    }
    return OK;
}

int capture_step(const GPT *m, TpState *t, int B) {
    if (t->graph && t->graph_B == B && t->graph_T == t->kv_T && t->graph_prec == precision()) return OK;
    drop_graph(t);
    cudaGraph_t g = nullptr;
    CG_CUDA(cudaStreamBeginCapture(t->cap_stream, cudaStreamCaptureModeThreadLocal));
    const int st = decode_step(m, t, B, t->cap_stream);
    const cudaError_t e = cudaStreamEndCapture(t->cap_stream, &g);
    if (st != OK) {
        if (g) cudaGraphDestroy(g);
        return st;
    }
    if (e != cudaSuccess) {
        set_last_error(ERR_CUDA, "tp decode graph capture: %s", cudaGetErrorString(e));
        return ERR_CUDA;
    }
    const cudaError_t ei = cudaGraphInstantiate(&t->graph, g, 0);
    cudaGraphDestroy(g);
    if (ei != cudaSuccess) {
        t->graph = nullptr;
        set_last_error(ERR_CUDA, "tp decode graph instantiate: %s", cudaGetErrorString(ei));
        return ERR_CUDA;
    }
    t->graph_B = B;
    t->graph_T = t->kv_T;
    t->graph_prec = precision();
    return OK;
}

void release(TpState *t) {
    cudaStreamSynchronize(g_stream);
    if (t->cap_stream) cudaStreamSynchronize(t->cap_stream);
    drop_graph(t);  // before the communicator its NCCL nodes use
    // No collective here: a peer pushes into this rank's buffer only before
    // raising the flag this rank waited for, so once every call of this rank
    // has completed no peer writes into it any more (all ranks make the same
    // calls), and a rank whose tp_init failed must not wait for the others.
    for (int r = 0; r < TP_MAX_WORLD; ++r)
        if (t->peer[r] && t->peer[r] != t->pbuf) cudaIpcCloseMemHandle(t->peer[r]);
    dev_free(t->pbuf);
    dev_free(t->d_peers);
    dev_free(t->d_step);
    dev_free(t->d_ticket);
    dev_free(t->d_stats);
    dev_free(t->am_key);
    dev_free(t->mk_bar);
    float *bufs[] = {t->wbuf, t->x,  t->ln,     t->qkv, t->aout, t->hid, t->mean, t->rstd,
                     t->xl,   t->al, t->logits, t->lgath, t->kc,  t->vc, t->dec_part};
    for (auto b : bufs) dev_free(b);
    int *ibufs[] = {t->pairs, t->gath, t->tok, t->next, t->gen, t->ctr};
    for (auto b : ibufs) dev_free(b);
    if (t->ev_a) cudaEventDestroy(t->ev_a);
    if (t->ev_b) cudaEventDestroy(t->ev_b);
    if (t->cap_stream) cudaStreamDestroy(t->cap_stream);
    fast_free(&t->fctx);
    nccl_comm_destroy(t->comm);
    delete t;
}

// Peer memory for the decode exchange: every rank allocates its receive
// buffer, the IPC handles are all-gathered over NCCL, and each rank maps the
// others' buffers (NVLink peer access). Plain loads and stores only.
int setup_peers(TpState *t) {
    const size_t bytes = tp_buf_bytes(t->world, t->C);
    CG_TRY(dev_alloc((void **)&t->pbuf, bytes, false));
    CG_CUDA(cudaMemset(t->pbuf, 0, bytes));
    CG_CUDA(cudaDeviceSynchronize());  // zeroed before the agreement below lets any peer push
    cudaIpcMemHandle_t h;
    CG_CUDA(cudaIpcGetMemHandle(&h, t->pbuf));
    static_assert(sizeof(cudaIpcMemHandle_t) % 4 == 0, "handle size");
    const size_t words = sizeof(cudaIpcMemHandle_t) / 4;
    int *dh = nullptr;
    CG_TRY(dev_alloc((void **)&dh, (t->world + 1) * sizeof(cudaIpcMemHandle_t), false));
    CG_CUDA(cudaMemcpy(dh, &h, sizeof(h), cudaMemcpyHostToDevice));
    int st = nccl_allgather_words(dh, dh + words, words, t->comm, g_stream);
    std::vector<cudaIpcMemHandle_t> all(t->world);
    if (st == OK && cudaStreamSynchronize(g_stream) == cudaSuccess &&
        cudaMemcpy(all.data(), dh + words, t->world * sizeof(h), cudaMemcpyDeviceToHost) == cudaSuccess) {
        for (int r = 0; r < t->world && st == OK; ++r) {
            if (r == t->rank) {
                t->peer[r] = t->pbuf;
                continue;
            }
            void *p = nullptr;
            if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                set_last_error(ERR_CUDA, "tp_init: mapping rank %d's buffer failed: %s", r,
                               cudaGetErrorString(cudaGetLastError()));
                st = ERR_CUDA;
            }
            t->peer[r] = (char *)p;
        }
    } else if (st == OK) {
        set_last_error(ERR_CUDA, "tp_init: exchanging buffer handles failed");
        st = ERR_CUDA;
    }
    dev_free(dh);
    // every rank learns whether every rank mapped its peers (all ranks reach
    // this collective, failed or not), so that either all ranks continue or
    // all return the error; it also orders every buffer's zeroing before any
    // rank can push into it
    float *flag = nullptr;
    CG_TRY(dev_alloc((void **)&flag, sizeof(float), false));
    const float bad = st == OK ? 0.f : 1.f;
    cudaMemcpy(flag, &bad, sizeof(float), cudaMemcpyHostToDevice);
    const int st2 = nccl_allreduce_sum(flag, 1, t->comm, g_stream);
    float nbad = 1.f;
    cudaStreamSynchronize(g_stream);
    cudaMemcpy(&nbad, flag, sizeof(float), cudaMemcpyDeviceToHost);
    dev_free(flag);
    if (st != OK) return st;
    if (st2 != OK) return st2;
    if (nbad != 0.f) {
        set_last_error(ERR_CUDA, "tp_init: another rank could not map the peer buffers");
        return ERR_CUDA;
    }
    CG_TRY(dev_alloc((void **)&t->d_peers, TP_MAX_WORLD * sizeof(char *), false));
    CG_CUDA(cudaMemcpy(t->d_peers, t->peer, TP_MAX_WORLD * sizeof(char *), cudaMemcpyHostToDevice));
    CG_TRY(dev_alloc((void **)&t->d_step, sizeof(int), false));
    CG_TRY(dev_alloc((void **)&t->d_ticket, sizeof(int), false));
    CG_TRY(dev_alloc((void **)&t->d_stats, 2 * TP_MAX_ROWS * sizeof(float), false));
    CG_CUDA(cudaMemset(t->d_step, 0, sizeof(int)));
    CG_CUDA(cudaMemset(t->d_ticket, 0, sizeof(int)));
    return OK;
}

}  // namespace

void tp_release(const GPT *m) {
    TpState *t = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_tp_mu);
        auto it = g_tp.find(m);
        if (it == g_tp.end()) return;
        t = it->second;
        g_tp.erase(it);
    }
    release(t);
}

}  // namespace cg

using namespace cg;

extern "C" int cngpt_cuda_tp_plan(int n_head, int n_embd, int vocab, int world, int rank, int plan[7]) {
    TpPlan p;
    CG_TRY(make_plan(n_head, n_embd, vocab, world, rank, &p));
    const int v[7] = {p.h0, p.nh, p.f0, p.nf, p.v0, p.nv, p.vpad};
    memcpy(plan, v, sizeof(v));
    return OK;
}

extern "C" int cngpt_cuda_tp_init(GPT *m, const unsigned char id[128], int world, int rank) {
    ModelCtx *c = model_ctx(m);
    if (!c) return ERR_STATE;
    tp_release(m);
    TpPlan p;
    const GPTConfig &cfg = m->cfg;
    CG_TRY(make_plan(cfg.n_head, cfg.n_embd, cfg.vocab_size, world, rank, &p));
    TpState *t = new TpState;
    fast_init(&t->fctx);
    t->world = world;
    t->rank = rank;
    t->p = p;
    t->L = cfg.n_layer;
    t->C = cfg.n_embd;
    t->V = cfg.vocab_size;
    t->H = cfg.n_head;
    t->hs = t->C / t->H;
    t->Cl = p.nh * t->hs;
    t->ldlog = (p.vpad + 3) & ~3L;
    auto fail = [&](int st) {
        release(t);
        return st;
    };
    if (world > 1) {
        const int st = nccl_comm_init(&t->comm, id, world, rank);
        if (st != OK) return fail(st);
    }
    // pack this rank's q, k and v rows (and biases) of every layer
    const size_t C = t->C, Cl = t->Cl, L = t->L, off = (size_t)p.h0 * t->hs;
    int st = dev_alloc((void **)&t->wbuf, (L * 3 * Cl * C + L * 3 * Cl) * 4, false);
    if (st != OK) return fail(st);
    for (size_t l = 0; l < L; ++l) {
        float *dw = t->wbuf + l * 3 * Cl * C;
        float *db = t->wbuf + L * 3 * Cl * C + l * 3 * Cl;
        for (size_t part = 0; part < 3; ++part) {
            const float *sw = m->params.c_attn_w[l] + (part * C + off) * C;
            const float *sb = m->params.c_attn_b[l] + part * C + off;
            if (cudaMemcpyAsync(dw + part * Cl * C, sw, Cl * C * 4, cudaMemcpyDeviceToDevice, g_stream) !=
                    cudaSuccess ||
                cudaMemcpyAsync(db + part * Cl, sb, Cl * 4, cudaMemcpyDeviceToDevice, g_stream) !=
                    cudaSuccess) {
                set_last_error(ERR_CUDA, "tp_init: packing the qkv slices failed");
                return fail(ERR_CUDA);
            }
        }
    }
    if (cudaStreamCreateWithFlags(&t->cap_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&t->ev_a, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&t->ev_b, cudaEventDisableTiming) != cudaSuccess) {
        set_last_error(ERR_CUDA, "tp_init: stream / event creation failed");
        return fail(ERR_CUDA);
    }
    st = dev_alloc((void **)&t->ctr, 2 * sizeof(int), false);
    if (st != OK) return fail(st);
    if ((st = dev_alloc((void **)&t->am_key, 8 * sizeof(unsigned long long), false)) != OK) return fail(st);
    if ((st = dev_alloc((void **)&t->mk_bar, 2 * sizeof(unsigned long long), false)) != OK) return fail(st);
    if (cudaMemset(t->am_key, 0, 8 * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(t->mk_bar, 0, 2 * sizeof(unsigned long long)) != cudaSuccess) {
        set_last_error(ERR_CUDA, "tp_init: clearing the argmax keys failed");
        return fail(ERR_CUDA);
    }
    if (world > 1 && world <= TP_MAX_WORLD && t->C <= 8 * 256 && !getenv("CNGPT_CUDA_TP_NCCL_ONLY")) {
        st = setup_peers(t);
        if (st != OK) return fail(st);
    }
    if (cudaStreamSynchronize(g_stream) != cudaSuccess) {
        set_last_error(ERR_CUDA, "tp_init: %s", cudaGetErrorString(cudaGetLastError()));
        return fail(ERR_CUDA);
    }
    std::lock_guard<std::mutex> lk(g_tp_mu);
    g_tp[m] = t;
    return OK;
}

extern "C" int cngpt_cuda_tp_forward_last(GPT *m, const int *tokens, int B, int T, float *logits_out) {
    TpState *t = tp_state(m);
    if (!t) return ERR_STATE;
    if (B <= 0 || T <= 0 || T > m->cfg.block_size) {
        set_last_error(ERR_ARG, "tp_forward_last: bad shape B=%d T=%d", B, T);
        return ERR_ARG;
    }
    cudaStream_t s = g_stream;
    CG_TRY(resize(t, B, T));
    const int *tok = nullptr;
    CG_TRY(stage_tokens(tokens, (size_t)B * T, &t->tok, &t->tok_cap, &tok, s));
    CG_TRY(prefill(m, t, tok, B, T, false, s));
    if (!logits_out) {
        CG_CUDA(cudaStreamSynchronize(s));
        return check_device_error();
    }
    const float *g = t->logits;
    if (t->world > 1) {
        CG_TRY(nccl_allgather_words(t->logits, t->lgath, (size_t)B * t->ldlog, t->comm, s));
        g = t->lgath;
    }
    std::vector<float> h((size_t)t->world * B * t->ldlog);
    CG_CUDA(cudaMemcpyAsync(h.data(), g, h.size() * 4, cudaMemcpyDeviceToHost, s));
    CG_CUDA(cudaStreamSynchronize(s));
    CG_TRY(check_device_error());
    for (int r = 0; r < t->world; ++r) {
        const int v0 = r * t->p.vpad, nv = std::min(t->p.vpad, t->V - v0);
        for (int b = 0; b < B; ++b)
            memcpy(logits_out + (size_t)b * t->V + v0, h.data() + ((size_t)r * B + b) * t->ldlog,
                   (size_t)nv * 4);
    }
    return OK;
}

extern "C" int cngpt_cuda_tp_set_decode_mode(GPT *m, int mode) {
    TpState *t = tp_state(m);
    if (!t) return ERR_STATE;
    if (mode < 0 || mode > 2) {
        set_last_error(ERR_ARG, "tp_set_decode_mode: mode %d (0 auto, 1 split, 2 replicated)", mode);
        return ERR_ARG;
    }
    t->decode_mode = mode;
    return OK;
}

extern "C" int cngpt_cuda_tp_generate(GPT *m, const int *prompt, int B, int T, int n_new, int *out_tokens) {
    TpState *t = tp_state(m);
    if (!t) return ERR_STATE;
    if (B <= 0 || T <= 0 || n_new <= 0 || T + n_new - 1 > m->cfg.block_size) {
        set_last_error(ERR_ARG, "tp_generate: B=%d T=%d n_new=%d exceeds block_size %d", B, T, n_new,
                       m->cfg.block_size);
        return ERR_ARG;
    }
    // At batch 1 a split step is bound by its two exchanges per layer (a few
    // microseconds each over NVLink, 96 per GPT-2 XL token) rather than by its
    // weight stream, which it divides by the world size: measured on B200, a
    // split step at batch 1 is slower than one GPU at every world size, and
    // faster at batch 8. Every rank holds the whole model, so at batch 1 each
    // rank runs the one-GPU decode itself, bit-identically (same weights, same
    // deterministic kernels), and no exchange is needed.
    const bool replicate = t->world > 1 && (t->decode_mode == 2 || (t->decode_mode == 0 && B == 1));
    if (replicate) return cngpt_cuda_generate(m, &t->fctx, prompt, B, T, n_new, out_tokens);
    cudaStream_t s = g_stream;
    CG_TRY(resize(t, B, T));
    const int Tmax = T + n_new;
    const size_t Cl = t->Cl, L = t->L;
    if (t->kv_B != B || t->kv_T < Tmax) {
        CG_CUDA(cudaStreamSynchronize(s));
        CG_CUDA(cudaStreamSynchronize(t->cap_stream));
        drop_graph(t);
        dev_free(t->kc);
        dev_free(t->vc);
        dev_free(t->next);
        dev_free(t->dec_part);
        t->kc = t->vc = t->dec_part = nullptr;
        t->next = nullptr;
        CG_TRY(dev_alloc((void **)&t->kc, L * B * Tmax * Cl * 4, false));
        CG_TRY(dev_alloc((void **)&t->vc, L * B * Tmax * Cl * 4, false));
        CG_TRY(dev_alloc((void **)&t->dec_part, attention_decode_scratch_floats(B, t->p.nh, Tmax) * 4, false));
        CG_CUDA(cudaMemsetAsync(t->dec_part, 0, attention_decode_scratch_floats(B, t->p.nh, Tmax) * 4, s));
        CG_TRY(dev_alloc((void **)&t->next, (size_t)B * 4, false));
        t->kv_B = B;
        t->kv_T = Tmax;
    }
    if ((size_t)B * n_new > t->gen_cap) {
        CG_CUDA(cudaStreamSynchronize(s));
        CG_CUDA(cudaStreamSynchronize(t->cap_stream));
        drop_graph(t);
        dev_free(t->gen);
        t->gen = nullptr;
        CG_TRY(dev_alloc((void **)&t->gen, (size_t)B * n_new * 4, false));
        t->gen_cap = (size_t)B * n_new;
    }
    const int *tok = nullptr;
    CG_TRY(stage_tokens(prompt, (size_t)B * T, &t->tok, &t->tok_cap, &tok, s));
    const int ctr0[2] = {T - 1, 0};
    CG_CUDA(cudaMemcpyAsync(t->ctr, ctr0, sizeof(ctr0), cudaMemcpyHostToDevice, s));
    CG_TRY(prefill(m, t, tok, B, T, true, s));
    CG_TRY(greedy(t, B, s));
    CG_TRY(decode_advance(t->ctr, s));
    if (n_new > 1) {
        CG_CUDA(cudaEventRecord(t->ev_a, s));
        CG_CUDA(cudaStreamWaitEvent(t->cap_stream, t->ev_a, 0));
        CG_TRY(decode_step(m, t, B, t->cap_stream));
        if (n_new > 2) {
            CG_TRY(capture_step(m, t, B));
            for (int i = 2; i < n_new; ++i) CG_CUDA(cudaGraphLaunch(t->graph, t->cap_stream));
        }
        CG_CUDA(cudaEventRecord(t->ev_b, t->cap_stream));
        CG_CUDA(cudaStreamWaitEvent(s, t->ev_b, 0));
    }
    std::vector<int> h((size_t)B * n_new);
    CG_CUDA(cudaMemcpyAsync(h.data(), t->gen, h.size() * 4, cudaMemcpyDeviceToHost, s));
    CG_CUDA(cudaStreamSynchronize(s));
    CG_TRY(check_device_error());
    for (int b = 0; b < B; ++b)
        for (int i = 0; i < n_new; ++i) out_tokens[(size_t)b * n_new + i] = h[(size_t)i * B + b];
    return OK;
}

// Self-test of the decode exchange's bounded wait on one GPU: a receive
// buffer of world 1 holds `partial` [rows, C] in the slot of exchange 1, and
// its flag is raised to that exchange only when `publish` is set. Without it
// nothing ever publishes, so tp_reduce_kernel's wait runs out after the wait
// limit (cngpt_cuda_set_wait_limit_ns), records DEV_ERR_TP_FLAG and leaves x
// untouched; the call then returns CNGPT_ERR_DEVICE_WAIT.
extern "C" int cngpt_cuda_selftest_tp_reduce(float *x, const float *partial, int rows, int C, int publish,
                                             float *stats) {
    if (rows < 1 || rows > TP_MAX_ROWS || C < 1 || C > 8 * 256 || !x || !partial || !stats ||
        mem_kind(x) == MEM_HOST || mem_kind(partial) == MEM_HOST || mem_kind(stats) == MEM_HOST) {
        set_last_error(ERR_ARG, "selftest_tp_reduce: rows=%d (1..%d), C=%d (1..2048), device pointers", rows,
                       TP_MAX_ROWS, C);
        return ERR_ARG;
    }
    cudaStream_t s = g_stream;
    char *buf = nullptr;
    int *step = nullptr;
    const size_t bytes = tp_buf_bytes(1, C);
    CG_TRY(dev_alloc((void **)&buf, bytes, false));
    int st = dev_alloc((void **)&step, sizeof(int), false);
    const unsigned long long flag = publish ? 1ull : 0ull;
    if (st == OK &&
        (cudaMemsetAsync(buf, 0, bytes, s) != cudaSuccess || cudaMemsetAsync(step, 0, sizeof(int), s) != cudaSuccess ||
         cudaMemcpyAsync(tp_slot(buf, 1, C, 1, 0), partial, (size_t)rows * C * 4, cudaMemcpyDeviceToDevice, s) !=
             cudaSuccess ||
         cudaMemcpyAsync(buf, &flag, sizeof(flag), cudaMemcpyHostToDevice, s) != cudaSuccess)) {
        set_last_error(ERR_CUDA, "selftest_tp_reduce: buffer set-up failed");
        st = ERR_CUDA;
    }
    if (st == OK) {
        tp_reduce_kernel<<<rows, 256, 0, s>>>(buf, 1, C, step, 1, 0, x, stats);
        ++g_launch_count;
        if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess) {
            set_last_error(ERR_CUDA, "selftest_tp_reduce: launch failed");
            st = ERR_CUDA;
        }
    }
    dev_free(buf);
    dev_free(step);
    return st != OK ? st : check_device_error();
}

extern "C" int cngpt_cuda_tp_free(GPT *m) {
    if (!model_ctx(m)) return ERR_STATE;
    tp_release(m);
    return OK;
}
