// model_ctx.h - device-side state attached to a caller's GPT / FastCtx
// (internal). The reference's structs are kept byte-identical, so the extra
// state lives in side tables keyed by the struct's address.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

extern "C" {
#include "cngpt/fast.h"
#include "cngpt/model.h"
}

namespace cg {

struct ModelCtx {
    GPTConfig cfg{};
    bool managed = false;
    // activation arena capacity (floats / bytes); the current layout is (B, T)
    size_t act_cap = 0, mask_cap = 0;
    int B = 0, T = 0;
    // buffers beyond the reference arena, sized for (B, T)
    size_t extra_BT = 0;      // B*T the extras were sized for
    float *dlogits = nullptr;  // [BT, ldlog], ldlog = V rounded up to 4 (TMA pitch)
    long ldlog = 0;
    float *d_x = nullptr, *d_ln = nullptr, *d_mlp = nullptr, *d_ao = nullptr, *d_qkv = nullptr;
    float *scratch = nullptr;  // LN / column-sum / attention / CE partials
    size_t scratch_bytes = 0;
    int *tok = nullptr, *tgt = nullptr;  // staged token ids
    float *dev_scalars = nullptr;        // [0] loss, [1] grad norm, [2] clip factor
    double *norm_scratch = nullptr;      // grad-norm partials (allocated by gpt_init)
    float *host_loss = nullptr;          // pinned
    const int *fwd_targets = nullptr;    // caller's targets pointer of the last forward
    bool dlogits_valid = false;
    // data parallel
    void *nccl_comm = nullptr;
    int world = 1, rank = 0;
    // gradient buckets averaged on their own stream while the backward runs
    cudaStream_t comm_stream = nullptr;
    cudaEvent_t ev_ready = nullptr, ev_done = nullptr;
};

struct FastDev {
    size_t cap_BT = 0;
    int cap_B = 0;
    float *xl = nullptr, *al = nullptr;  // last-row gathers [B, C]
    int *tok = nullptr;
    size_t tok_cap = 0;
    // KV cache for greedy decode: [L][B][Tmax][C] each
    float *kc = nullptr, *vc = nullptr;
    float *dec_part = nullptr;  // split-context decode attention partials
    int kv_B = 0, kv_T = 0;
    int *next = nullptr;   // [B] argmax tokens (the next step's input)
    int *gen = nullptr;    // [n_new][B] generated tokens
    size_t gen_cap = 0;
    int *ctr = nullptr;    // [0] position of the incoming token, [1] step index
    float *ln_stats = nullptr;  // [2][8][2] LayerNorm statistics handed between decode GEMVs
    int *ln_ticket = nullptr;   // [4] last-block tickets of the statistics GEMVs ([0..1] used)
    unsigned long long *am_key = nullptr;  // [8] greedy argmax keys of the LM-head GEMV
    unsigned long long *mk_bar = nullptr;  // grid-barrier counter + abort word of the single-launch step
    unsigned long long *mk_trace = nullptr;  // phase stamps of the last step (CNGPT_CUDA_DECODE_TRACE=1)
    // one decode step captured as a CUDA graph, reused while the key matches
    cudaStream_t cap_stream = nullptr;
    cudaEvent_t ev_a = nullptr, ev_b = nullptr;
    cudaGraphExec_t step_graph = nullptr;
    const void *graph_params = nullptr;
    int graph_B = 0, graph_T = 0, graph_prec = -1;
    const float *graph_logits = nullptr;
};

ModelCtx *model_ctx(const GPT *m);  // nullptr (and ERR_STATE recorded) if unknown
FastDev *fast_dev(const FastCtx *f, bool create);
int dev_alloc(void **p, size_t bytes, bool managed);
void dev_free(void *p);
// copy token ids to the device unless they already are device-accessible
int stage_tokens(const int *src, size_t n, int **buf, size_t *cap, const int **out, cudaStream_t s);
int dp_allreduce(ModelCtx *c, float *buf, size_t n, cudaStream_t s);

// NCCL, opened with dlopen on first use (dist.cu)
int nccl_open();
int nccl_comm_init(void **comm, const unsigned char id[128], int world, int rank);
void nccl_comm_destroy(void *comm);
int nccl_allreduce_sum(float *buf, size_t n, void *comm, cudaStream_t s);
int nccl_allgather_words(const void *src, void *dst, size_t words, void *comm, cudaStream_t s);

// tensor-parallel state of a model, released by gpt_free (tp_abi.cu)
void tp_release(const GPT *m);

}  // namespace cg
