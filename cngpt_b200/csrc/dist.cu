// dist.cu - data-parallel gradient exchange over NCCL (one process per GPU).
//
// The reference has no distributed path. Data parallelism here follows the
// plan of a single-process step over the global batch: every rank runs the
// forward/backward of its own B x T slice (mean loss over B*T), then the
// gradient arena is averaged across ranks (sum / world) before the clip norm
// and AdamW, which therefore see the gradient of the mean loss over the
// global batch on every rank.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>

#include "abi_common.h"
#include "model_ctx.h"

extern "C" {
#include "cngpt_cuda.h"
}

extern "C" int cngpt_cuda_dp_free(GPT *m);

namespace cg {

// NCCL is opened on first use rather than linked: a process that loads this
// library before PyTorch must not pin the system libnccl.so.2 ahead of the
// one PyTorch ships (and a process without collectives needs none).
namespace {
struct Nccl {
    void *h = nullptr;
    ncclResult_t (*getUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*commInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*allReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*allGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*commDestroy)(ncclComm_t) = nullptr;
    const char *(*errorString)(ncclResult_t) = nullptr;
} g_nccl;

int nccl_fail(const char *what, ncclResult_t r) {
    set_last_error(ERR_NCCL, "%s: %s", what, g_nccl.errorString(r));
    return ERR_NCCL;
}
}  // namespace

int nccl_open() {
    if (g_nccl.h) return OK;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
        set_last_error(ERR_NCCL, "cannot open libnccl.so.2: %s", dlerror());
        return ERR_NCCL;
    }
    g_nccl.getUniqueId = (decltype(g_nccl.getUniqueId))dlsym(h, "ncclGetUniqueId");
    g_nccl.commInitRank = (decltype(g_nccl.commInitRank))dlsym(h, "ncclCommInitRank");
    g_nccl.allReduce = (decltype(g_nccl.allReduce))dlsym(h, "ncclAllReduce");
    g_nccl.allGather = (decltype(g_nccl.allGather))dlsym(h, "ncclAllGather");
    g_nccl.commDestroy = (decltype(g_nccl.commDestroy))dlsym(h, "ncclCommDestroy");
    g_nccl.errorString = (decltype(g_nccl.errorString))dlsym(h, "ncclGetErrorString");
    if (!g_nccl.getUniqueId || !g_nccl.commInitRank || !g_nccl.allReduce || !g_nccl.allGather ||
        !g_nccl.commDestroy || !g_nccl.errorString) {
        set_last_error(ERR_NCCL, "libnccl.so.2 lacks an expected entry point");
        return ERR_NCCL;
    }
    g_nccl.h = h;
    return OK;
}

int nccl_comm_init(void **comm, const unsigned char id[128], int world, int rank) {
    CG_TRY(nccl_open());
    ncclUniqueId uid;
    memcpy(&uid, id, 128);
    ncclComm_t c;
    const ncclResult_t r = g_nccl.commInitRank(&c, world, uid, rank);
    if (r != ncclSuccess) return nccl_fail("ncclCommInitRank", r);
    *comm = c;
    return OK;
}

void nccl_comm_destroy(void *comm) {
    if (comm && g_nccl.h) g_nccl.commDestroy((ncclComm_t)comm);
}

int nccl_allreduce_sum(float *buf, size_t n, void *comm, cudaStream_t s) {
    const ncclResult_t r = g_nccl.allReduce(buf, buf, n, ncclFloat, ncclSum, (ncclComm_t)comm, s);
    return r == ncclSuccess ? OK : nccl_fail("ncclAllReduce", r);
}

int nccl_allgather_words(const void *src, void *dst, size_t words, void *comm, cudaStream_t s) {
    const ncclResult_t r = g_nccl.allGather(src, dst, words, ncclInt32, (ncclComm_t)comm, s);
    return r == ncclSuccess ? OK : nccl_fail("ncclAllGather", r);
}

int dp_allreduce(ModelCtx *c, float *buf, size_t n, cudaStream_t s) {
    if (c->world <= 1 || !c->nccl_comm) return OK;
    ncclResult_t r = g_nccl.allReduce(buf, buf, n, ncclFloat, ncclAvg, (ncclComm_t)c->nccl_comm, s);
    return r == ncclSuccess ? OK : nccl_fail("ncclAllReduce", r);
}

}  // namespace cg

using namespace cg;

extern "C" int cngpt_cuda_dp_unique_id(unsigned char id[128]) {
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    CG_TRY(nccl_open());
    ncclUniqueId uid;
    ncclResult_t r = g_nccl.getUniqueId(&uid);
    if (r != ncclSuccess) {
        set_last_error(ERR_NCCL, "ncclGetUniqueId: %s", g_nccl.errorString(r));
        return ERR_NCCL;
    }
    memcpy(id, &uid, 128);
    return OK;
}

extern "C" int cngpt_cuda_dp_init(GPT *m, const unsigned char id[128], int world, int rank) {
    ModelCtx *c = model_ctx(m);
    if (!c) return ERR_STATE;
    if (world < 1 || rank < 0 || rank >= world) {
        set_last_error(ERR_ARG, "dp_init: rank %d / world %d", rank, world);
        return ERR_ARG;
    }
    // a second dp_init replaces the communicator of the first
    if (c->nccl_comm) cngpt_cuda_dp_free(m);
    c->world = 1;
    c->rank = 0;
    if (world == 1) return OK;
    // the gradient buckets' stream: non-blocking (no implicit order with the
    // legacy default stream) and at the highest priority, so the collectives
    // start as soon as their bucket is final
    if (!c->comm_stream) {
        int lo = 0, hi = 0;
        CG_CUDA(cudaDeviceGetStreamPriorityRange(&lo, &hi));
        CG_CUDA(cudaStreamCreateWithPriority(&c->comm_stream, cudaStreamNonBlocking, hi));
        CG_CUDA(cudaEventCreateWithFlags(&c->ev_ready, cudaEventDisableTiming));
        CG_CUDA(cudaEventCreateWithFlags(&c->ev_done, cudaEventDisableTiming));
    }
    void *comm = nullptr;
    CG_TRY(nccl_comm_init(&comm, id, world, rank));
    c->nccl_comm = comm;
    c->world = world;
    c->rank = rank;
    return OK;
}

extern "C" int cngpt_cuda_dp_allreduce_grads(GPT *m) {
    ModelCtx *c = model_ctx(m);
    if (!c) return ERR_STATE;
    return dp_allreduce(c, m->grad_buf, (size_t)m->n_params, g_stream);
}

extern "C" int cngpt_cuda_dp_free(GPT *m) {
    ModelCtx *c = model_ctx(m);
    if (!c) return ERR_STATE;
    cudaStreamSynchronize(g_stream);
    if (c->comm_stream) cudaStreamSynchronize(c->comm_stream);
    if (c->nccl_comm) {
        nccl_comm_destroy(c->nccl_comm);
        c->nccl_comm = nullptr;
    }
    if (c->comm_stream) {
        cudaStreamDestroy(c->comm_stream);
        cudaEventDestroy(c->ev_ready);
        cudaEventDestroy(c->ev_done);
        c->comm_stream = nullptr;
        c->ev_ready = c->ev_done = nullptr;
    }
    c->world = 1;
    c->rank = 0;
    return OK;
}
