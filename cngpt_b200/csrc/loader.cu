// loader.cu - training batches from a host token array to the device, one
// batch ahead of the training step.
//
// The reference's DataLoader (src/dataloader.c:62-82) mmaps a file of uint16
// token ids and fills host int arrays inputs[b*T + t] = data[pos + b*T + t],
// targets[b*T + t] = data[pos + b*T + t + 1] (indices mod n_tokens), then
// advances pos by B*T and rewinds to 0 when pos + B*T + 1 would pass the end.
// Its training loop hands those host arrays to every step, so each step's
// forward starts with an upload. Here the same batch sequence is produced in
// device memory: the window data[pos, pos + B*T + 1) is copied into a pinned
// staging buffer, uploaded as uint16 (half the bytes of the int arrays) on a
// copy stream, and widened into the int inputs/targets by one small kernel.
// Two slots alternate, so the upload of batch i+1 runs while the step of
// batch i computes; the compute stream waits only on the slot it consumes.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>

#include "abi_common.h"
#include "model_ctx.h"

extern "C" {
#include "cngpt_cuda.h"
}

namespace cg {
namespace {

// inputs / targets of one batch from its window w[0, B*T + 1) (mod n_win:
// the window wraps only when the whole array is shorter than B*T + 1 + pos)
__global__ void widen_batch_kernel(const uint16_t *__restrict__ w, long n, int *__restrict__ inputs,
                                   int *__restrict__ targets) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        inputs[i] = (int)w[i];
        targets[i] = (int)w[i + 1];
    }
}

struct Slot {
    uint16_t *pinned = nullptr;  // host staging of the window
    uint16_t *win = nullptr;     // device copy of the window
    int *inputs = nullptr, *targets = nullptr;
    cudaEvent_t ready = nullptr;     // window uploaded and widened (copy stream)
    cudaEvent_t consumed = nullptr;  // the step that read this slot is enqueued before it (compute stream)
    cudaEvent_t staged = nullptr;    // the pinned buffer may be refilled
    bool filled = false;
    bool consumed_valid = false;
};

}  // namespace
}  // namespace cg

struct cngpt_cuda_loader {
    const uint16_t *data = nullptr;
    size_t n_tokens = 0;
    int B = 0, T = 0;
    size_t pos = 0;      // position of the next batch to stage (one batch ahead of the caller)
    int cur = 0;         // slot the next call returns
    cudaStream_t copy = nullptr;
    cg::Slot slot[2];
};

namespace cg {
namespace {

void release(cngpt_cuda_loader *dl) {
    if (dl->copy) cudaStreamSynchronize(dl->copy);
    for (Slot &s : dl->slot) {
        if (s.pinned) cudaFreeHost(s.pinned);
        dev_free(s.win);
        dev_free(s.inputs);
        dev_free(s.targets);
        if (s.ready) cudaEventDestroy(s.ready);
        if (s.consumed) cudaEventDestroy(s.consumed);
        if (s.staged) cudaEventDestroy(s.staged);
    }
    if (dl->copy) cudaStreamDestroy(dl->copy);
    delete dl;
}

// Stage the batch at dl->pos into slot k on the copy stream, then advance pos
// exactly as dataloader_next_batch does.
int prepare(cngpt_cuda_loader *dl, int k) {
    Slot &s = dl->slot[k];
    const size_t BT = (size_t)dl->B * dl->T, n = dl->n_tokens;
    // the previous upload from this pinned buffer must have finished
    if (s.filled) CG_CUDA(cudaEventSynchronize(s.staged));
    const size_t p = dl->pos;
    if (p + BT + 1 <= n) {
        memcpy(s.pinned, dl->data + p, (BT + 1) * sizeof(uint16_t));
    } else {  // only reachable when n < B*T + 1 + pos, i.e. never after a rewind
        for (size_t i = 0; i <= BT; ++i) s.pinned[i] = dl->data[(p + i) % n];
    }
    // the step that last read this slot's device buffers must be enqueued
    // before they are overwritten
    if (s.consumed_valid) CG_CUDA(cudaStreamWaitEvent(dl->copy, s.consumed, 0));
    CG_CUDA(cudaMemcpyAsync(s.win, s.pinned, (BT + 1) * sizeof(uint16_t), cudaMemcpyHostToDevice, dl->copy));
    CG_CUDA(cudaEventRecord(s.staged, dl->copy));
    const int threads = 256;
    const long blocks = std::min<long>(((long)BT + threads - 1) / threads, 148L * 8);
    widen_batch_kernel<<<(unsigned)blocks, threads, 0, dl->copy>>>(s.win, (long)BT, s.inputs, s.targets);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    CG_CUDA(cudaEventRecord(s.ready, dl->copy));
    s.filled = true;
    dl->pos += BT;
    if (dl->pos + BT + 1 > n) dl->pos = 0;
    return OK;
}

}  // namespace
}  // namespace cg

using namespace cg;

extern "C" int cngpt_cuda_loader_create(cngpt_cuda_loader **out, const unsigned short *data, size_t n_tokens,
                                        int B, int T) {
    if (!out || !data || B <= 0 || T <= 0 || n_tokens < (size_t)B * T + 1) {
        set_last_error(ERR_ARG, "loader_create: %zu tokens for B=%d T=%d (needs at least B*T+1)", n_tokens, B, T);
        return ERR_ARG;
    }
    *out = nullptr;
    cngpt_cuda_loader *dl = new (std::nothrow) cngpt_cuda_loader;
    if (!dl) {
        set_last_error(ERR_ALLOC, "loader_create: host allocation");
        return ERR_ALLOC;
    }
    dl->data = (const uint16_t *)data;
    dl->n_tokens = n_tokens;
    dl->B = B;
    dl->T = T;
    const size_t BT = (size_t)B * T;
    int st = cudaStreamCreateWithFlags(&dl->copy, cudaStreamNonBlocking) == cudaSuccess ? OK : ERR_CUDA;
    for (Slot &s : dl->slot) {
        if (st != OK) break;
        if (cudaMallocHost((void **)&s.pinned, (BT + 1) * sizeof(uint16_t)) != cudaSuccess ||
            cudaEventCreateWithFlags(&s.ready, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&s.consumed, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&s.staged, cudaEventDisableTiming) != cudaSuccess) {
            st = ERR_CUDA;
            break;
        }
        st = dev_alloc((void **)&s.win, (BT + 1) * sizeof(uint16_t), false);
        if (st == OK) st = dev_alloc((void **)&s.inputs, BT * sizeof(int), false);
        if (st == OK) st = dev_alloc((void **)&s.targets, BT * sizeof(int), false);
    }
    if (st != OK) {
        if (st == ERR_CUDA) set_last_error(ERR_CUDA, "loader_create: stream, event or pinned buffer");
        release(dl);
        return st;
    }
    *out = dl;
    return OK;
}

extern "C" int cngpt_cuda_loader_next(cngpt_cuda_loader *dl, const int **inputs, const int **targets) {
    if (!dl || !inputs || !targets) {
        set_last_error(ERR_ARG, "loader_next: null argument");
        return ERR_ARG;
    }
    const int k = dl->cur;
    Slot &s = dl->slot[k];
    Slot &o = dl->slot[k ^ 1];
    // everything enqueued so far on the compute stream includes the steps that
    // read the other slot's batch: its buffers may be refilled after that
    if (o.filled) {
        CG_CUDA(cudaEventRecord(o.consumed, g_stream));
        o.consumed_valid = true;
    }
    if (!s.filled) CG_TRY(prepare(dl, k));  // first call (or after a reset)
    CG_CUDA(cudaStreamWaitEvent(g_stream, s.ready, 0));
    *inputs = s.inputs;
    *targets = s.targets;
    // upload the following batch while this one is consumed
    CG_TRY(prepare(dl, k ^ 1));
    dl->cur = k ^ 1;
    return OK;
}

extern "C" int cngpt_cuda_loader_reset(cngpt_cuda_loader *dl) {
    if (!dl) {
        set_last_error(ERR_ARG, "loader_reset: null loader");
        return ERR_ARG;
    }
    CG_CUDA(cudaStreamSynchronize(dl->copy));
    for (Slot &s : dl->slot) s.filled = false;
    dl->pos = 0;
    dl->cur = 0;
    return OK;
}

extern "C" size_t cngpt_cuda_loader_num_batches(const cngpt_cuda_loader *dl) {
    return dl ? dl->n_tokens / ((size_t)dl->B * dl->T) : 0;
}

extern "C" void cngpt_cuda_loader_free(cngpt_cuda_loader *dl) {
    if (dl) release(dl);
}
