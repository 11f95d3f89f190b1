// noalloc.cu - LayerNorm backward that allocates no device memory.
//
// layernorm_bwd (cngpt/ops.h) reduces dw/db through a scratch buffer of
// per-chunk partial sums, which the library grows with cudaMalloc on demand.
// Some callers cannot have a library allocate behind their back: cudaMalloc
// synchronises the whole device (a stall in the middle of a latency-critical
// loop), and it fails outright for a caller that has already reserved all of
// HBM for its own pool or runs under a fixed memory budget. This entry point
// takes its scratch from a fixed-size array in the library's own device image
// instead, so the caller passes only its inputs and outputs.
#include <mutex>

#include "abi_common.h"
#include "common.cuh"
#include "kernels.h"

extern "C" {
#include "cngpt_cuda.h"
}

namespace cg {

// 512 Ki floats = 2 MiB, loaded once per GPU with the library and kept until
// the process exits. LayerNorm backward needs ceil(T / 128) * 2 * C floats
// of it, so any T * C up to about 33.5 million fits (T = 16384 rows at
// C = 2048).
constexpr size_t kNoAllocScratchFloats = 512 * 1024;
static __device__ __align__(256) float g_lnbwd_scratch[kNoAllocScratchFloats];

namespace {

constexpr int kMaxDevices = 64;
float *g_scratch_addr[kMaxDevices] = {};
std::mutex g_mu;

// Device address of the array on the current device. In host code the name
// g_lnbwd_scratch is only a host-side stand-in, so a kernel must be given the
// address cudaGetSymbolAddress returns for the device it runs on.
int scratch_address(float **out) {
    int dev = 0;
    CG_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxDevices) {
        set_last_error(ERR_ARG, "layernorm_bwd_noalloc: device ordinal %d out of range", dev);
        return ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_lnbwd_scratch);
        if (e != cudaSuccess || !p) {
            set_last_error(ERR_CUDA, "layernorm_bwd_noalloc: cudaGetSymbolAddress failed: %s",
                           cudaGetErrorString(e));
            return ERR_CUDA;
        }
        g_scratch_addr[dev] = (float *)p;
    }
    *out = g_scratch_addr[dev];
    return OK;
}

}  // namespace
}  // namespace cg

using namespace cg;

extern "C" int cngpt_cuda_layernorm_bwd_noalloc(const float *dout, const float *x, const float *w,
                                                const float *mean, const float *rstd, float *dx,
                                                float *dw, float *db, int T, int C) {
    if (T < 0 || C <= 0) {
        set_last_error(ERR_ARG, "layernorm_bwd_noalloc: bad shape T=%d C=%d", T, C);
        return ERR_ARG;
    }
    const size_t need = layernorm_bwd_scratch_bytes(T, C) / sizeof(float);
    if (need > kNoAllocScratchFloats) {
        set_last_error(ERR_ARG,
                       "layernorm_bwd_noalloc: T=%d x C=%d needs %zu floats of scratch; the static "
                       "array holds %zu (T*C up to ~33.5M)",
                       T, C, need, kNoAllocScratchFloats);
        return ERR_ARG;
    }
    const void *ptrs[] = {dout, x, w, mean, rstd, dx, dw, db};
    for (const void *p : ptrs)
        if (!p || mem_kind(p) == MEM_HOST) {
            set_last_error(ERR_ARG, "layernorm_bwd_noalloc: every argument must be device or managed "
                                    "memory (host memory would need staging buffers)");
            return ERR_ARG;
        }
    float *scratch = nullptr;
    CG_TRY(scratch_address(&scratch));
    // every scratch element the reduction reads is written earlier in this
    // same call, so the previous call's contents need no clearing
    return layernorm_bwd(dout, x, w, mean, rstd, dx, dw, db, T, C, scratch, g_stream);
}
