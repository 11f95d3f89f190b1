// ops_abi.cu - the C entry points of cngpt/ops.h and the generic parts of
// cngpt_cuda.h (status, configuration, GEMM, attention, copies).
//
// Each ops.h function keeps the reference's signature and meaning
// (src/ops.c); arguments in plain host memory are staged through device
// buffers and copied back before returning, arguments in device memory are
// used in place, and managed or host arguments make the call synchronous
// (the reference's calls are synchronous CPU code).
#include <cstdlib>
#include <cstring>
#include <vector>

#include "abi_common.h"
#include "common.cuh"
#include "decode_mk.h"
#include "kernels.h"

extern "C" {
#include "cngpt_cuda.h"
}

namespace cg {

cudaStream_t g_stream = 0;
bool g_managed = getenv("CNGPT_CUDA_MANAGED") && atoi(getenv("CNGPT_CUDA_MANAGED")) != 0;

int mem_kind(const void *p) {
    if (!p) return MEM_DEVICE;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return MEM_HOST;
    }
    if (a.type == cudaMemoryTypeDevice) return MEM_DEVICE;
    if (a.type == cudaMemoryTypeManaged) return MEM_MANAGED;
    return MEM_HOST;
}

Stage::~Stage() {
    for (int i = 0; i < n; ++i)
        if (e[i].dev) cudaFree(e[i].dev);
}

void *Stage::add(const void *p, size_t bytes, bool copy_in, bool copy_out) {
    if (!p) return nullptr;
    const int k = mem_kind(p);
    if (k == MEM_MANAGED) sync = true;
    if (k != MEM_HOST) return const_cast<void *>(p);
    sync = true;
    if (n >= 12) {
        set_last_error(ERR_ARG, "too many host arguments");
        status = ERR_ARG;
        return nullptr;
    }
    void *d = nullptr;
    if (cudaMalloc(&d, bytes ? bytes : 4) != cudaSuccess) {
        cudaGetLastError();
        set_last_error(ERR_ALLOC, "staging allocation of %zu bytes failed", bytes);
        status = ERR_ALLOC;
        return nullptr;
    }
    if (copy_in && bytes && cudaMemcpyAsync(d, p, bytes, cudaMemcpyHostToDevice, g_stream) != cudaSuccess) {
        set_last_error(ERR_CUDA, "staging copy failed");
        status = ERR_CUDA;
    }
    e[n++] = {const_cast<void *>(p), d, bytes, copy_out};
    return d;
}

int Stage::finish(int st) {
    if (status != OK) return status;
    if (st != OK) return st;
    for (int i = 0; i < n; ++i)
        if (e[i].copy_out && e[i].bytes)
            CG_CUDA(cudaMemcpyAsync(e[i].host, e[i].dev, e[i].bytes, cudaMemcpyDeviceToHost, g_stream));
    if (sync) {
        CG_CUDA(cudaStreamSynchronize(g_stream));
        CG_TRY(check_device_error());
    }
    return OK;
}

// Grow-only device scratch for op-level calls (model calls use their own).
void *op_scratch(size_t bytes) {
    static void *p = nullptr;
    static size_t cap = 0;
    if (bytes <= cap) return p;
    cudaStreamSynchronize(g_stream);
    if (p) cudaFree(p);
    cap = 0;
    p = nullptr;
    size_t want = std::max(bytes, (size_t)1 << 20);
    if (cudaMalloc(&p, want) != cudaSuccess) {
        cudaGetLastError();
        set_last_error(ERR_ALLOC, "scratch allocation of %zu bytes failed", want);
        return nullptr;
    }
    cap = want;
    return p;
}

}  // namespace cg

using namespace cg;

// ============================================================ ops.h

extern "C" void linear_fwd(const float *X, const float *W, const float *b, float *Y, int M, int K,
                           int N) {
    Stage st;
    const float *x = st.in(X, (size_t)M * K), *w = st.in(W, (size_t)N * K), *bb = st.in(b, (size_t)N);
    float *y = st.out(Y, (size_t)M * N);
    int s = st.status;
    if (s == OK) {
        GemmEpi e;
        e.mode = EPI_STORE;
        e.D = y;
        e.ldd = N;
        e.bias = bb;
        s = gemm(x, K, false, w, K, false, M, N, K, e, g_stream);
    }
    st.finish(s);
}

extern "C" void linear_bwd_dx(const float *dY, const float *W, float *dX, int M, int K, int N) {
    Stage st;
    const float *dy = st.in(dY, (size_t)M * N), *w = st.in(W, (size_t)N * K);
    float *dx = st.inout(dX, (size_t)M * K);
    int s = st.status;
    if (s == OK) {
        GemmEpi e;
        e.mode = EPI_ACCUM;
        e.D = dx;
        e.ldd = K;
        // out [M, K]: A = dY (K-major over N), B(n=k, c=n) = W[n][k] -> MN-major, ld K
        s = gemm(dy, N, false, w, K, true, M, K, N, e, g_stream);
    }
    st.finish(s);
}

extern "C" void linear_bwd_dw(const float *dY, const float *X, float *dW, float *db, int M, int K,
                              int N) {
    Stage st;
    const float *dy = st.in(dY, (size_t)M * N), *x = st.in(X, (size_t)M * K);
    float *dw = st.inout(dW, (size_t)N * K), *dbb = st.inout(db, (size_t)N);
    int s = st.status;
    if (s == OK) {
        GemmEpi e;
        e.mode = EPI_ACCUM;
        e.D = dw;
        e.ldd = K;
        // out [N, K]: A(n, m) = dY[m][n] (MN-major, ld N); B(k, m) = X[m][k] (MN-major, ld K)
        s = gemm(dy, N, true, x, K, true, N, K, M, e, g_stream);
        if (s == OK && dbb) {
            float *scr = (float *)op_scratch(colsum_scratch_bytes(M, N));
            s = scr ? colsum_add(dy, N, M, N, dbb, scr, g_stream) : ERR_ALLOC;
        }
    }
    st.finish(s);
}

extern "C" void attn_scores(const float *Q, const float *K, float *scores, int B, int T, int hs) {
    Stage st;
    const float *q = st.in(Q, (size_t)B * T * hs), *k = st.in(K, (size_t)B * T * hs);
    float *sc = st.out(scores, (size_t)B * T * T);
    int s = st.status;
    const float scale = 1.0f / sqrtf((float)hs);
    for (int b = 0; s == OK && b < B; ++b) {
        GemmEpi e;
        e.mode = EPI_STORE;
        e.alpha = scale;
        e.D = sc + (size_t)b * T * T;
        e.ldd = T;
        s = gemm(q + (size_t)b * T * hs, hs, false, k + (size_t)b * T * hs, hs, false, T, T, hs, e,
                 g_stream);
    }
    st.finish(s);
}

extern "C" void attn_values(const float *scores, const float *V, float *out, int B, int T, int hs) {
    Stage st;
    const float *sc = st.in(scores, (size_t)B * T * T), *v = st.in(V, (size_t)B * T * hs);
    float *o = st.out(out, (size_t)B * T * hs);
    int s = st.status;
    for (int b = 0; s == OK && b < B; ++b) {
        GemmEpi e;
        e.mode = EPI_STORE;
        e.D = o + (size_t)b * T * hs;
        e.ldd = hs;
        // out[T, hs] = S[T, T] V[T, hs]: B(n=d, k=j) = V[j][d] -> MN-major, ld hs
        s = gemm(sc + (size_t)b * T * T, T, false, v + (size_t)b * T * hs, hs, true, T, hs, T, e,
                 g_stream);
    }
    st.finish(s);
}

extern "C" void layernorm_fwd(const float *x, const float *w, const float *b, float *out,
                              float *mean, float *rstd, int T, int C) {
    Stage st;
    const float *xx = st.in(x, (size_t)T * C), *ww = st.in(w, (size_t)C), *bb = st.in(b, (size_t)C);
    float *o = st.out(out, (size_t)T * C), *mn = st.out(mean, (size_t)T), *rs = st.out(rstd, (size_t)T);
    int s = st.status;
    if (s == OK) s = cg::layernorm_fwd(xx, C, ww, bb, o, C, mn, rs, T, C, g_stream);
    st.finish(s);
}

extern "C" void layernorm_bwd(const float *dout, const float *x, const float *w, const float *mean,
                              const float *rstd, float *dx, float *dw, float *db, int T, int C) {
    Stage st;
    const float *d = st.in(dout, (size_t)T * C), *xx = st.in(x, (size_t)T * C);
    const float *ww = st.in(w, (size_t)C), *mn = st.in(mean, (size_t)T), *rs = st.in(rstd, (size_t)T);
    float *ddx = st.inout(dx, (size_t)T * C), *ddw = st.inout(dw, (size_t)C), *ddb = st.inout(db, (size_t)C);
    int s = st.status;
    if (s == OK) {
        float *scr = (float *)op_scratch(layernorm_bwd_scratch_bytes(T, C));
        s = scr ? cg::layernorm_bwd(d, xx, ww, mn, rs, ddx, ddw, ddb, T, C, scr, g_stream) : ERR_ALLOC;
    }
    st.finish(s);
}

extern "C" void gelu_fwd(const float *x, float *out, int n) {
    Stage st;
    const float *xx = st.in(x, (size_t)n);
    float *o = st.out(out, (size_t)n);
    int s = st.status;
    if (s == OK) s = cg::gelu_fwd(xx, o, n, g_stream);
    st.finish(s);
}

extern "C" void gelu_bwd(const float *dout, const float *x, float *dx, int n) {
    Stage st;
    const float *d = st.in(dout, (size_t)n), *xx = st.in(x, (size_t)n);
    float *o = st.inout(dx, (size_t)n);
    int s = st.status;
    if (s == OK) s = cg::gelu_bwd(d, xx, o, n, g_stream);
    st.finish(s);
}

extern "C" void softmax_inplace(float *x, int rows, int cols) {
    Stage st;
    float *xx = st.inout(x, (size_t)rows * cols);
    int s = st.status;
    if (s == OK) s = softmax_rows(xx, rows, cols, g_stream);
    st.finish(s);
}

extern "C" void causal_mask(float *scores, int T) {
    Stage st;
    float *sc = st.inout(scores, (size_t)T * T);
    int s = st.status;
    if (s == OK) s = cg::causal_mask(sc, T, g_stream);
    st.finish(s);
}

extern "C" void cross_entropy_fwd(const float *logits, const int *targets, float *probs_out,
                                  float *loss_out, int B, int T, int V) {
    Stage st;
    const int rows = B * T;
    const float *lg = st.in(logits, (size_t)rows * V);
    const int *tg = st.in(targets, (size_t)rows);
    float *pr = st.out(probs_out, (size_t)rows * V), *ls = st.out(loss_out, 1);
    int s = st.status;
    if (s == OK) {
        float *rowterm = (float *)op_scratch((size_t)rows * sizeof(float));
        s = rowterm ? cross_entropy_rows(lg, V, tg, pr, V, nullptr, 0, 0.f, rowterm, rows, V, g_stream)
                    : ERR_ALLOC;
        if (s == OK) s = cross_entropy_loss(rowterm, rows, ls, g_stream);
    }
    st.finish(s);
}

extern "C" void cross_entropy_bwd(float *dlogits, const float *probs, const int *targets,
                                  float scale, int B, int T, int V) {
    Stage st;
    const int rows = B * T;
    float *dl = st.inout(dlogits, (size_t)rows * V);
    const float *pr = st.in(probs, (size_t)rows * V);
    const int *tg = st.in(targets, (size_t)rows);
    int s = st.status;
    if (s == OK) s = cg::cross_entropy_bwd(dl, pr, tg, scale, rows, V, g_stream);
    st.finish(s);
}

extern "C" void residual_add(float *dst, const float *src, int n) {
    Stage st;
    float *d = st.inout(dst, (size_t)n);
    const float *sr = st.in(src, (size_t)n);
    int s = st.status;
    if (s == OK) s = axpy1(d, sr, n, g_stream);
    st.finish(s);
}

// The keep mask is drawn from the host rand() stream exactly as the reference
// does (src/ops.c:610-616), so a run's mask matches the CPU build bit for bit.
extern "C" void dropout_fwd(float *x, unsigned char *mask, int n, float p) {
    if (n <= 0) return;
    std::vector<unsigned char> hm((size_t)n, 1);
    if (p > 0.0f)
        for (int i = 0; i < n; i++) {
            unsigned int r = (unsigned int)rand();
            hm[i] = (r > (unsigned int)(p * (float)RAND_MAX)) ? 1 : 0;
        }
    Stage st;
    unsigned char *mk = mask ? st.out(mask, (size_t)n) : nullptr;
    int s = st.status;
    if (s == OK && mk) {
        const cudaError_t e = cudaMemcpyAsync(mk, hm.data(), (size_t)n, cudaMemcpyHostToDevice, g_stream);
        if (e != cudaSuccess) { set_last_error(ERR_CUDA, "dropout mask upload"); s = ERR_CUDA; }
        // the staging copy-back reads the device buffer after this upload
        if (s == OK) cudaStreamSynchronize(g_stream);
    }
    if (s == OK && p > 0.0f) {
        float *xx = st.inout(x, (size_t)n);
        const unsigned char *dm = mk;
        unsigned char *tmp = nullptr;
        if (!dm) {
            if (cudaMalloc(&tmp, (size_t)n) != cudaSuccess) { cudaGetLastError(); s = ERR_ALLOC; }
            else {
                cudaMemcpy(tmp, hm.data(), (size_t)n, cudaMemcpyHostToDevice);
                dm = tmp;
            }
        }
        if (s == OK && st.status == OK) s = mask_mul(xx, dm, n, 1.0f / (1.0f - p), g_stream);
        if (tmp) {
            cudaStreamSynchronize(g_stream);
            cudaFree(tmp);
        }
    }
    st.finish(s);
}

extern "C" void dropout_bwd(float *dx, const unsigned char *mask, int n, float p) {
    if (p <= 0.0f || n <= 0) return;
    Stage st;
    float *d = st.inout(dx, (size_t)n);
    const unsigned char *mk = st.in(mask, (size_t)n);
    int s = st.status;
    if (s == OK) s = mask_mul(d, mk, n, 1.0f / (1.0f - p), g_stream);
    st.finish(s);
}

extern "C" float global_grad_norm(const float *grads, int n) {
    Stage st;
    const float *g = st.in(grads, (size_t)n);
    float result = 0.0f;
    int s = st.status;
    float *dn = (float *)op_scratch(norm_scratch_bytes() + 64);
    if (s == OK && !dn) s = ERR_ALLOC;
    if (s == OK) {
        double *part = (double *)dn;
        float *out = (float *)((char *)dn + norm_scratch_bytes());
        s = grad_norm(g, n, part, out, nullptr, 0.f, g_stream);
        if (s == OK) {
            if (cudaMemcpyAsync(&result, out, sizeof(float), cudaMemcpyDeviceToHost, g_stream) != cudaSuccess ||
                cudaStreamSynchronize(g_stream) != cudaSuccess) {
                set_last_error(ERR_CUDA, "global_grad_norm readback");
                s = ERR_CUDA;
            }
        }
    }
    st.finish(s);
    return result;
}

extern "C" void scale_grads(float *grads, int n, float sc) {
    Stage st;
    float *g = st.inout(grads, (size_t)n);
    int s = st.status;
    if (s == OK) s = cg::scale(g, n, nullptr, sc, g_stream);
    st.finish(s);
}

// ============================================================ cngpt_cuda.h (generic)

extern "C" int cngpt_cuda_last_status(void) { return last_status(); }
extern "C" const char *cngpt_cuda_last_message(void) { return last_message(); }
extern "C" void cngpt_cuda_clear_status(void) { set_last_error(OK, ""); }

extern "C" int cngpt_cuda_check(void) {
    CG_CUDA(cudaStreamSynchronize(g_stream));
    CG_CUDA(cudaGetLastError());
    return check_device_error();
}

extern "C" int cngpt_cuda_set_precision(int mode) {
    if (mode < PREC_TF32 || mode > PREC_FP32) {
        set_last_error(ERR_ARG, "unknown precision mode %d", mode);
        return ERR_ARG;
    }
    set_precision(mode);
    return OK;
}

extern "C" int cngpt_cuda_get_precision(void) { return precision(); }

extern "C" int cngpt_cuda_set_stream(void *stream) {
    g_stream = (cudaStream_t)stream;
    return OK;
}

extern "C" void *cngpt_cuda_get_stream(void) { return (void *)g_stream; }

extern "C" int cngpt_cuda_set_managed(int on) {
    g_managed = on != 0;
    return OK;
}

extern "C" unsigned long long cngpt_cuda_launch_count(void) { return g_launch_count; }

extern "C" int cngpt_cuda_set_decode_step_kernel(int on) {
    set_decode_step_kernel(on != 0);
    return OK;
}

extern "C" int cngpt_cuda_set_wait_limit_ns(unsigned long long ns) {
    // the device variables are read by kernels in flight: finish them first
    CG_CUDA(cudaDeviceSynchronize());
    return set_wait_limit_ns(ns ? ns : kWaitLimitNs);
}

extern "C" int cngpt_cuda_gemm(const float *A, long lda, int a_mn, const float *B, long ldb, int b_mn,
                               int M, int N, int K, int epi_mode, float alpha, float *D, long ldd,
                               const float *bias, float *D2, long ldd2, const float *R, long ldr,
                               const float *G, long ldg) {
    if (epi_mode < EPI_STORE || epi_mode > EPI_GELU_BWD) {
        set_last_error(ERR_ARG, "unknown epilogue %d", epi_mode);
        return ERR_ARG;
    }
    if ((epi_mode != EPI_GELU && epi_mode != EPI_RESID && !D) ||
        ((epi_mode == EPI_GELU || epi_mode == EPI_RESID) && !D2) || (epi_mode == EPI_RESID && !R) ||
        (epi_mode == EPI_GELU_BWD && !G)) {
        set_last_error(ERR_ARG, "missing epilogue operand for mode %d", epi_mode);
        return ERR_ARG;
    }
    GemmEpi e;
    e.mode = epi_mode;
    e.alpha = alpha;
    e.D = D;
    e.ldd = ldd;
    e.bias = bias;
    e.D2 = D2;
    e.ldd2 = ldd2;
    e.R = R;
    e.ldr = ldr;
    e.G = G;
    e.ldg = ldg;
    return gemm(A, lda, a_mn != 0, B, ldb, b_mn != 0, M, N, K, e, g_stream);
}

extern "C" int cngpt_cuda_attention_fwd(const float *qkv, float *out, float *lse, int B, int T, int C,
                                        int H) {
    if (H <= 0 || C % H != 0) {
        set_last_error(ERR_ARG, "attention: C=%d not divisible by H=%d", C, H);
        return ERR_ARG;
    }
    return attention_fwd(qkv, out, lse, B, T, C, H, g_stream);
}

extern "C" int cngpt_cuda_attention_bwd(const float *qkv, const float *out, const float *dout,
                                        const float *lse, float *dqkv, int B, int T, int C, int H) {
    if (H <= 0 || C % H != 0) {
        set_last_error(ERR_ARG, "attention: C=%d not divisible by H=%d", C, H);
        return ERR_ARG;
    }
    float *scr = (float *)op_scratch(attention_bwd_scratch_bytes(B, T, H));
    if (!scr) return ERR_ALLOC;
    return attention_bwd(qkv, out, dout, lse, dqkv, scr, B, T, C, H, g_stream);
}

extern "C" int cngpt_cuda_copy(void *dst, const void *src, size_t bytes) {
    CG_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, g_stream));
    CG_CUDA(cudaStreamSynchronize(g_stream));
    return OK;
}
