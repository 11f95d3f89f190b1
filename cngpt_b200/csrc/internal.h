// internal.h - host-side internal API of libcngpt_cuda (not exported).
#pragma once

#include <cuda_runtime.h>
#include <cstdint>
#include <cstdio>

struct CUtensorMap_st;

namespace cg {

// ---------------------------------------------------------------- errors
// Library status codes (mirrored in include/cngpt_cuda.h).
enum Status : int {
    OK = 0,
    ERR_CUDA = 1,        // a CUDA runtime call failed
    ERR_ARG = 2,         // invalid shape / pointer / alignment
    ERR_ALLOC = 3,       // device allocation failed
    ERR_DEVICE_WAIT = 4, // a bounded device-side wait gave up (see dev error code)
    ERR_NCCL = 5,        // a collective failed
    ERR_STATE = 6,       // call order / unknown model handle
};

// Device wait sites, recorded in the device error word.
enum DevError : int {
    DEV_ERR_GEMM_PRODUCER = 101,
    DEV_ERR_GEMM_MMA = 102,
    DEV_ERR_GEMM_EPILOGUE = 103,
    DEV_ERR_GEMM_TRANSFORM = 104,
    DEV_ERR_TP_FLAG = 201,  // a peer's partial sum did not arrive in time
    DEV_ERR_DECODE_BARRIER = 301,  // a grid barrier of the single-launch decode step gave up
};

void set_last_error(int status, const char *fmt, ...);
int last_status();
const char *last_message();
int check_device_error();  // reads and clears the device error words
int gemm_take_dev_error();
int attn_take_dev_error();
int tp_take_dev_error();
int attn_tc_take_dev_error();
int mk_take_dev_error();
// set the limit of every bounded device wait of one translation unit (0 on
// success); set_wait_limit_ns sets all of them
int gemm_set_wait_limit(unsigned long long ns);
int attn_set_wait_limit(unsigned long long ns);
int tp_set_wait_limit(unsigned long long ns);
int attn_tc_set_wait_limit(unsigned long long ns);
int mk_set_wait_limit(unsigned long long ns);
int set_wait_limit_ns(unsigned long long ns);

#define CG_CUDA(call)                                                                 \
    do {                                                                              \
        cudaError_t e_ = (call);                                                      \
        if (e_ != cudaSuccess) {                                                      \
            ::cg::set_last_error(::cg::ERR_CUDA, "%s:%d %s: %s", __FILE__, __LINE__,  \
                                 #call, cudaGetErrorString(e_));                      \
            return ::cg::ERR_CUDA;                                                    \
        }                                                                             \
    } while (0)

#define CG_TRY(call)                     \
    do {                                 \
        int s_ = (call);                 \
        if (s_ != ::cg::OK) return s_;   \
    } while (0)

// ------------------------------------------------------------- precision
enum Precision : int { PREC_TF32 = 0, PREC_3XTF32 = 1, PREC_FP32 = 2 };
int precision();
void set_precision(int p);

// ------------------------------------------------------------------ GEMM
enum EpiMode : int {
    EPI_STORE = 0,     // D = alpha*acc + bias
    EPI_ACCUM = 1,     // D = D + alpha*acc (+ bias)
    EPI_GELU = 2,      // t = acc + bias; D = t (if D); D2 = gelu(t)
    EPI_RESID = 3,     // t = acc + bias; D = t (if D); D2 = R + t
    EPI_GELU_BWD = 4,  // D = acc * gelu'(G)
};

struct GemmEpi {
    int mode = EPI_STORE;
    float alpha = 1.0f;
    float *D = nullptr;
    long ldd = 0;
    const float *bias = nullptr;
    float *D2 = nullptr;
    long ldd2 = 0;
    const float *R = nullptr;
    long ldr = 0;
    const float *G = nullptr;
    long ldg = 0;
    int vec4 = 0;  // set by gemm(): every pointer 16B-aligned and every pitch % 4 == 0
    int fast_act = 0;  // set by gemm() in TF32 mode: GELU epilogues use tanh_fast
    int stream_out = 0;  // STORE outputs far larger than L2: evict-first stores (pair GEMM)
    // KV-cache decode (STORE mode, D = packed qkv rows): the K and V columns
    // [kv_C, 3 kv_C) are also written to kc / vc at position *kv_pos:
    // kc[m * kv_ld + pos * kv_C + (n - kv_C)], vc likewise for n >= 2 kv_C
    float *kc = nullptr, *vc = nullptr;
    long kv_ld = 0;
    const int *kv_pos = nullptr;
    int kv_C = 0;
    // decode (RESID mode): LayerNorm statistics (mean, rstd) of each finished
    // D2 row into ln_stats_out[2m], [2m+1], for the next LayerNorm-fused GEMV;
    // ln_ticket: one int, zero before the call and left at zero after it
    float *ln_stats_out = nullptr;
    int *ln_ticket = nullptr;
    // tensor-parallel decode (GEMV path, STORE or RESID): instead of writing
    // D / D2, every value is pushed into the receive buffer of every rank
    // (peer memory over NVLink, slot = epoch & 1, source = push_rank), and the
    // last block raises this rank's flag on every rank to the epoch
    // (*push_step * push_nk + push_k + 1). Layout of each rank's buffer:
    // uint64 flags[TP_MAX_WORLD] (256 B), then float data[2][world][8][push_ld].
    char *const *push_bufs = nullptr;
    int push_world = 0, push_rank = 0, push_ld = 0, push_k = 0, push_nk = 0;
    const int *push_step = nullptr;
    int *push_ticket = nullptr;
    // greedy decode (STORE mode, D = logits rows): each row's largest value
    // (lowest column on ties) is folded into argmax_key[m] by atomicMax on an
    // order-preserving 64-bit key (keys start at zero); greedy_finalize()
    // turns the keys into tokens and clears them
    unsigned long long *argmax_key = nullptr;
    // fused cross-entropy statistics (STORE mode without bias, D = logits
    // rows): for every row m and every 64-column group p of the output, the
    // pair (max, sum of exp(x - max)) over the group's columns goes to
    // ce_part[m * ce_ld + p], ce_ld = ceil(N / 64); cross_entropy_fused()
    // merges them into the row's log-sum-exp
    float2 *ce_part = nullptr;
    int ce_ld = 0;
};

constexpr int TP_MAX_WORLD = 8;
constexpr int TP_MAX_ROWS = 8;
constexpr int TP_FLAG_BYTES = 256;
__host__ __device__ inline size_t tp_buf_bytes(int world, int ld) {
    return TP_FLAG_BYTES + (size_t)2 * world * TP_MAX_ROWS * ld * sizeof(float);
}
__host__ __device__ inline float *tp_slot(char *buf, int world, int ld, int slot, int src) {
    return (float *)(buf + TP_FLAG_BYTES) + ((size_t)slot * world + src) * TP_MAX_ROWS * ld;
}

// out[M,N] = op(A)[M,K] * op(B)[N,K]^T, with the epilogue applied per element.
// A element (m,k) is A[m*lda+k] (a_mn=false, K-major) or A[k*lda+m] (a_mn=true).
// B element (n,k) is B[n*ldb+k] (b_mn=false, K-major) or B[k*ldb+n] (b_mn=true).
int gemm(const float *A, long lda, bool a_mn, const float *B, long ldb, bool b_mn,
         int M, int N, int K, const GemmEpi &epi, cudaStream_t s);

// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialisation attribute may start before its predecessor finishes;
// it must call pdl_wait() before reading anything the predecessor writes.
// pdl_trigger() lets the dependent start launching (harmless without one).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// y = LayerNorm(X) (eps 1e-5, weights ln_w / ln_b) then the GEMM above with
// A = y (K-major, M x K). For M <= 8 the normalisation is fused into the GEMV
// (no y is written), with the row statistics taken from ln_stats (mean, rstd
// per row, e.g. written by the producer's ln_stats_out) when given, else
// computed in every block; otherwise y goes to ln_out [M, K] first.
int gemm_ln(const float *X, long ldx, const float *ln_w, const float *ln_b, const float *ln_stats,
            float *ln_out, const float *B, long ldb, int M, int N, int K, const GemmEpi &epi, cudaStream_t s);

// 2-D fp32 TMA descriptor (cached): inner x outer elements, row pitch ld;
// box0 x box1; K-major operands use the 128B swizzle, MN-major (mn_major)
// the 128B swizzle with 32-byte atoms. CUtensorMap_st is the driver API's
// struct, forward-declared at global scope so that files without <cuda.h>
// can include this header.
int make_tensor_map(CUtensorMap_st *out, const float *p, long inner, long outer, long ld, int box0, int box1,
                    bool mn_major);

// Counts of kernel launches issued by this library (for benchmarks).
extern unsigned long long g_launch_count;

int num_sms();

}  // namespace cg
