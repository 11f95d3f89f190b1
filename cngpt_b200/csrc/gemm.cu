// gemm.cu - fp32-in / fp32-out GEMMs on the sm_100a tensor cores.
//
// One persistent, warp-specialised kernel covers every contraction of the
// reference's linear layers (src/ops.c:109-149 and the call sites in
// src/model.c / src/fast.c):
//
//   warp 0      TMA producer: 128B-swizzled tiles of A and B into a ring of
//               shared-memory stages (plain per-CTA loads of this GPU's memory)
//   warp 1      MMA issuer: tcgen05.mma.kind::tf32, 128 x BN x 8 per
//               instruction, accumulating into one of two TMEM buffers
//   warps 2-9   epilogue: tcgen05.ld of the finished accumulator, then the
//               fused bias / GELU / residual / accumulate / GELU-backward
//               step and the global stores, overlapping the next tile's
//               main loop (double-buffered TMEM)
//   warps 10-13 (3xTF32 only) split transform: each staged fp32 tile x is
//               rewritten as hi = rna_tf32(x) in place and lo = rna_tf32(x-hi)
//               into a twin buffer, and the MMA warp issues lo*hi + hi*lo +
//               hi*hi into a fresh accumulator per 32-wide k-block; the
//               epilogue warps add those partials in fp32 registers. The
//               tensor core accumulates with truncation, so its error grows
//               with the number of accumulation steps (measured: ~7e-9*K
//               normwise for one accumulator over K); per-k-block partials keep
//               3xTF32 at fp32-level accuracy for any K
//
// The warp roles above are the single-CTA kernel's (gemm_tc_kernel: 3xTF32,
// short M). The TF32 CTA-pair kernel (gemm_tc2_kernel: two CTAs of a
// cluster share one 256-row tile through tcgen05.mma.cta_group::2, tile
// widths 256 / 192 / 128) runs BN / 16 epilogue warps that read the
// accumulator in the 16x256b layout and store from registers (store_frag),
// one instantiation per epilogue mode of the training step; the LM head
// keeps an 8-warp epilogue that transposes through shared memory
// (store_block) and folds the cross-entropy statistics.
//
// Operands may be K-major or MN-major in global memory (the instruction
// descriptor's transpose bits), so X W^T (forward), dY W (dX) and dY^T X (dW)
// all load straight from their row-major buffers without a transpose pass.
// Shapes or pointers TMA cannot describe (row pitch not a multiple of 16
// bytes, unaligned base) run a CUDA-core fp32 kernel instead.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "kernels.h"

namespace cg {

unsigned long long g_launch_count = 0;

CG_DEV_ERROR_ACCESSORS(gemm_take_dev_error, gemm_set_wait_limit)

namespace {

constexpr int BM = 128;
constexpr int BK = 32;              // fp32 elements per k-block = one 128B swizzle row
constexpr int KB_BYTES = BK * 4;    // 128
constexpr int MMA_K = 8;            // tf32 K per tcgen05.mma

template <int BN, bool SPLIT>
struct Cfg {
    static constexpr int A_BYTES = BM * KB_BYTES;
    static constexpr int B_BYTES = BN * KB_BYTES;
    static constexpr int STAGE_BYTES = (A_BYTES + B_BYTES) * (SPLIT ? 2 : 1);
    static constexpr int STAGES = SPLIT ? 3 : (BN == 256 ? 4 : 6);
    static constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter, each half the columns
    static constexpr int THREADS = (2 + EPI_WARPS + (SPLIT ? 4 : 0)) * 32;
    static constexpr int TMEM_COLS = 2 * BN;  // two accumulators
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256 + EPI_WARPS * 32 * 33 * 4;
};

struct SmemCtl {
    uint64_t full[8];
    uint64_t empty[8];
    uint64_t ready[8];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint32_t tmem_base;
    int abort;
};

// Fused epilogue for one output element (m, n) holding the raw product a;
// `aux` is the element's prefetched second operand (D for ACCUM, R for RESID,
// G for GELU_BWD).
// D is the output in place of e.D (the split-K kernels offset it per split).
__device__ __forceinline__ void epi_apply_d(const GemmEpi &e, float *D, long m, int n, float a, float bias,
                                            float aux) {
    a *= e.alpha;
    switch (e.mode) {
        case EPI_STORE:
            D[m * e.ldd + n] = a + bias;
            break;
        case EPI_ACCUM:
            D[m * e.ldd + n] = (aux + a) + bias;
            break;
        case EPI_GELU:
            a += bias;
            if (D) D[m * e.ldd + n] = a;
            e.D2[m * e.ldd2 + n] = gelu_tanh(a, e.fast_act);
            break;
        case EPI_RESID:
            a += bias;
            if (D) D[m * e.ldd + n] = a;
            e.D2[m * e.ldd2 + n] = aux + a;
            break;
        case EPI_GELU_BWD:
            D[m * e.ldd + n] = a * gelu_tanh_grad(aux, e.fast_act);
            break;
    }
}

__device__ __forceinline__ void epi_apply(const GemmEpi &e, long m, int n, float a, float bias, float aux) {
    epi_apply_d(e, e.D, m, n, a, bias, aux);
}

__device__ __forceinline__ const float *epi_aux(const GemmEpi &e, long &ld) {
    switch (e.mode) {
        case EPI_ACCUM: ld = e.ldd; return e.D;
        case EPI_RESID: ld = e.ldr; return e.R;
        case EPI_GELU_BWD: ld = e.ldg; return e.G;
        default: ld = 0; return nullptr;
    }
}

// Cross-entropy statistics of one row's 32 columns [n0, n0 + 32) (thread =
// row, v its raw products), folded into the running (max, sum exp(x - max))
// of the row's current 64-column group. `fast` (TF32 mode, GemmEpi::fast_act)
// sums the terms with the __expf intrinsic: each term is <= 1 and the group
// sum is dominated by the terms near the maximum, where its error is a few
// ulp - far below the TF32 products' own error.
__device__ __forceinline__ void ce_fold(const float (&v)[32], int n0, int N, float alpha, float &m, float &s,
                                        bool fast) {
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < 32; ++j)
        if (n0 + j < N) mx = fmaxf(mx, v[j] * alpha);
    if (mx == -INFINITY) return;
    float add = 0.f;
    if (fast) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (n0 + j < N) add += __expf(v[j] * alpha - mx);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (n0 + j < N) add += expf(v[j] * alpha - mx);
    }
    if (mx > m) {
        s = s * expf(m - mx) + add;
        m = mx;
    } else {
        s += add * expf(mx - m);
    }
}

// After chunk c (of 32 columns starting at n0) of a row: every second chunk
// closes a 64-column group, whose (max, sum) is stored and reset.
__device__ __forceinline__ void ce_flush(const GemmEpi &ep, int c, long m, int n0, int M, int N, float &cm,
                                         float &cs) {
    if (!(c & 1)) return;
    const int g0 = n0 - 32;  // first column of the group
    if (m < M && g0 < N) ep.ce_part[m * ep.ce_ld + g0 / 64] = make_float2(cm, cs);
    cm = -INFINITY;
    cs = 0.f;
}

// Epilogue of one 32x32 output block (thread = row on entry, `v` its 32
// columns): transposed through the warp's padded shared tile `stile`; lane l
// then handles row (4i + l/8) and columns 4(l%8)..+3 for i = 0..7 -
// conflict-free shared reads, 16-byte global accesses, and the epilogue mode
// switch outside the element loop.
__device__ __forceinline__ void store_block(const GemmEpi &ep, float *stile, int lane, const float (&v)[32],
                                            int m0, int n0, int M, int N, const float *aux, long ldaux) {
#pragma unroll
    for (int j = 0; j < 32; ++j) stile[lane * 33 + j] = v[j];
    __syncwarp();
    const int rsub = lane >> 3, c4 = (lane & 7) * 4;
    const int n = n0 + c4;
    if (ep.vec4 && n + 3 < N) {
        const float4 b4 = ep.bias ? *(const float4 *)(ep.bias + n) : make_float4(0.f, 0.f, 0.f, 0.f);
        const float al = ep.alpha;
        const bool fa = ep.fast_act != 0;
        auto run = [&](auto op) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int r = i * 4 + rsub;
                if (m0 + r < M) {
                    const float *sp = stile + r * 33 + c4;
                    float4 a = make_float4(sp[0] * al, sp[1] * al, sp[2] * al, sp[3] * al);
                    op((long)(m0 + r), a);
                }
            }
        };
        switch (ep.mode) {
            case EPI_STORE:
                if (ep.stream_out) {
                    run([&](long m, float4 a) {
                        __stcs((float4 *)(ep.D + m * ep.ldd + n),
                               make_float4(a.x + b4.x, a.y + b4.y, a.z + b4.z, a.w + b4.w));
                    });
                } else {
                    run([&](long m, float4 a) {
                        *(float4 *)(ep.D + m * ep.ldd + n) =
                            make_float4(a.x + b4.x, a.y + b4.y, a.z + b4.z, a.w + b4.w);
                    });
                }
                break;
            case EPI_ACCUM:
                run([&](long m, float4 a) {
                    float4 *d = (float4 *)(ep.D + m * ep.ldd + n);
                    const float4 o = *d;
                    *d = make_float4((o.x + a.x) + b4.x, (o.y + a.y) + b4.y, (o.z + a.z) + b4.z,
                                     (o.w + a.w) + b4.w);
                });
                break;
            case EPI_GELU:
                run([&](long m, float4 a) {
                    a = make_float4(a.x + b4.x, a.y + b4.y, a.z + b4.z, a.w + b4.w);
                    if (ep.D) *(float4 *)(ep.D + m * ep.ldd + n) = a;
                    *(float4 *)(ep.D2 + m * ep.ldd2 + n) =
                        make_float4(gelu_tanh(a.x, fa), gelu_tanh(a.y, fa), gelu_tanh(a.z, fa), gelu_tanh(a.w, fa));
                });
                break;
            case EPI_RESID:
                run([&](long m, float4 a) {
                    a = make_float4(a.x + b4.x, a.y + b4.y, a.z + b4.z, a.w + b4.w);
                    if (ep.D) *(float4 *)(ep.D + m * ep.ldd + n) = a;
                    const float4 r = *(const float4 *)(ep.R + m * ep.ldr + n);
                    *(float4 *)(ep.D2 + m * ep.ldd2 + n) =
                        make_float4(r.x + a.x, r.y + a.y, r.z + a.z, r.w + a.w);
                });
                break;
            case EPI_GELU_BWD:
                run([&](long m, float4 a) {
                    const float4 g = *(const float4 *)(ep.G + m * ep.ldg + n);
                    *(float4 *)(ep.D + m * ep.ldd + n) =
                        make_float4(a.x * gelu_tanh_grad(g.x, fa), a.y * gelu_tanh_grad(g.y, fa),
                                    a.z * gelu_tanh_grad(g.z, fa), a.w * gelu_tanh_grad(g.w, fa));
                });
                break;
        }
    } else {
        // ragged edge or unaligned operands: one element at a time
#pragma unroll 1
        for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + rsub;
            if (m0 + r >= M) continue;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int nj = n + j;
                if (nj >= N) break;
                const float x = aux ? aux[(long)(m0 + r) * ldaux + nj] : 0.0f;
                epi_apply(ep, m0 + r, nj, stile[r * 33 + c4 + j], ep.bias ? ep.bias[nj] : 0.0f, x);
            }
        }
    }
    __syncwarp();
    }

// ---- epilogue on the 16x256b TMEM layout (CTA-pair kernel)
//
// A 32 x 32 output block arrives as two 16-lane tcgen05.ld of 16x256b.x4:
// v[16h + 4j + 2u + e] is row 16h + 8u + lane/4, column 8j + 2(lane%4) + e of
// the block. Pair k = 8h + 2j + u (values v[2k], v[2k+1]) is one 8-byte
// access, and a warp's access of one pair covers 8 rows x 32 contiguous bytes:
// whole sectors, written straight from registers with no shared-memory
// transpose.
__device__ __forceinline__ long frag_row(int k, int lane) { return 16 * (k >> 3) + 8 * (k & 1) + (lane >> 2); }
__device__ __forceinline__ int frag_col(int k, int lane) { return 8 * ((k >> 1) & 3) + (lane & 3) * 2; }

// p[0] = o.x and, when `two`, p[1] = o.y: one 8-byte store when `vec` (p is
// then 8-byte aligned), else two scalar stores.
__device__ __forceinline__ void put2(float *p, float2 o, bool two, bool vec) {
    if (two && vec) {
        *(float2 *)p = o;
    } else {
        p[0] = o.x;
        if (two) p[1] = o.y;
    }
}

__device__ __forceinline__ float2 get2(const float *p, bool two, bool vec) {
    if (two && vec) return *(const float2 *)p;
    return make_float2(p[0], two ? p[1] : 0.f);
}

// `vec`: every operand pointer 16-byte aligned and every pitch a multiple of
// 4 floats (GemmEpi::vec4), so the pairs at even columns are 8-byte aligned.
// MODE: the epilogue mode when the kernel is specialised for one (>= 0), or
// -1 to switch on GemmEpi::mode at run time. A block wholly inside the output
// with aligned operands takes the unchecked path.
template <int MODE>
__device__ __forceinline__ void store_frag(const GemmEpi &ep, float *D, const float (&v)[32], int lane, int m0,
                                           int n0, int M, int N, const float *aux, long ldaux) {
    const bool vec = ep.vec4 != 0;
    const int mode = MODE >= 0 ? MODE : ep.mode;
    const bool full = vec && m0 + 32 <= M && n0 + 32 <= N;
    float2 b[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int n = n0 + frag_col(2 * j, lane);
        b[j] = make_float2(0.f, 0.f);
        if (ep.bias) {
            if (full) b[j] = *(const float2 *)(ep.bias + n);
            else if (n < N) b[j] = get2(ep.bias + n, n + 1 < N, vec);
        }
    }
    const float al = ep.alpha;
    const bool fa = ep.fast_act != 0;
    // two halves of 16 rows; in each, the second operands are loaded first so
    // their loads are in flight together
    auto run = [&](auto op) {
        if (full) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float2 x[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int k = 8 * h + i;
                    x[i] = aux ? *(const float2 *)(aux + (m0 + frag_row(k, lane)) * ldaux + n0 + frag_col(k, lane))
                               : make_float2(0.f, 0.f);
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int k = 8 * h + i;
                    op(m0 + frag_row(k, lane), n0 + frag_col(k, lane),
                       make_float2(v[2 * k] * al, v[2 * k + 1] * al), b[(k >> 1) & 3], x[i], true, true);
                }
            }
            return;
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float2 x[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int k = 8 * h + i;
                const long m = m0 + frag_row(k, lane);
                const int n = n0 + frag_col(k, lane);
                x[i] = aux && m < M && n < N ? get2(aux + m * ldaux + n, n + 1 < N, vec) : make_float2(0.f, 0.f);
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int k = 8 * h + i;
                const long m = m0 + frag_row(k, lane);
                const int n = n0 + frag_col(k, lane);
                if (m < M && n < N)
                    op(m, n, make_float2(v[2 * k] * al, v[2 * k + 1] * al), b[(k >> 1) & 3], x[i], n + 1 < N, vec);
            }
        }
    };
    switch (mode) {
        case EPI_STORE:
            run([&](long m, int n, float2 a, float2 bb, float2, bool two, bool vv) {
                put2(D + m * ep.ldd + n, make_float2(a.x + bb.x, a.y + bb.y), two, vv);
            });
            break;
        case EPI_ACCUM:
            run([&](long m, int n, float2 a, float2 bb, float2 o, bool two, bool vv) {
                put2(D + m * ep.ldd + n, make_float2((o.x + a.x) + bb.x, (o.y + a.y) + bb.y), two, vv);
            });
            break;
        case EPI_GELU:
            run([&](long m, int n, float2 a, float2 bb, float2, bool two, bool vv) {
                a = make_float2(a.x + bb.x, a.y + bb.y);
                if (D) put2(D + m * ep.ldd + n, a, two, vv);
                put2(ep.D2 + m * ep.ldd2 + n, make_float2(gelu_tanh(a.x, fa), gelu_tanh(a.y, fa)), two, vv);
            });
            break;
        case EPI_RESID:
            run([&](long m, int n, float2 a, float2 bb, float2 r, bool two, bool vv) {
                a = make_float2(a.x + bb.x, a.y + bb.y);
                if (D) put2(D + m * ep.ldd + n, a, two, vv);
                put2(ep.D2 + m * ep.ldd2 + n, make_float2(r.x + a.x, r.y + a.y), two, vv);
            });
            break;
        case EPI_GELU_BWD:
            run([&](long m, int n, float2 a, float2, float2 g, bool two, bool vv) {
                put2(D + m * ep.ldd + n,
                     make_float2(a.x * gelu_tanh_grad(g.x, fa), a.y * gelu_tanh_grad(g.y, fa)), two, vv);
            });
            break;
    }
}

template <int BN, bool A_MN, bool B_MN, bool SPLIT>
__global__ void __launch_bounds__(Cfg<BN, SPLIT>::THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           int M, int N, int K, int tiles_m, int tiles_n, int ksplit, int kb_per,
           long split_stride, GemmEpi epi) {
    using C = Cfg<BN, SPLIT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    SmemCtl *ctl = (SmemCtl *)(base + C::STAGES * C::STAGE_BYTES);
    auto sA = [&](int s) { return base + s * C::STAGE_BYTES; };
    auto sB = [&](int s) { return base + s * C::STAGE_BYTES + C::A_BYTES; };
    auto sAlo = [&](int s) { return base + s * C::STAGE_BYTES + C::A_BYTES + C::B_BYTES; };
    auto sBlo = [&](int s) { return base + s * C::STAGE_BYTES + 2 * C::A_BYTES + C::B_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // work unit = (output tile, K split); split s covers k-blocks
    // [s * kb_per, min(kblocks, (s + 1) * kb_per)), never empty (host-checked)
    const int mn_tiles = tiles_m * tiles_n;
    const int num_tiles = mn_tiles * ksplit;
    const int kblocks = (K + BK - 1) / BK;
    auto krange = [&](int tile, int &kb0, int &kb1) {
    kb0 = (tile / mn_tiles) * kb_per;
    kb1 = min(kblocks, kb0 + kb_per);
    };
    volatile int *abort = &ctl->abort;

    if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
        mbar_init(&ctl->full[s], 1);
        mbar_init(&ctl->empty[s], 1);
        mbar_init(&ctl->ready[s], 4);
    }
    for (int b = 0; b < 2; ++b) {
        mbar_init(&ctl->tfull[b], 1);
        mbar_init(&ctl->tempty[b], C::EPI_WARPS);
    }
    ctl->abort = 0;
    fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
    tmem_alloc(&ctl->tmem_base, C::TMEM_COLS);
    tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_base;

    if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
        int stage = 0;
        uint32_t phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            const int tm = (tile % mn_tiles) % tiles_m, tn = (tile % mn_tiles) / tiles_m;
            int kb0, kb1;
            krange(tile, kb0, kb1);
            for (int kb = kb0; kb < kb1; ++kb) {
                if (!mbar_wait(&ctl->empty[stage], phase ^ 1u, DEV_ERR_GEMM_PRODUCER, abort))
                    goto done;
                mbar_arrive_expect_tx(&ctl->full[stage], C::A_BYTES + C::B_BYTES);
                if (A_MN) {
#pragma unroll
                    for (int j = 0; j < BM / 32; ++j)
                        tma_load_2d(sA(stage) + j * (BK * 128), &tmA, &ctl->full[stage],
                                    tm * BM + j * 32, kb * BK);
                } else {
                    tma_load_2d(sA(stage), &tmA, &ctl->full[stage], kb * BK, tm * BM);
                }
                if (B_MN) {
#pragma unroll
                    for (int j = 0; j < BN / 32; ++j)
                        tma_load_2d(sB(stage) + j * (BK * 128), &tmB, &ctl->full[stage],
                                    tn * BN + j * 32, kb * BK);
                } else {
                    tma_load_2d(sB(stage), &tmB, &ctl->full[stage], kb * BK, tn * BN);
                }
                if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
            }
        }
    }
    } else if (warp == 1) {
    // ------------------------------------------------- MMA issuer
    if (lane == 0) {
        constexpr uint32_t idesc = idesc_tf32(BM, BN, A_MN, B_MN);
        // K-major (128B swizzle): rows of 128B, 8-row atoms 1024B apart; a
        // k-step of 8 elements advances the start address by 32B in the atom.
        // MN-major (128B swizzle, 32B atoms): 32-element MN atoms 4096B apart
        // (one TMA box of BK rows each), 4-row K groups 512B apart; a k-step
        // of 8 rows advances by 1024B.
        auto descA = [&](uint8_t *p, int kk) -> uint64_t {
            return A_MN ? smem_desc(smem_u32(p) + kk * 1024, BK * 128, 512, 1)
                        : smem_desc(smem_u32(p) + kk * 32, 16, 1024, 2);
        };
        auto descB = [&](uint8_t *p, int kk) -> uint64_t {
            return B_MN ? smem_desc(smem_u32(p) + kk * 1024, BK * 128, 512, 1)
                        : smem_desc(smem_u32(p) + kk * 32, 16, 1024, 2);
        };
        int stage = 0, acc = 0;
        uint32_t phase = 0, acc_phase = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
            int kb0, kb1;
            krange(tile, kb0, kb1);
            if constexpr (SPLIT) {
                // one fresh TMEM accumulator per k-block: the epilogue adds
                // the k-block partials in fp32 (round to nearest), which
                // bounds the tensor core's truncating accumulation to 12
                // steps per partial
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&ctl->tempty[acc], acc_phase ^ 1u, DEV_ERR_GEMM_MMA, abort))
                        goto done;
                    if (!mbar_wait(&ctl->ready[stage], phase, DEV_ERR_GEMM_MMA, abort)) goto done;
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
#pragma unroll
                    for (int kk = 0; kk < BK / MMA_K; ++kk) {
                        const uint64_t a = descA(sA(stage), kk), b = descB(sB(stage), kk);
                        mma_tf32(d_tmem, descA(sAlo(stage), kk), b, idesc, kk != 0);
                        mma_tf32(d_tmem, a, descB(sBlo(stage), kk), idesc, 1);
                        mma_tf32(d_tmem, a, b, idesc, 1);
                    }
                    mma_commit(&ctl->empty[stage]);
                    mma_commit(&ctl->tfull[acc]);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                    if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
                }
            } else {
                if (!mbar_wait(&ctl->tempty[acc], acc_phase ^ 1u, DEV_ERR_GEMM_MMA, abort))
                    goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&ctl->full[stage], phase, DEV_ERR_GEMM_MMA, abort)) goto done;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < BK / MMA_K; ++kk)
                        mma_tf32(d_tmem, descA(sA(stage), kk), descB(sB(stage), kk), idesc,
                                 (kb != kb0 || kk != 0));
                    mma_commit(&ctl->empty[stage]);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
                mma_commit(&ctl->tfull[acc]);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
        }
    }
    } else if (warp < 2 + C::EPI_WARPS) {
    // --------------------------------------------------- epilogue
    // Warp w owns TMEM lanes [32q, 32q+32), q = w % 4, and half of the
    // tile's columns. A 32x32 block is read with one tcgen05.ld (thread =
    // row), transposed through padded shared memory, and written back by
    // rows so every global access of the warp is coalesced; the block's
    // second operand rows (residual / GELU input / accumulator) are all
    // loaded before use so 32 loads are in flight per thread.
    const int q = warp & 3, half = (warp - 2) >> 2;
    constexpr int CH = BN / 64;  // 32-column chunks per warp
    float *stile = (float *)(base + C::STAGES * C::STAGE_BYTES + 256) + (warp - 2) * (32 * 33);
    int acc = 0;
    uint32_t acc_phase = 0;
    GemmEpi ep = epi;  // ep.D moves to the split's partial-sum slice
    long ldaux = 0;
    const float *aux = epi_aux(epi, ldaux);
    auto store_block_ = [&](const float (&v)[32], int m0, int n0) {
        store_block(ep, stile, lane, v, m0, n0, M, N, aux, ldaux);
    };
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int tm = (tile % mn_tiles) % tiles_m, tn = (tile % mn_tiles) / tiles_m;
        int kb0, kb1;
        krange(tile, kb0, kb1);
        ep.D = epi.D + (tile / mn_tiles) * split_stride;
        const int m0 = tm * BM + q * 32;
        const int c0 = half * CH;
        if constexpr (SPLIT) {
            float sum[CH * 32];
#pragma unroll
            for (int j = 0; j < CH * 32; ++j) sum[j] = 0.0f;
            bool ok = true;
            for (int kb = kb0; kb < kb1 && ok; ++kb) {
                if (!mbar_wait(&ctl->tfull[acc], acc_phase, DEV_ERR_GEMM_EPILOGUE, abort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < CH; ++c) {
                    float v[32];
                    tmem_ld_32x32b_x32(tmem_base + (uint32_t)(acc * BN + (c0 + c) * 32) +
                                           ((uint32_t)(q * 32) << 16), v);
#pragma unroll
                    for (int j = 0; j < 32; ++j) sum[c * 32 + j] += v[j];
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ctl->tempty[acc]);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
            if (!ok) break;
            float cm = -INFINITY, cs = 0.f;
#pragma unroll
            for (int c = 0; c < CH; ++c) {
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = sum[c * 32 + j];
                const int n0 = tn * BN + (c0 + c) * 32;
                if (ep.ce_part) ce_fold(v, n0, N, ep.alpha, cm, cs, ep.fast_act != 0);
                store_block_(v, m0, n0);
                if (ep.ce_part) ce_flush(ep, c, m0 + lane, n0, M, N, cm, cs);
            }
        } else {
            if (!mbar_wait(&ctl->tfull[acc], acc_phase, DEV_ERR_GEMM_EPILOGUE, abort)) break;
            tc_fence_after();
            float cm = -INFINITY, cs = 0.f;
#pragma unroll 1
            for (int c = 0; c < CH; ++c) {
                float v[32];
                tmem_ld_32x32b_x32(tmem_base + (uint32_t)(acc * BN + (c0 + c) * 32) +
                                       ((uint32_t)(q * 32) << 16), v);
                const int n0 = tn * BN + (c0 + c) * 32;
                if (ep.ce_part) ce_fold(v, n0, N, ep.alpha, cm, cs, ep.fast_act != 0);
                store_block_(v, m0, n0);
                if (ep.ce_part) ce_flush(ep, c, m0 + lane, n0, M, N, cm, cs);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->tempty[acc]);
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
    }
    } else if (SPLIT) {
    // ---------------------------------------- 3xTF32 split transform
    const int t = threadIdx.x - (2 + C::EPI_WARPS) * 32;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        int kb0, kb1;
        krange(tile, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
            if (!mbar_wait(&ctl->full[stage], phase, DEV_ERR_GEMM_TRANSFORM, abort)) goto done;
            float4 *hi = (float4 *)sA(stage);
            float4 *lo = (float4 *)sAlo(stage);
            constexpr int n4 = (C::A_BYTES + C::B_BYTES) / 16;
            for (int i = t; i < n4; i += 128) {
                float4 x = hi[i], h, l;
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(*(uint32_t *)&h.x) : "f"(x.x));
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(*(uint32_t *)&h.y) : "f"(x.y));
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(*(uint32_t *)&h.z) : "f"(x.z));
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(*(uint32_t *)&h.w) : "f"(x.w));
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(*(uint32_t *)&l.x) : "f"(x.x - h.x));
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(*(uint32_t *)&l.y) : "f"(x.y - h.y));
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(*(uint32_t *)&l.z) : "f"(x.z - h.z));
                asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(*(uint32_t *)&l.w) : "f"(x.w - h.w));
                hi[i] = h;
                lo[i] = l;
            }
            // generic-proxy smem writes -> visible to the tensor core (async proxy)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->ready[stage]);
            if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
        }
    }
    }
done:
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// ------------------------------------------- CTA-pair (cta_group::2) GEMM
// The same persistent warp-specialised GEMM over a 2-CTA cluster: the pair
// owns a 256 x BN output tile, each CTA loads its own 128 rows of A and half
// of the BN rows of B into its shared memory, and the leader CTA (rank 0)
// issues tcgen05.mma.cta_group::2 with M = 256, which reads both CTAs' halves
// and leaves rows [128r, 128r + 128) of the accumulator in CTA r's TMEM. Per
// CTA that halves the B bytes per FLOP, so a k-block stage is 24-32 KB
// instead of 48 KB and 6-8 stages fit. Every load is a plain per-CTA load; both
// CTAs' TMA completions count on the leader's `full` barrier, the MMA commits
// arrive on `empty` / `tfull` in both CTAs, and the epilogue warps of both
// CTAs release an accumulator on the leader's `tempty`. TF32 mode only.
// BN: 256, 192 or 128 output columns per pair tile (192 fills whole waves
// on the N = 768 products of GPT-2 small: 128 tiles instead of 96 on 74
// pairs). ROWT selects the epilogue flavour. false: BN / 16 epilogue warps
// (at BN = 256 four per TMEM lane quarter, two 32-column chunks each) reading the
// accumulator in the 16x256b layout and storing 8-byte pairs from registers
// (store_frag) - enough warps to hide the global stores and the GELU /
// GELU-backward arithmetic behind the next tile's main loop. true: 8 warps
// reading the 32x32b layout (thread = row), transposing each 32 x 32 block
// through a padded shared tile and writing whole 128-byte row segments
// (store_block), with the cross-entropy statistics folded in - measured
// faster on the forward GEMMs whose output is far larger than L2 (the LM
// head: 8192 x 50257 x 768, 1.46 ms against 1.79 ms).
template <int BN, bool ROWT = false>
struct Cfg2 {
    static constexpr int BNH = BN / 2;  // B rows per CTA
    static constexpr int A_BYTES = BM * KB_BYTES;
    static constexpr int B_BYTES = BNH * KB_BYTES;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int STAGES = BN == 256 ? 6 : 8;
    static constexpr int EPI_WARPS = ROWT ? 8 : BN / 16;  // two 32-column chunks per warp and tile
    static constexpr int CHUNKS = BN / 32 / (EPI_WARPS / 4);  // per warp and tile
    static constexpr int THREADS = (2 + EPI_WARPS) * 32;
    static constexpr int TMEM_COLS = BN == 192 ? 512 : 2 * BN;  // two accumulators, a power of two
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256 + (ROWT ? EPI_WARPS * 32 * 33 * 4 : 0);
    static_assert(CHUNKS % 2 == 0, "the cross-entropy groups need chunk pairs");
};

template <int BN, bool A_MN, bool B_MN, bool ROWT, int MODE = -1>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Cfg2<BN, ROWT>::THREADS, 1)
gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                int M, int N, int K, int tiles_m, int tiles_n, int ksplit, int kb_per, long split_stride,
                GemmEpi epi) {
    using C = Cfg2<BN, ROWT>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    SmemCtl *ctl = (SmemCtl *)(base + C::STAGES * C::STAGE_BYTES);
    auto sA = [&](int s) { return base + s * C::STAGE_BYTES; };
    auto sB = [&](int s) { return base + s * C::STAGE_BYTES + C::A_BYTES; };

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int mn_tiles = tiles_m * tiles_n;
    const int num_tiles = mn_tiles * ksplit;
    const int kblocks = (K + BK - 1) / BK;
    auto krange = [&](int tile, int &kb0, int &kb1) {
        kb0 = (tile / mn_tiles) * kb_per;
        kb1 = min(kblocks, kb0 + kb_per);
    };
    volatile int *abort = &ctl->abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&ctl->full[s], 1);
            mbar_init(&ctl->empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&ctl->tfull[b], 1);
            mbar_init(&ctl->tempty[b], 2 * C::EPI_WARPS);
        }
        ctl->abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        tmem_alloc_pair(&ctl->tmem_base, C::TMEM_COLS);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();  // both CTAs' barriers exist before any remote arrive
    tc_fence_after();
    const uint32_t tmem_base = ctl->tmem_base;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer (both CTAs)
        if (lane == 0) {
            const uint32_t full_leader = mapa_shared(smem_u32(&ctl->full[0]), 0);
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = pair; tile < num_tiles; tile += npairs) {
                const int tm = (tile % mn_tiles) % tiles_m, tn = (tile % mn_tiles) / tiles_m;
                const int row0 = tm * 2 * BM + (int)rank * BM, col0 = tn * BN + (int)rank * C::BNH;
                int kb0, kb1;
                krange(tile, kb0, kb1);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&ctl->empty[stage], phase ^ 1u, DEV_ERR_GEMM_PRODUCER, abort))
                        goto done;
                    if (rank == 0) mbar_arrive_expect_tx(&ctl->full[stage], 2 * C::STAGE_BYTES);
                    const uint32_t bar = full_leader + stage * 8;
                    if (A_MN) {
#pragma unroll
                        for (int j = 0; j < BM / 32; ++j)
                            tma_load_2d_pair(sA(stage) + j * (BK * 128), &tmA, bar, row0 + j * 32, kb * BK);
                    } else {
                        tma_load_2d_pair(sA(stage), &tmA, bar, kb * BK, row0);
                    }
                    if (B_MN) {
#pragma unroll
                        for (int j = 0; j < C::BNH / 32; ++j)
                            tma_load_2d_pair(sB(stage) + j * (BK * 128), &tmB, bar, col0 + j * 32, kb * BK);
                    } else {
                        tma_load_2d_pair(sB(stage), &tmB, bar, kb * BK, col0);
                    }
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
            }
        }
    } else if (warp == 1) {
        // --------------------------------------------- MMA issuer (leader CTA)
        if (lane == 0 && rank == 0) {
            constexpr uint32_t idesc = idesc_tf32(2 * BM, BN, A_MN, B_MN);
            auto descA = [&](uint8_t *p, int kk) -> uint64_t {
                return A_MN ? smem_desc(smem_u32(p) + kk * 1024, BK * 128, 512, 1)
                            : smem_desc(smem_u32(p) + kk * 32, 16, 1024, 2);
            };
            auto descB = [&](uint8_t *p, int kk) -> uint64_t {
                return B_MN ? smem_desc(smem_u32(p) + kk * 1024, BK * 128, 512, 1)
                            : smem_desc(smem_u32(p) + kk * 32, 16, 1024, 2);
            };
            int stage = 0, acc = 0;
            uint32_t phase = 0, acc_phase = 0;
            for (int tile = pair; tile < num_tiles; tile += npairs) {
                int kb0, kb1;
                krange(tile, kb0, kb1);
                if (!mbar_wait(&ctl->tempty[acc], acc_phase ^ 1u, DEV_ERR_GEMM_MMA, abort)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(&ctl->full[stage], phase, DEV_ERR_GEMM_MMA, abort)) goto done;
                    tc_fence_after();
#pragma unroll
                    for (int kk = 0; kk < BK / MMA_K; ++kk)
                        mma_tf32_pair(d_tmem, descA(sA(stage), kk), descB(sB(stage), kk), idesc,
                                      (kb != kb0 || kk != 0));
                    mma_commit_pair(&ctl->empty[stage]);
                    if (++stage == C::STAGES) { stage = 0; phase ^= 1u; }
                }
                mma_commit_pair(&ctl->tfull[acc]);
                if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
            }
        }
    } else {
        // ------------------------------------------------- epilogue (both CTAs)
        // warp w reads TMEM lane quarter w % 4 and the column slice (w - 2) / 4
        const int q = warp & 3, slice = (warp - 2) >> 2;
        constexpr int CH = C::CHUNKS;
        const uint32_t tempty_leader = mapa_shared(smem_u32(&ctl->tempty[0]), 0);
        long ldaux = 0;
        const float *aux = epi_aux(epi, ldaux);
        float *stile = (float *)(base + C::STAGES * C::STAGE_BYTES + 256) + (warp - 2) * (32 * 33);
        int acc = 0;
        uint32_t acc_phase = 0;
        for (int tile = pair; tile < num_tiles; tile += npairs) {
            const int tm = (tile % mn_tiles) % tiles_m, tn = (tile % mn_tiles) / tiles_m;
            float *const D = epi.D ? epi.D + (tile / mn_tiles) * split_stride : nullptr;
            const int m0 = tm * 2 * BM + (int)rank * BM + q * 32;
            if (!mbar_wait(&ctl->tfull[acc], acc_phase, DEV_ERR_GEMM_EPILOGUE, abort)) break;
            tc_fence_after();
            float cm = -INFINITY, cs = 0.f;
#pragma unroll 1
            for (int c = 0; c < CH; ++c) {
                const int col = (slice * CH + c) * 32;
                const int n0 = tn * BN + col;
                const uint32_t ta = tmem_base + (uint32_t)(acc * BN + col) + ((uint32_t)(q * 32) << 16);
                auto release = [&] {  // the accumulator is read: the MMA warp may reuse it
                    if (c == CH - 1) {
                        tc_fence_before();
                        __syncwarp();
                        // relaxed: the TMEM reads are complete (tcgen05.wait::ld)
                        // and the signal orders no memory writes, so it need not
                        // wait for this warp's stores of the first chunk
                        if (lane == 0) mbar_arrive_cluster_relaxed(tempty_leader + acc * 8);
                    }
                };
                if constexpr (ROWT) {
                    float v[32];
                    tmem_ld_32x32b_x32(ta, v);
                    release();
                    GemmEpi ep = epi;
                    ep.D = D;
                    if (epi.ce_part) ce_fold(v, n0, N, epi.alpha, cm, cs, epi.fast_act != 0);
                    store_block(ep, stile, lane, v, m0, n0, M, N, aux, ldaux);
                    if (epi.ce_part) ce_flush(epi, c, m0 + lane, n0, M, N, cm, cs);
                } else {
                    uint32_t r[32];
                    tmem_ld_16x256b_x4_nowait(ta, r);
                    tmem_ld_16x256b_x4_nowait(ta + (16u << 16), r + 16);
                    tmem_ld_wait32(r);
                    release();
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
                    store_frag<MODE>(epi, D, v, lane, m0, n0, M, N, aux, ldaux);
                }
            }
            if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
        }
    }
done:
    __syncwarp();
    tc_fence_before();
    cluster_sync_all();  // no CTA leaves while its pair may still signal or read it
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
    }
}

// ------------------------------------------------ CUDA-core fp32 fallback
// 64x64 output tile per 256-thread block, 4x4 outputs per thread, fp32 FMA.
__global__ void __launch_bounds__(256)
gemm_simt_kernel(const float *__restrict__ A, long lda, int a_mn, const float *__restrict__ B,
                 long ldb, int b_mn, int M, int N, int K, GemmEpi epi) {
    __shared__ float As[16][64 + 4];
    __shared__ float Bs[16][64 + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int i = threadIdx.x; i < 16 * 64; i += 256) {
            int kk = i / 64, r = i % 64;
            int m = m0 + r, n = n0 + r, k = k0 + kk;
            float a = 0.f, b = 0.f;
            if (m < M && k < K) a = a_mn ? A[(long)k * lda + m] : A[(long)m * lda + k];
            if (n < N && k < K) b = b_mn ? B[(long)k * ldb + n] : B[(long)n * ldb + k];
            As[kk][r] = a;
            Bs[kk][r] = b;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + ty * 4 + i;
        if (m >= M) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int n = n0 + tx * 4 + j;
            if (n < N) {
                long ld = 0;
                const float *ax = epi_aux(epi, ld);
                epi_apply(epi, m, n, acc[i][j], epi.bias ? epi.bias[n] : 0.0f, ax ? ax[(long)m * ld + n] : 0.0f);
            }
        }
    }
}

// ------------------------------------------------- skinny GEMM (GEMV) path
// out[m, n] = sum_k X[m, k] W[n, k] for M <= 8 rows (batch-1..8 decode and
// the LM head of the last positions): HBM-bound on W, which is streamed once
// with evict-first loads. A block of 256 threads owns GV_R rows of W and its
// threads split K in float4 units, so every block keeps R 16-byte loads per
// thread in flight whatever the shape. The R*MT partial sums of a thread are
// reduced across the warp by recursive halving (lane L ends with one total),
// then across the 8 warps through shared memory in warp order (fixed order,
// deterministic).
//
// Launched with programmatic dependent launch: the first two K-steps of W are
// loaded (and the rest prefetched into L2) before griddepcontrol.wait, so the
// weight stream overlaps the tail of the kernel that produces X.
constexpr int GV_R = 4, GV_THREADS = 256;

__device__ __forceinline__ float dot4(const float4 a, const float4 b) {
    return a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
}

template <int N>
__device__ __forceinline__ void halve_step(float *acc, int lane, int o, int &idx) {
    constexpr int h = N / 2;
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
        const float send = up ? acc[i] : acc[i + h];
        const float keep = up ? acc[i + h] : acc[i];
        acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
    if (up) idx += h;
}

// LayerNorm statistics of M <= MT rows of X ([M, 4*K4], row pitch ldx):
// the mean, then the biased variance about it (two passes, as
// src/ops.c:231-247), each block-reduced over the 256 threads in fixed
// order; eps 1e-5. CG reads bypass L1 (rows written by other blocks).
template <int MT, bool CG>
__device__ __forceinline__ void block_row_stats(const float *X, long ldx, int M, int K4, float (&mu)[MT],
                                                float (&rs)[MT], float (*lnred)[MT], float (*lnstat)[MT]) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
        float ps[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) ps[m] = 0.f;
        for (int k = t; k < K4; k += GV_THREADS) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m < M) {
                    const float4 *p = (const float4 *)(X + (long)m * ldx) + k;
                    const float4 xv = CG ? __ldcg(p) : __ldg(p);
                    if (pass == 0) {
                        ps[m] += (xv.x + xv.y) + (xv.z + xv.w);
                    } else {
                        const float a = xv.x - mu[m], b = xv.y - mu[m], c = xv.z - mu[m], d = xv.w - mu[m];
                        ps[m] += (a * a + b * b) + (c * c + d * d);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const float v = warp_sum(ps[m]);
            if (lane == 0) lnred[warp][m] = v;
        }
        __syncthreads();
        if (t < MT) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < GV_THREADS / 32; ++w) v += lnred[w][t];
            lnstat[pass][t] = v / (float)(4 * K4);
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (pass == 0) mu[m] = lnstat[0][m];
            else rs[m] = 1.0f / sqrtf(lnstat[1][m] + 1e-5f);
        }
    }
}

template <int MT, bool LNF>
__global__ void __launch_bounds__(GV_THREADS)
gemv_kernel(const float *__restrict__ X, long ldx, const float *__restrict__ W, long ldw, int M, int N,
            int K, GemmEpi epi, const float *__restrict__ lnw, const float *__restrict__ lnb,
            const float *__restrict__ ln_stats) {
    constexpr int R = GV_R, NV = R * MT;
    __shared__ float red[GV_THREADS / 32][NV];
    __shared__ float lnred[GV_THREADS / 32][MT], lnstat[2][MT];
    pdl_trigger();
    const int n0 = blockIdx.x * R, K4 = K >> 2, t = threadIdx.x;
    const int lane = t & 31, warp = t >> 5;
    const float4 *w4[R];
#pragma unroll
    for (int r = 0; r < R; ++r) w4[r] = (const float4 *)(W + (long)min(n0 + r, N - 1) * ldw);
    // before the producer of X has finished: W of the first two K-steps into
    // registers, the rest of this thread's W into L2
    float4 wp[2][R];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int r = 0; r < R; ++r)
            wp[i][r] = (t + i * GV_THREADS < K4) ? __ldcs(w4[r] + t + i * GV_THREADS)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int k = t + 2 * GV_THREADS; k < K4; k += 2 * GV_THREADS)
#pragma unroll
        for (int r = 0; r < R; ++r) asm volatile("prefetch.global.L2 [%0];" ::"l"(w4[r] + k));
    pdl_wait();
    float mu[MT], rs[MT];
    if constexpr (LNF) {
        if (ln_stats) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                mu[m] = m < M ? ln_stats[2 * m] : 0.f;
                rs[m] = m < M ? ln_stats[2 * m + 1] : 0.f;
            }
        } else {
            block_row_stats<MT, false>(X, ldx, M, K4, mu, rs, lnred, lnstat);
        }
    }
    auto xload = [&](int m, int k) -> float4 {
        float4 xv = __ldg((const float4 *)(X + (long)m * ldx) + k);
        if constexpr (LNF) {
            const float4 g = __ldg((const float4 *)lnw + k), bb = __ldg((const float4 *)lnb + k);
            xv.x = (xv.x - mu[m]) * rs[m] * g.x + bb.x;
            xv.y = (xv.y - mu[m]) * rs[m] * g.y + bb.y;
            xv.z = (xv.z - mu[m]) * rs[m] * g.z + bb.z;
            xv.w = (xv.w - mu[m]) * rs[m] * g.w + bb.w;
        }
        return xv;
    };
    float acc[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) acc[i] = 0.f;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int k = t + i * GV_THREADS;
        if (k < K4) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m < M) {
                    const float4 xv = xload(m, k);
#pragma unroll
                    for (int r = 0; r < R; ++r) acc[r * MT + m] += dot4(wp[i][r], xv);
                }
            }
        }
    }
#pragma unroll 2
    for (int k = t + 2 * GV_THREADS; k < K4; k += GV_THREADS) {
        float4 wv[R];
#pragma unroll
        for (int r = 0; r < R; ++r) wv[r] = __ldcs(w4[r] + k);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m < M) {
                const float4 xv = xload(m, k);
#pragma unroll
                for (int r = 0; r < R; ++r) acc[r * MT + m] += dot4(wv[r], xv);
            }
        }
    }
    // recursive halving: at offset o a lane keeps the upper half of its
    // values if (lane & o), the lower half otherwise, and adds the partner's
    int idx = 0, o = 16;
    if constexpr (NV >= 32) { halve_step<32>(acc, lane, o, idx); o >>= 1; }
    if constexpr (NV >= 16) { halve_step<16>(acc, lane, o, idx); o >>= 1; }
    if constexpr (NV >= 8) { halve_step<8>(acc, lane, o, idx); o >>= 1; }
    if constexpr (NV >= 4) { halve_step<4>(acc, lane, o, idx); o >>= 1; }
    if constexpr (NV >= 2) { halve_step<2>(acc, lane, o, idx); o >>= 1; }
    for (; o > 0; o >>= 1) acc[0] += __shfl_xor_sync(0xffffffffu, acc[0], o);
    if ((lane & (32 / NV - 1)) == 0) red[warp][idx] = acc[0];
    __syncthreads();
    unsigned long long amkey = 0;  // greedy key of this thread's (m, n), 0 = none
    if (t < NV) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < GV_THREADS / 32; ++w) v += red[w][t];
        const int r = t / MT, m = t % MT, n = n0 + r;
        if (epi.argmax_key && m < M && n < N) {
            const uint32_t u = __float_as_uint(v * epi.alpha + (epi.bias ? epi.bias[n] : 0.0f));
            const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
            amkey = ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n);
        }
        if (m < M && n < N) {
            long ld = 0;
            const float *ax = epi_aux(epi, ld);
            const float bias = epi.bias ? epi.bias[n] : 0.0f;
            if (epi.push_bufs) {
                // tensor-parallel partial: to every rank's receive slot
                const float a = v * epi.alpha + bias;
                const float val = epi.mode == EPI_RESID ? (ax ? ax[(long)m * ld + n] : 0.0f) + a : a;
                const unsigned long long ep =
                    (unsigned long long)(*epi.push_step) * epi.push_nk + epi.push_k + 1;
                for (int r = 0; r < epi.push_world; ++r)
                    tp_slot(epi.push_bufs[r], epi.push_world, epi.push_ld, (int)(ep & 1), epi.push_rank)
                        [(long)m * epi.push_ld + n] = val;
            } else {
                epi_apply(epi, m, n, v, bias, ax ? ax[(long)m * ld + n] : 0.0f);
            }
            if (epi.kc && n >= epi.kv_C) {  // STORE mode: the K / V value just stored
                const float val = v * epi.alpha + bias;
                const long at = (long)m * epi.kv_ld + (long)(*epi.kv_pos) * epi.kv_C;
                if (n < 2 * epi.kv_C) epi.kc[at + (n - epi.kv_C)] = val;
                else epi.vc[at + (n - 2 * epi.kv_C)] = val;
            }
        }
    }
    if (epi.argmax_key) {
        // rows m of this block's NV values sit in lanes t = r * MT + m of warp
        // 0; a block only issues the atomic when it beats the current key
        if (warp == 0) {
#pragma unroll
            for (int o = MT; o < 32; o <<= 1) {
                const unsigned long long other = __shfl_xor_sync(0xffffffffu, amkey, o);
                amkey = other > amkey ? other : amkey;
            }
            if (t < MT && t < M && amkey > *(volatile unsigned long long *)(epi.argmax_key + t))
                atomicMax(epi.argmax_key + t, amkey);
        }
    }
    if (epi.ln_stats_out) {
        // the last block to finish (integer ticket, writes fenced first)
        // computes the LayerNorm statistics of the completed D2 rows for the
        // consumer of this residual stream; the ticket is left at zero
        __shared__ int last;
        __threadfence();
        __syncthreads();
        if (t == 0) last = atomicAdd(epi.ln_ticket, 1) == (int)gridDim.x - 1;
        __syncthreads();
        if (last) {
            __threadfence();
            float smu[MT], srs[MT];
            block_row_stats<MT, true>(epi.D2, epi.ldd2, M, N >> 2, smu, srs, lnred, lnstat);
            if (t < MT && t < M) {
                epi.ln_stats_out[2 * t] = lnstat[0][t];
                epi.ln_stats_out[2 * t + 1] = 1.0f / sqrtf(lnstat[1][t] + 1e-5f);
            }
            if (t == 0) *epi.ln_ticket = 0;
        }
    }
    if (epi.push_bufs) {
        // every block's pushes are fenced at system scope before its ticket;
        // the last block then publishes the epoch on every rank's flag
        // (the CTA barrier makes the block's pushes visible to thread 0, whose
        // system-scope fence is cumulative over them)
        __shared__ int plast;
        __syncthreads();
        if (t == 0) {
            __threadfence_system();
            plast = atomicAdd(epi.push_ticket, 1) == (int)gridDim.x - 1;
        }
        __syncthreads();
        if (plast && t < epi.push_world) {
            __threadfence_system();
            const unsigned long long ep = (unsigned long long)(*epi.push_step) * epi.push_nk + epi.push_k + 1;
            unsigned long long *flag = (unsigned long long *)epi.push_bufs[t] + epi.push_rank;
            asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(ep) : "memory");
            if (t == 0) *epi.push_ticket = 0;
        }
    }
}

template <int MT, bool LNF>
int launch_gemv(const float *A, long lda, const float *B, long ldb, int M, int N, int K, const GemmEpi &epi,
                const float *lnw, const float *lnb, const float *lns, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((N + GV_R - 1) / GV_R);
    cfg.blockDim = dim3(GV_THREADS);
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    CG_CUDA(cudaLaunchKernelEx(&cfg, gemv_kernel<MT, LNF>, A, lda, B, ldb, M, N, K, epi, lnw, lnb, lns));
    ++g_launch_count;
    return OK;
}

template <bool LNF>
int dispatch_gemv(const float *A, long lda, const float *B, long ldb, int M, int N, int K, const GemmEpi &epi,
                  const float *lnw, const float *lnb, const float *lns, cudaStream_t s) {
    if (M <= 1) return launch_gemv<1, LNF>(A, lda, B, ldb, M, N, K, epi, lnw, lnb, lns, s);
    if (M <= 2) return launch_gemv<2, LNF>(A, lda, B, ldb, M, N, K, epi, lnw, lnb, lns, s);
    if (M <= 4) return launch_gemv<4, LNF>(A, lda, B, ldb, M, N, K, epi, lnw, lnb, lns, s);
    return launch_gemv<8, LNF>(A, lda, B, ldb, M, N, K, epi, lnw, lnb, lns, s);
}

// LayerNorm statistics (mean, rstd) of M rows, one block per row: the
// stand-alone form of the GEMV's last-block statistics
__global__ void __launch_bounds__(GV_THREADS) ln_stats_kernel(const float *__restrict__ X, long ldx, int K,
                                                              float *__restrict__ out) {
    __shared__ float lnred[GV_THREADS / 32][1], lnstat[2][1];
    float mu[1], rs[1];
    block_row_stats<1, true>(X + (long)blockIdx.x * ldx, ldx, 1, K >> 2, mu, rs, lnred, lnstat);
    if (threadIdx.x == 0) {
        out[2 * blockIdx.x] = mu[0];
        out[2 * blockIdx.x + 1] = rs[0];
    }
}

bool gemv_ok(const float *A, long lda, bool a_mn, const float *B, long ldb, bool b_mn, int M, int N, int K,
             const GemmEpi &epi) {
    auto al = [](const void *p) { return ((uintptr_t)p % 16) == 0; };
    return M <= 8 && !a_mn && !b_mn && K % 4 == 0 && lda % 4 == 0 && ldb % 4 == 0 && al(A) && al(B) &&
           (!epi.kc || epi.mode == EPI_STORE) &&
           (!epi.ln_stats_out || (epi.mode == EPI_RESID && N % 4 == 0 && epi.ldd2 % 4 == 0 && al(epi.D2))) &&
           (!epi.push_bufs || ((epi.mode == EPI_RESID || epi.mode == EPI_STORE) && !epi.ln_stats_out && !epi.kc)) &&
           (!epi.argmax_key || (epi.mode == EPI_STORE && !epi.push_bufs && !epi.kc));
}

// ------------------------------------------------------- tensor maps
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::mutex g_mu;

int get_encoder() {
    if (g_encode) return OK;
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) {
        set_last_error(ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
        return ERR_CUDA;
    }
    g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    return OK;
}

struct MapKey {
    const void *p;
    long inner, outer, ld;
    int box0, box1;
    bool operator==(const MapKey &o) const {
        return p == o.p && inner == o.inner && outer == o.outer && ld == o.ld && box0 == o.box0 &&
               box1 == o.box1;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        size_t h = std::hash<const void *>()(k.p);
        h ^= std::hash<long>()(k.inner * 1315423911L + k.outer * 2654435761L + k.ld) + 0x9e3779b9 +
             (h << 6) + (h >> 2);
        h ^= (size_t)k.box0 * 31 + (size_t)k.box1;
        return h;
    }
};
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

// 2-D fp32 tensor map: dim0 (contiguous) of extent `inner`, dim1 of extent
// `outer` with a pitch of `ld` elements; OOB reads fill zero. K-major
// operands use the 128B swizzle, MN-major ones the 128B swizzle with 32B
// atoms (the layout tcgen05 requires for MN-major tf32).
int make_map(CUtensorMap *out, const float *p, long inner, long outer, long ld, int box0,
             int box1, bool mn_major) {
    std::lock_guard<std::mutex> lk(g_mu);
    MapKey key{p, inner, outer, ld, box0, box1 | (mn_major ? 0x10000 : 0)};
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
        *out = it->second;
        return OK;
    }
    CG_TRY(get_encoder());
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    cuuint32_t box[2] = {(cuuint32_t)box0, (cuuint32_t)box1};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(out, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)p, dims, strides, box,
                          estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_last_error(ERR_ARG, "cuTensorMapEncodeTiled failed (%d) inner=%ld outer=%ld ld=%ld",
                       (int)r, inner, outer, ld);
        return ERR_ARG;
    }
    if (g_maps.size() > 8192) g_maps.clear();
    g_maps.emplace(key, *out);
    return OK;
}

// Split-K partial sums live in one fixed device buffer, allocated on first
// use outside stream capture and never moved, so a captured graph that
// replays a split GEMM keeps a valid pointer.
constexpr size_t SPLITK_WS_FLOATS = size_t(32) << 20;  // 128 MiB
float *g_splitk_ws = nullptr;
int g_splitk_dev = -1;

float *splitk_workspace(size_t floats, cudaStream_t s) {
    if (floats > SPLITK_WS_FLOATS) return nullptr;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_splitk_ws) return g_splitk_dev == dev ? g_splitk_ws : nullptr;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return nullptr;
    if (cudaMalloc(&g_splitk_ws, SPLITK_WS_FLOATS * sizeof(float)) != cudaSuccess) {
        cudaGetLastError();
        g_splitk_ws = nullptr;
        return nullptr;
    }
    g_splitk_dev = dev;
    return g_splitk_ws;
}


// out = epilogue(sum over splits of ws[s]) in split order (deterministic).
// Vector form: 4 consecutive columns per thread (N % 4 == 0, 16-byte aligned
// partials); the epilogue is applied per element.
__global__ void splitk_reduce_kernel(const float *__restrict__ ws, int S, long stride, int M, int N,
                                     GemmEpi epi) {
    long ld = 0;
    const float *aux = epi_aux(epi, ld);
    if ((N & 3) == 0) {
        const int N4 = N >> 2;
        const int total = M * N4;
        const float4 *w4 = (const float4 *)ws;
        const long s4 = stride >> 2;
        for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
            float4 a = w4[i];
            for (int k = 1; k < S; ++k) {
                const float4 b = w4[k * s4 + i];
                a.x += b.x;
                a.y += b.y;
                a.z += b.z;
                a.w += b.w;
            }
            const int m = i / N4, n = (i - m * N4) * 4;
            if (epi.vec4 && (epi.mode == EPI_ACCUM || epi.mode == EPI_STORE)) {
                // the weight-gradient products: 16-byte accesses of D
                const float4 b4 = epi.bias ? *(const float4 *)(epi.bias + n) : make_float4(0.f, 0.f, 0.f, 0.f);
                float4 *d = (float4 *)(epi.D + (long)m * epi.ldd + n);
                const float al = epi.alpha;
                if (epi.mode == EPI_ACCUM) {
                    const float4 o = *d;
                    *d = make_float4((o.x + a.x * al) + b4.x, (o.y + a.y * al) + b4.y, (o.z + a.z * al) + b4.z,
                                     (o.w + a.w * al) + b4.w);
                } else {
                    *d = make_float4(a.x * al + b4.x, a.y * al + b4.y, a.z * al + b4.z, a.w * al + b4.w);
                }
                continue;
            }
            const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
            for (int j = 0; j < 4; ++j)
                epi_apply(epi, m, n + j, av[j], epi.bias ? epi.bias[n + j] : 0.0f,
                          aux ? aux[(long)m * ld + n + j] : 0.0f);
        }
        return;
    }
    const long total = (long)M * N;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        float a = ws[i];
        for (int k = 1; k < S; ++k) a += ws[k * stride + i];
        const long m = i / N;
        const int n = (int)(i - m * N);
        epi_apply(epi, m, n, a, epi.bias ? epi.bias[n] : 0.0f, aux ? aux[m * ld + n] : 0.0f);
    }
}

// Cross-entropy statistics of stored rows, for the paths whose epilogue does
// not form them (split-K, CUDA-core, GEMV): one block per row, warp w takes
// the 64-column groups w, w + 8, ... (two columns per lane), same layout as
// the fused epilogue's.
__global__ void __launch_bounds__(256)
ce_stats_kernel(const float *__restrict__ D, long ldd, int N, float2 *__restrict__ part, int ce_ld) {
    const long m = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *row = D + m * ldd;
    for (int g = warp; g * 64 < N; g += 8) {
        const int n0 = g * 64 + lane, n1 = n0 + 32;
        const float a = n0 < N ? row[n0] : -INFINITY, b = n1 < N ? row[n1] : -INFINITY;
        float mx = warp_max(fmaxf(a, b));
        float sm = (n0 < N ? expf(a - mx) : 0.f) + (n1 < N ? expf(b - mx) : 0.f);
        sm = warp_sum(sm);
        if (lane == 0) part[m * ce_ld + g] = make_float2(mx, sm);
    }
}

int ce_stats_pass(const GemmEpi &e, int M, int N, cudaStream_t s) {
    ce_stats_kernel<<<M, 256, 0, s>>>(e.D, e.ldd, N, e.ce_part, e.ce_ld);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    return OK;
}

// Modelled time of a GEMM run as `units` persistent work units on `workers`
// (SMs, or CTA pairs): the slower of the tensor rate and the L2-to-SM operand
// stream (bytes per FLOP of the CTA tile: (rows + loaded B rows) x 128 B per
// 2 x rows x BN x 32 FLOP per k-block), both scaled by the last wave's fill,
// plus the split-K partial sums (written and read once each).
struct GemmModel {
    static constexpr double kTensor = 745e12;  // TF32 sustained, this kernel
    static constexpr double kL2 = 11.5e12;     // measured L2 -> SM operand stream
    static constexpr double kHbm = 6e12;
    static double time(double flops, double bpf, long units, long workers, int ks, long MN, bool split3) {
        const double waves = std::ceil((double)units / workers);
        const double eff = (double)units / (waves * workers);
        const double t_mma = flops * (split3 ? 3.0 : 1.0) / (kTensor * eff);
        const double t_l2 = flops * bpf / (kL2 * eff);
        return std::max(t_mma, t_l2) + (ks > 1 ? 2.0 * ks * MN * 4 / kHbm : 0.0);
    }
};

// Number of K splits for a GEMM with `tiles` output tiles of width bn (rows
// per CTA 128; pair kernels load bn / 2 B rows per CTA).
// CNGPT_CUDA_SPLITK=<n>: at most n K splits (1 disables split-K; default 8)
int max_ksplit() {
    static int mx = 0;
    if (mx == 0) {
        const char *e = getenv("CNGPT_CUDA_SPLITK");
        mx = e ? std::max(1, std::min(8, atoi(e))) : 8;
    }
    return mx;
}

int choose_ksplit(int tiles, int kblocks, int M, int N, long K, bool split3, int workers = 0, int bn = 128,
                  bool pair = false, double *t_out = nullptr) {
    const long w = workers > 0 ? workers : num_sms();
    const double flops = 2.0 * M * (double)N * K;
    const double bpf = (128.0 + (pair ? bn / 2 : bn)) * 128.0 / (2.0 * 128 * bn * 32);
    int best = 1;
    double bt = GemmModel::time(flops, bpf, tiles, w, 1, (long)M * N, split3);
    for (int k = 2; k <= max_ksplit() && kblocks / k >= 4; ++k) {
        const double t = GemmModel::time(flops, bpf, (long)tiles * k, w, k, (long)M * N, split3);
        if (t < 0.97 * bt) {
            bt = t;
            best = k;
        }
    }
    if (t_out) *t_out = bt;
    return best;
}

template <int BN, bool A_MN, bool B_MN, bool SPLIT>
int launch_tc(const float *A, long lda, const float *B, long ldb, int M, int N, int K,
              const GemmEpi &epi, cudaStream_t s) {
    using C = Cfg<BN, SPLIT>;
    static bool attr_set = false;
    auto kern = gemm_tc_kernel<BN, A_MN, B_MN, SPLIT>;
    if (!attr_set) {
        CG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr_set = true;
    }
    CUtensorMap ta, tb;
    if (A_MN) CG_TRY(make_map(&ta, A, M, K, lda, 32, BK, true));
    else      CG_TRY(make_map(&ta, A, K, M, lda, BK, BM, false));
    if (B_MN) CG_TRY(make_map(&tb, B, N, K, ldb, 32, BK, true));
    else      CG_TRY(make_map(&tb, B, K, N, ldb, BK, BN, false));
    const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
    const int tiles = tiles_m * tiles_n;
    const int kblocks = (K + BK - 1) / BK;
    int ks = choose_ksplit(tiles, kblocks, M, N, K, SPLIT, 0, BN, false);
    int kb_per = (kblocks + ks - 1) / ks;
    ks = (kblocks + kb_per - 1) / kb_per;  // every split non-empty
    float *ws = ks > 1 ? splitk_workspace((size_t)ks * M * N, s) : nullptr;
    if (!ws) {
        ks = 1;
        kb_per = kblocks;
    }
    const int grid = std::min(tiles * ks, num_sms());
    if (ks == 1) {
        kern<<<grid, C::THREADS, C::SMEM, s>>>(ta, tb, M, N, K, tiles_m, tiles_n, 1, kb_per, 0L, epi);
        ++g_launch_count;
        CG_CUDA(cudaGetLastError());
        return OK;
    }
    GemmEpi pe;
    pe.mode = EPI_STORE;
    pe.D = ws;
    pe.ldd = N;
    pe.vec4 = (N % 4) == 0;
    const long stride = (long)M * N;
    kern<<<grid, C::THREADS, C::SMEM, s>>>(ta, tb, M, N, K, tiles_m, tiles_n, ks, kb_per, stride, pe);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    const int rgrid = (int)std::min<long>((stride / 4 + 255) / 256, (long)num_sms() * 16);
    splitk_reduce_kernel<<<rgrid, 256, 0, s>>>(ws, ks, stride, M, N, epi);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    return epi.ce_part ? ce_stats_pass(epi, M, N, s) : OK;
}

bool pair_gemm_enabled() {
    static int on = -1;
    if (on < 0) {
        const char *e = getenv("CNGPT_CUDA_GEMM_PAIR");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

// CTA pairs that can be resident at once for the pair kernel (clusters of 2
// need both CTAs in one GPC; the count can be below num_sms / 2)
template <typename Kern>
int pair_slots(Kern kern, int threads, int smem) {
    static int cached = -1;
    if (cached > 0) return cached;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = num_sms() / 2;
    }
    cached = n;
    return n;
}

// The dynamic shared-memory limit of each kernel, raised once per kernel.
int smem_attr_once(const void *kern, int bytes) {
    static std::mutex mu;
    static std::unordered_map<const void *, int> done;
    std::lock_guard<std::mutex> g(mu);
    if (done.count(kern)) return OK;
    CG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    done[kern] = bytes;
    return OK;
}

// The pair kernel for one epilogue mode: instantiations specialised to the
// (orientation, mode) pairs of the training step - forward STORE / RESID /
// GELU, dX STORE / ACCUM / GELU_BWD, dW STORE / ACCUM - carry only their own
// epilogue code; every other pair runs the kernel that switches at run time.
template <int BN, bool A_MN, bool B_MN>
auto tc2_kernel_for(int mode) {
    auto k = gemm_tc2_kernel<BN, A_MN, B_MN, false, -1>;
    if constexpr (BN == 256 && !A_MN && !B_MN) {
        if (mode == EPI_STORE) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_STORE>;
        if (mode == EPI_RESID) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_RESID>;
        if (mode == EPI_GELU) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_GELU>;
    } else if constexpr (BN == 256 && !A_MN && B_MN) {
        if (mode == EPI_STORE) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_STORE>;
        if (mode == EPI_ACCUM) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_ACCUM>;
        if (mode == EPI_GELU_BWD) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_GELU_BWD>;
    } else if constexpr (BN == 256 && A_MN && B_MN) {
        if (mode == EPI_STORE) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_STORE>;
        if (mode == EPI_ACCUM) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_ACCUM>;
    } else if constexpr (BN == 192 && !A_MN && !B_MN) {  // the N = 768 products
        if (mode == EPI_STORE) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_STORE>;
        if (mode == EPI_RESID) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_RESID>;
    } else if constexpr (BN == 192 && !A_MN && B_MN) {
        if (mode == EPI_STORE) k = gemm_tc2_kernel<BN, A_MN, B_MN, false, EPI_STORE>;
    }
    return k;
}

template <int BN, bool A_MN, bool B_MN>
int launch_tc2(const float *A, long lda, const float *B, long ldb, int M, int N, int K, const GemmEpi &epi,
               cudaStream_t s) {
    using C = Cfg2<BN, false>;
    // the row-transposed epilogue (Cfg2<BN, true>) is instantiated for the
    // forward orientation at BN = 256 only: the LM head, whose statistics it
    // folds, and STORE GEMMs whose output is far larger than L2
    constexpr bool kRowT = !A_MN && !B_MN && BN == 256;
    using CR = Cfg2<BN, kRowT>;
    auto kern_rt = gemm_tc2_kernel<BN, A_MN, B_MN, kRowT>;
    CUtensorMap ta, tb;
    if (A_MN) CG_TRY(make_map(&ta, A, M, K, lda, 32, BK, true));
    else      CG_TRY(make_map(&ta, A, K, M, lda, BK, BM, false));
    if (B_MN) CG_TRY(make_map(&tb, B, N, K, ldb, 32, BK, true));
    else      CG_TRY(make_map(&tb, B, K, N, ldb, BK, C::BNH, false));
    const int tiles_m = (M + 2 * BM - 1) / (2 * BM), tiles_n = (N + BN - 1) / BN;
    const int tiles = tiles_m * tiles_n;
    const int kblocks = (K + BK - 1) / BK;
    auto kern_any = gemm_tc2_kernel<BN, A_MN, B_MN, false, -1>;
    CG_TRY(smem_attr_once((const void *)kern_any, C::SMEM));
    const int slots = pair_slots(kern_any, C::THREADS, C::SMEM);
    int ks = choose_ksplit(tiles, kblocks, M, N, K, false, slots, BN, true);
    int kb_per = (kblocks + ks - 1) / ks;
    ks = (kblocks + kb_per - 1) / kb_per;
    float *ws = ks > 1 ? splitk_workspace((size_t)ks * M * N, s) : nullptr;
    if (!ws) {
        ks = 1;
        kb_per = kblocks;
    }
    const int grid = 2 * std::min(tiles * ks, slots);
    if (ks == 1) {
        const bool huge = (long)M * N >= (64L << 20);  // 256 MB of output, twice L2
        const bool rowt = kRowT && (epi.ce_part || (epi.mode == EPI_STORE && huge));
        if (rowt) {
            // an output that large is not read again from L2: stores marked
            // evict-first keep the operand tiles resident instead
            GemmEpi e2 = epi;
            e2.stream_out = huge;
            CG_TRY(smem_attr_once((const void *)kern_rt, CR::SMEM));
            const int grid_rt = 2 * std::min(tiles, pair_slots(kern_rt, CR::THREADS, CR::SMEM));
            kern_rt<<<grid_rt, CR::THREADS, CR::SMEM, s>>>(ta, tb, M, N, K, tiles_m, tiles_n, 1, kb_per, 0L, e2);
        } else {
            auto kern = tc2_kernel_for<BN, A_MN, B_MN>(epi.mode);
            CG_TRY(smem_attr_once((const void *)kern, C::SMEM));
            kern<<<grid, C::THREADS, C::SMEM, s>>>(ta, tb, M, N, K, tiles_m, tiles_n, 1, kb_per, 0L, epi);
        }
        ++g_launch_count;
        CG_CUDA(cudaGetLastError());
        return epi.ce_part && !rowt ? ce_stats_pass(epi, M, N, s) : OK;
    }
    GemmEpi pe;
    pe.mode = EPI_STORE;
    pe.D = ws;
    pe.ldd = N;
    pe.vec4 = (N % 4) == 0;
    const long stride = (long)M * N;
    auto kern = tc2_kernel_for<BN, A_MN, B_MN>(EPI_STORE);
    CG_TRY(smem_attr_once((const void *)kern, C::SMEM));
    kern<<<grid, C::THREADS, C::SMEM, s>>>(ta, tb, M, N, K, tiles_m, tiles_n, ks, kb_per, stride, pe);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    const int rgrid = (int)std::min<long>((stride / 4 + 255) / 256, (long)num_sms() * 16);
    splitk_reduce_kernel<<<rgrid, 256, 0, s>>>(ws, ks, stride, M, N, epi);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    return epi.ce_part ? ce_stats_pass(epi, M, N, s) : OK;
}

// Tile width for the pair kernel: the modelled-fastest of 256, 192 (unless
// `no192`) and 128, each with its best K split. CNGPT_CUDA_PAIR_BN=256|192|128
// forces one.
int pair_tile_width(int M, int N, int K, bool no192) {
    static int forced = -1;
    if (forced < 0) {
        const char *e = getenv("CNGPT_CUDA_PAIR_BN");
        const int v = e ? atoi(e) : 0;
        forced = (v == 256 || v == 192 || v == 128) ? v : 0;
    }
    if (forced) return forced;
    const int pairs = num_sms() / 2, tm = (M + 2 * BM - 1) / (2 * BM), kblocks = (K + BK - 1) / BK;
    if (N <= 128) return 128;
    int best = 256;
    double tb = 0;
    choose_ksplit(tm * ((N + 255) / 256), kblocks, M, N, K, false, pairs, 256, true, &tb);
    for (int bn : {192, 128}) {
        if (bn == 192 && no192) continue;
        double t = 0;
        choose_ksplit(tm * ((N + bn - 1) / bn), kblocks, M, N, K, false, pairs, bn, true, &t);
        if (t < tb) {
            tb = t;
            best = bn;
        }
    }
    return best;
}

template <bool A_MN, bool B_MN>
int dispatch_tc(const float *A, long lda, const float *B, long ldb, int M, int N, int K,
                const GemmEpi &epi, cudaStream_t s, bool split) {
    if (split) return launch_tc<128, A_MN, B_MN, true>(A, lda, B, ldb, M, N, K, epi, s);
    if (pair_gemm_enabled() && M > BM) {
        // CTA pairs with 256 x 256, 256 x 192 or 256 x 128 tiles, whichever
        // the model below times fastest (tile width trades wave fill against
        // the L2-to-SM bytes per FLOP)
        // both operands MN-major (the dW products): 192-wide tiles measured
        // slower than 256 (2304 x 768 x 8192: 70.3 against 66.0 us)
        const int bn = pair_tile_width(M, N, K, A_MN && B_MN);
        if (bn == 256) return launch_tc2<256, A_MN, B_MN>(A, lda, B, ldb, M, N, K, epi, s);
        if (bn == 192) return launch_tc2<192, A_MN, B_MN>(A, lda, B, ldb, M, N, K, epi, s);
        return launch_tc2<128, A_MN, B_MN>(A, lda, B, ldb, M, N, K, epi, s);
    }
    // 128 x 256 tiles halve the A traffic per FLOP; take them unless their
    // last wave leaves the machine much emptier than 128 x 128 tiles would
    const long sms = num_sms(), tm = (M + BM - 1) / BM;
    const long t256 = tm * ((N + 255) / 256);
    auto eff = [&](long t) { return (double)t / (double)(((t + sms - 1) / sms) * sms); };
    if (N > 128 && t256 >= sms && eff(t256) >= 0.8)
        return launch_tc<256, A_MN, B_MN, false>(A, lda, B, ldb, M, N, K, epi, s);
    return launch_tc<128, A_MN, B_MN, false>(A, lda, B, ldb, M, N, K, epi, s);
}

bool tma_ok(const float *p, long ld) {
    return ((uintptr_t)p % 16) == 0 && (ld % 4) == 0 && ld > 0;
}

}  // namespace

int gemm_ln(const float *X, long ldx, const float *ln_w, const float *ln_b, const float *ln_stats,
            float *ln_out, const float *B, long ldb, int M, int N, int K, const GemmEpi &epi, cudaStream_t s) {
    auto al = [](const void *p) { return ((uintptr_t)p % 16) == 0; };
    if (M > 0 && N > 0 && gemv_ok(X, ldx, false, B, ldb, false, M, N, K, epi) && al(ln_w) && al(ln_b))
        return dispatch_gemv<true>(X, ldx, B, ldb, M, N, K, epi, ln_w, ln_b, ln_stats, s);
    CG_TRY(layernorm_fwd(X, ldx, ln_w, ln_b, ln_out, K, nullptr, nullptr, M, K, s));
    return gemm(ln_out, K, false, B, ldb, false, M, N, K, epi, s);
}

int gemm(const float *A, long lda, bool a_mn, const float *B, long ldb, bool b_mn, int M, int N,
         int K, const GemmEpi &epi, cudaStream_t s) {
    if (M < 0 || N < 0 || K < 0) {
        set_last_error(ERR_ARG, "gemm: negative shape M=%d N=%d K=%d", M, N, K);
        return ERR_ARG;
    }
    if (M == 0 || N == 0) return OK;
    if (epi.ce_part && (epi.mode != EPI_STORE || !epi.D || epi.bias || epi.ce_ld != (N + 63) / 64)) {
        set_last_error(ERR_ARG, "gemm: cross-entropy statistics need STORE without bias and ce_ld = ceil(N/64)");
        return ERR_ARG;
    }
    GemmEpi e2 = epi;
    {
        auto al = [](const void *p) { return ((uintptr_t)p % 16) == 0; };
        e2.vec4 = al(epi.D) && al(epi.D2) && al(epi.R) && al(epi.G) && al(epi.bias) &&
                  (!epi.D || epi.ldd % 4 == 0) && (!epi.D2 || epi.ldd2 % 4 == 0) &&
                  (!epi.R || epi.ldr % 4 == 0) && (!epi.G || epi.ldg % 4 == 0);
    }
    const int prec = precision();
    e2.fast_act = prec == PREC_TF32;
    if (epi.ce_part && (M <= 8 || prec == PREC_FP32)) {  // paths without the fused statistics
        GemmEpi e3 = epi;
        e3.ce_part = nullptr;
        CG_TRY(gemm(A, lda, a_mn, B, ldb, b_mn, M, N, K, e3, s));
        return ce_stats_pass(epi, M, N, s);
    }
    if (gemv_ok(A, lda, a_mn, B, ldb, b_mn, M, N, K, epi) &&
        ((long)N * K >= (1L << 16) || epi.kc || epi.ln_stats_out || epi.push_bufs || epi.argmax_key))
        return dispatch_gemv<false>(A, lda, B, ldb, M, N, K, epi, nullptr, nullptr, nullptr, s);
    if (epi.push_bufs) {
        set_last_error(ERR_ARG, "gemm: peer push needs the GEMV path (M <= 8, aligned K-major operands)");
        return ERR_ARG;
    }
    if (epi.argmax_key) {  // greedy step outside the GEMV path: the GEMM, then the row keys
        GemmEpi e3 = epi;
        e3.argmax_key = nullptr;
        CG_TRY(gemm(A, lda, a_mn, B, ldb, b_mn, M, N, K, e3, s));
        if (epi.mode != EPI_STORE) {
            set_last_error(ERR_ARG, "gemm: the fused argmax needs STORE mode");
            return ERR_ARG;
        }
        return argmax_keys(epi.D, epi.ldd, M, N, epi.argmax_key, s);
    }
    if (epi.ln_stats_out) {  // statistics requested outside the GEMV path: a separate pass
        GemmEpi e3 = epi;
        e3.ln_stats_out = nullptr;
        e3.ln_ticket = nullptr;
        CG_TRY(gemm(A, lda, a_mn, B, ldb, b_mn, M, N, K, e3, s));
        if (epi.mode != EPI_RESID || N % 4 != 0 || epi.ldd2 % 4 != 0 || ((uintptr_t)epi.D2 % 16) != 0) {
            set_last_error(ERR_ARG, "gemm: LayerNorm statistics need an aligned RESID output");
            return ERR_ARG;
        }
        ln_stats_kernel<<<M, GV_THREADS, 0, s>>>(epi.D2, epi.ldd2, N, epi.ln_stats_out);
        ++g_launch_count;
        CG_CUDA(cudaGetLastError());
        return OK;
    }
    if (epi.kc) {  // KV-cache columns: the GEMM, then the cache append
        GemmEpi e3 = epi;
        e3.kc = e3.vc = nullptr;
        CG_TRY(gemm(A, lda, a_mn, B, ldb, b_mn, M, N, K, e3, s));
        if (epi.mode != EPI_STORE || epi.ldd != 3L * epi.kv_C) {
            set_last_error(ERR_ARG, "gemm: KV-cache epilogue needs STORE into packed qkv rows");
            return ERR_ARG;
        }
        return kv_append_at(epi.D, epi.kc, epi.vc, M, epi.kv_ld / epi.kv_C, epi.kv_C, epi.kv_pos, s);
    }
    const bool big = (long)M * N * (long)std::max(K, 1) >= (1L << 18) && K > 0;
    const bool tc = prec != PREC_FP32 && big && tma_ok(A, lda) && tma_ok(B, ldb) &&
                    (a_mn ? lda >= M : lda >= K) && (b_mn ? ldb >= N : ldb >= K);
    if (tc) {
        const bool split = prec == PREC_3XTF32;
        if (!a_mn && !b_mn) return dispatch_tc<false, false>(A, lda, B, ldb, M, N, K, e2, s, split);
        if (!a_mn && b_mn) return dispatch_tc<false, true>(A, lda, B, ldb, M, N, K, e2, s, split);
        if (a_mn && b_mn) return dispatch_tc<true, true>(A, lda, B, ldb, M, N, K, e2, s, split);
        return dispatch_tc<true, false>(A, lda, B, ldb, M, N, K, e2, s, split);
    }
    dim3 grid((N + 63) / 64, (M + 63) / 64);
    gemm_simt_kernel<<<grid, 256, 0, s>>>(A, lda, a_mn, B, ldb, b_mn, M, N, K, epi);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    return epi.ce_part ? ce_stats_pass(epi, M, N, s) : OK;
}

int make_tensor_map(CUtensorMap_st *out, const float *p, long inner, long outer, long ld, int box0, int box1,
                    bool mn_major) {
    return make_map(out, p, inner, outer, ld, box0, box1, mn_major);
}

}  // namespace cg
