// attention_tc.cu - causal self-attention forward on the tcgen05 tensor cores
// (TF32 mode, head size 64), the forward of src/model.c:514-563 /
// src/fast.c:264-298 without the T x T matrices.
//
// One CTA per (query tile of 128 rows, sequence * head), heaviest tiles
// first. Warp roles:
//   warp 4  TMA producer: Q once, then K and V tiles of 128 keys into a
//           two-stage ring (K K-major, V MN-major: V^T is the B operand);
//   warp 5  MMA issuer (one thread): S = Q K^T into one of two TMEM score
//           buffers (128 x 128 fp32), and O_t = P V into one of two TMEM
//           output buffers (128 x 64);
//   warps 0-3  softmax, one thread per query row (TMEM lane = row): row max
//           over the scores (pass 1), then P = exp2(S - m) written to shared
//           memory in the 128B-swizzled K-major layout the MMA reads (pass 2),
//           and the running output O = O * alpha + O_t kept in registers.
// The next tile's S runs on the tensor cores while a tile's softmax runs on
// the CUDA cores, and each P V product overlaps the next tile's first pass.
// Every mbarrier wait is bounded (common.cuh); on expiry the CTA records a
// device error, frees its TMEM and returns.
#include <cuda.h>

#include <cmath>

#include "common.cuh"
#include "kernels.h"

namespace cg {
namespace {

constexpr int AQ = 128, AK = 128, AHS = 64;
constexpr int Q_BYTES = AQ * AHS * 4;  // two 128B-swizzled k-blocks of 32 dims
constexpr int K_BYTES = AK * AHS * 4;
constexpr int V_BYTES = AK * AHS * 4;  // 4 key blocks x 2 dim atoms (32 x 32 each)
constexpr int P_BYTES = AQ * AK * 4;   // 4 key blocks of 128 rows x 128 B
constexpr int SM_Q = 0, SM_K = SM_Q + Q_BYTES, SM_V = SM_K + 2 * K_BYTES, SM_P = SM_V + 2 * V_BYTES;
constexpr int SM_CTL = SM_P + P_BYTES;
constexpr int ATT_SMEM = SM_CTL + 256 + 1024;
constexpr int ATT_THREADS = 192;
constexpr int ATT_TMEM_COLS = 512;  // S[2] at columns 0 / 128, O[2] at 256 / 320
constexpr float LN2f = 0.6931471805599453f;

enum : int { DEV_ERR_ATT_TMA = 301, DEV_ERR_ATT_MMA = 302, DEV_ERR_ATT_SOFTMAX = 303 };

struct AttCtl {
    uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], p_full, o_full[2];
    uint32_t tmem_base;
    int abort;
};

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__global__ void __launch_bounds__(ATT_THREADS, 1)
attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQK, const __grid_constant__ CUtensorMap tmV,
                   float *__restrict__ out, float *__restrict__ lse, int T, int C, int H, float sl2) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    AttCtl *ctl = (AttCtl *)(base + SM_CTL);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqt = (T + AQ - 1) / AQ, BH = gridDim.x / nqt;
    const int qt = nqt - 1 - (int)(blockIdx.x / BH), bh = blockIdx.x % BH;
    const int b = bh / H, h = bh % H;
    const int q0 = qt * AQ, nkv = qt + 1;
    const int row_base = b * T;
    volatile int *abort = &ctl->abort;
    auto sK = [&](int s) { return base + SM_K + s * K_BYTES; };
    auto sV = [&](int s) { return base + SM_V + s * V_BYTES; };

    if (threadIdx.x == 0) {
        mbar_init(&ctl->q_full, 1);
        mbar_init(&ctl->p_full, 4);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&ctl->kv_full[s], 1);
            mbar_init(&ctl->kv_empty[s], 1);
            mbar_init(&ctl->s_full[s], 1);
            mbar_init(&ctl->o_full[s], 1);
        }
        ctl->abort = 0;
        fence_mbar_init();
    }
    if (warp == 5) {
        tmem_alloc(&ctl->tmem_base, ATT_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == 4) {
        // ------------------------------------------------------------ TMA
        if (lane == 0) {
            tma_prefetch_desc(&tmQK);
            tma_prefetch_desc(&tmV);
            mbar_arrive_expect_tx(&ctl->q_full, Q_BYTES);
            tma_load_2d(base + SM_Q, &tmQK, &ctl->q_full, h * AHS, row_base + q0);
            tma_load_2d(base + SM_Q + Q_BYTES / 2, &tmQK, &ctl->q_full, h * AHS + 32, row_base + q0);
            for (int j = 0; j < nkv; ++j) {
                const int st = j & 1;
                if (!mbar_wait(&ctl->kv_empty[st], ((j >> 1) & 1) ^ 1u, DEV_ERR_ATT_TMA, abort)) break;
                mbar_arrive_expect_tx(&ctl->kv_full[st], K_BYTES + V_BYTES);
                const int k0 = row_base + j * AK;
                tma_load_2d(sK(st), &tmQK, &ctl->kv_full[st], C + h * AHS, k0);
                tma_load_2d(sK(st) + K_BYTES / 2, &tmQK, &ctl->kv_full[st], C + h * AHS + 32, k0);
#pragma unroll
                for (int kb = 0; kb < 4; ++kb)
#pragma unroll
                    for (int d = 0; d < 2; ++d)
                        tma_load_2d(sV(st) + kb * 8192 + d * 4096, &tmV, &ctl->kv_full[st],
                                    2 * C + h * AHS + 32 * d, k0 + 32 * kb);
            }
        }
    } else if (warp == 5) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_tf32(AQ, AK, false, false);
            constexpr uint32_t idesc_o = idesc_tf32(AQ, AHS, false, true);
            const uint32_t q_addr = smem_u32(base + SM_Q), p_addr = smem_u32(base + SM_P);
            auto issue_s = [&](int j) {
                const uint32_t k_addr = smem_u32(sK(j & 1));
#pragma unroll
                for (int kb = 0; kb < 2; ++kb)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_tf32(tmem + (uint32_t)((j & 1) * AK),
                                 smem_desc(q_addr + kb * (Q_BYTES / 2) + kk * 32, 16, 1024, 2),
                                 smem_desc(k_addr + kb * (K_BYTES / 2) + kk * 32, 16, 1024, 2), idesc_s,
                                 (kb | kk) != 0);
                mma_commit(&ctl->s_full[j & 1]);
            };
            bool ok = mbar_wait(&ctl->q_full, 0, DEV_ERR_ATT_MMA, abort) &&
                      mbar_wait(&ctl->kv_full[0], 0, DEV_ERR_ATT_MMA, abort);
            if (ok) {
                tc_fence_after();
                issue_s(0);
            }
            for (int j = 0; ok && j < nkv; ++j) {
                if (j + 1 < nkv) {
                    if (!mbar_wait(&ctl->kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, DEV_ERR_ATT_MMA, abort)) break;
                    tc_fence_after();
                    issue_s(j + 1);
                }
                // P(j) written by the softmax warps (and O(j - 2) already folded)
                if (!mbar_wait(&ctl->p_full, j & 1, DEV_ERR_ATT_MMA, abort)) break;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sV(j & 1));
#pragma unroll
                for (int kb = 0; kb < 4; ++kb)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_tf32(tmem + (uint32_t)(2 * AK + (j & 1) * AHS),
                                 smem_desc(p_addr + kb * (P_BYTES / 4) + kk * 32, 16, 1024, 2),
                                 smem_desc(v_addr + kb * 8192 + kk * 1024, 4096, 512, 1), idesc_o,
                                 (kb | kk) != 0);
                mma_commit(&ctl->o_full[j & 1]);
                mma_commit(&ctl->kv_empty[j & 1]);
            }
        }
    } else {
        // --------------------------------------------- softmax, row = thread
        const int r = warp * 32 + lane, q = q0 + r;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        uint8_t *prow = base + SM_P + (r >> 3) * 1024 + (r & 7) * 128;
        float o[AHS];
#pragma unroll
        for (int d = 0; d < AHS; ++d) o[d] = 0.f;
        float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
        bool ok = true;
        auto fold = [&](int j) -> bool {  // O = O * alpha_prev + O_t(j)
            if (!mbar_wait(&ctl->o_full[j & 1], (j >> 1) & 1, DEV_ERR_ATT_SOFTMAX, abort)) return false;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float v[32];
                tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)(2 * AK + (j & 1) * AHS + c * 32), v);
#pragma unroll
                for (int i = 0; i < 32; ++i) o[c * 32 + i] = o[c * 32 + i] * alpha_prev + v[i];
            }
            return true;
        };
        for (int j = 0; j < nkv; ++j) {
            if (!mbar_wait(&ctl->s_full[j & 1], (j >> 1) & 1, DEV_ERR_ATT_SOFTMAX, abort)) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t sb = tmem + lane_off + (uint32_t)((j & 1) * AK);
            const bool diag = (j == qt);
            const int kbase = j * AK;
            float mx = -INFINITY;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                float v[32];
                tmem_ld_32x32b_x32(sb + c * 32, v);
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const bool masked = diag && (kbase + c * 32 + i > q);
                    mx = fmaxf(mx, masked ? -INFINITY : v[i] * sl2);
                }
            }
            const float m_new = fmaxf(m, mx);
            const float alpha = ex2f(m - m_new);
            // P(j) may only be written once P V of tile j - 1 has read P
            if (j > 0 && !fold(j - 1)) {
                ok = false;
                break;
            }
            float rs = 0.f;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
                float v[32];
                tmem_ld_32x32b_x32(sb + c * 32, v);
                uint8_t *pblk = prow + c * (P_BYTES / 4);
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    float p4[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int i = ch * 4 + e;
                        const bool masked = diag && (kbase + c * 32 + i > q);
                        p4[e] = masked ? 0.f : ex2f(v[i] * sl2 - m_new);
                        rs += p4[e];
                    }
                    *(float4 *)(pblk + ((ch ^ (r & 7)) << 4)) = make_float4(p4[0], p4[1], p4[2], p4[3]);
                }
            }
            l = l * alpha + rs;
            m = m_new;
            alpha_prev = alpha;
            // generic-proxy P writes -> visible to the tensor core
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->p_full);
        }
        if (ok && fold(nkv - 1) && q < T) {
            const float inv = 1.0f / l;
            float *orow = out + (long)(row_base + q) * C + h * AHS;
#pragma unroll
            for (int d = 0; d < AHS; d += 4)
                *(float4 *)(orow + d) = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
            if (lse) lse[(long)bh * T + q] = m * LN2f + logf(l);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        tc_fence_after();
        tmem_dealloc(tmem, ATT_TMEM_COLS);
    }
}

}  // namespace

CG_DEV_ERROR_READER(attn_tc_take_dev_error)

// TF32 causal attention forward on tcgen05; returns ERR_ARG (nothing
// launched) when the shapes or alignment do not fit, so the caller can take
// another kernel.
int attention_fwd_tc(const float *qkv, float *out, float *lse, int B, int T, int C, int H, cudaStream_t s) {
    if (C / H != AHS || C % H != 0 || ((uintptr_t)qkv % 16) != 0 || ((uintptr_t)out % 16) != 0 ||
        (3L * C) % 4 != 0 || C % 4 != 0)
        return ERR_ARG;
    CUtensorMap tqk, tv;
    CG_TRY(make_tensor_map(&tqk, qkv, 3L * C, (long)B * T, 3L * C, 32, AQ, false));
    CG_TRY(make_tensor_map(&tv, qkv, 3L * C, (long)B * T, 3L * C, 32, 32, true));
    static bool attr = false;
    if (!attr) {
        CG_CUDA(cudaFuncSetAttribute(attn_fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM));
        attr = true;
    }
    const int nqt = (T + AQ - 1) / AQ;
    const float sl2 = (1.0f / sqrtf((float)AHS)) * 1.4426950408889634f;
    attn_fwd_tc_kernel<<<nqt * B * H, ATT_THREADS, ATT_SMEM, s>>>(tqk, tv, out, lse, T, C, H, sl2);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    return OK;
}

}  // namespace cg
