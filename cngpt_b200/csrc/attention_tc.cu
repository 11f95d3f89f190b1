// attention_tc.cu - causal self-attention forward on the tcgen05 tensor cores
// (TF32 mode, head size 64), the forward of src/model.c:514-563 /
// src/fast.c:264-298 without the T x T matrices.
//
// One CTA per (query tile of 128 rows, sequence * head), heaviest tiles
// first. Warp roles:
//   warp 16  TMA producer: Q once, then K and V tiles of 128 keys into a
//            two-stage ring (K K-major, V MN-major: V^T is the B operand);
//   warp 17  MMA issuer (one thread): S = Q K^T into one of two TMEM score
//            buffers (128 x 128 fp32), and O_t = P V into one of two TMEM
//            output buffers (128 x 64);
//   warps 0-15  softmax: warp w reads TMEM lane quarter w % 4 (thread = query
//            row). Every thread takes the row max over all 128 scores of the
//            tile (TMEM reads are cheap; no exchange between warps), then
//            writes P = exp2(S - m) for its own 32 keys (columns
//            32 * (w / 4) .. +31) straight into the 128B-swizzled K-major
//            layout the MMA reads, and keeps 16 columns of the running output
//            O = O * alpha + O_t in registers; the four partial row sums of a
//            row are added in column order at the end.
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
constexpr int SOFT_WARPS = 16;                       // 4 per TMEM lane quarter, 32 key columns each
constexpr int TMA_WARP = SOFT_WARPS, MMA_WARP = SOFT_WARPS + 1;
constexpr int ATT_THREADS = (SOFT_WARPS + 2) * 32;
constexpr int ATT_TMEM_COLS = 512;  // S[2] at columns 0 / 128, O[2] at 256 / 320
constexpr float LN2f = 0.6931471805599453f;

enum : int { DEV_ERR_ATT_TMA = 301, DEV_ERR_ATT_MMA = 302, DEV_ERR_ATT_SOFTMAX = 303 };

struct AttCtl {
    // kv_full / kv_empty guard the K stages (released once S = Q K^T is done),
    // v_full / v_empty the V stages (released once P V is done); p_full[t]:
    // the softmax warps' P of tiles j with j % 2 == t (P kept in shared
    // memory uses p_full[0] for every tile)
    uint64_t q_full, kv_full[2], kv_empty[2], s_full[2], p_full[2], o_full[2], v_full[2], v_empty[2];
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(AttCtl) <= 256, "control block");

__device__ __forceinline__ float ex2f(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <bool TS>
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
        for (int s = 0; s < 2; ++s) {
            mbar_init(&ctl->p_full[s], SOFT_WARPS);
            mbar_init(&ctl->kv_full[s], 1);
            mbar_init(&ctl->kv_empty[s], 1);
            mbar_init(&ctl->s_full[s], 1);
            mbar_init(&ctl->o_full[s], 1);
            mbar_init(&ctl->v_full[s], 1);
            mbar_init(&ctl->v_empty[s], 1);
        }
        ctl->abort = 0;
        fence_mbar_init();
    }
    if (warp == MMA_WARP) {
        tmem_alloc(&ctl->tmem_base, ATT_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;

    if (warp == TMA_WARP) {
        // --------------------------------------------------------------- TMA
        // lane 0 loads Q and the K ring, lane 1 the V ring: K(j) is free once
        // S(j) is done, V(j) only once P V(j) is, so K runs ahead of V
        if (lane == 0) {
            tma_prefetch_desc(&tmQK);
            tma_prefetch_desc(&tmV);
            mbar_arrive_expect_tx(&ctl->q_full, Q_BYTES);
            tma_load_2d(base + SM_Q, &tmQK, &ctl->q_full, h * AHS, row_base + q0);
            tma_load_2d(base + SM_Q + Q_BYTES / 2, &tmQK, &ctl->q_full, h * AHS + 32, row_base + q0);
            for (int j = 0; j < nkv; ++j) {
                const int st = j & 1;
                if (!mbar_wait(&ctl->kv_empty[st], ((j >> 1) & 1) ^ 1u, DEV_ERR_ATT_TMA, abort)) break;
                mbar_arrive_expect_tx(&ctl->kv_full[st], K_BYTES);
                tma_load_2d(sK(st), &tmQK, &ctl->kv_full[st], C + h * AHS, row_base + j * AK);
                tma_load_2d(sK(st) + K_BYTES / 2, &tmQK, &ctl->kv_full[st], C + h * AHS + 32, row_base + j * AK);
            }
        } else if (lane == 1) {
            for (int j = 0; j < nkv; ++j) {
                const int st = j & 1;
                if (!mbar_wait(&ctl->v_empty[st], ((j >> 1) & 1) ^ 1u, DEV_ERR_ATT_TMA, abort)) break;
                mbar_arrive_expect_tx(&ctl->v_full[st], V_BYTES);
#pragma unroll
                for (int kb = 0; kb < 4; ++kb)
#pragma unroll
                    for (int d = 0; d < 2; ++d)
                        tma_load_2d(sV(st) + kb * 8192 + d * 4096, &tmV, &ctl->v_full[st],
                                    2 * C + h * AHS + 32 * d, row_base + j * AK + 32 * kb);
            }
        }
    } else if (warp == MMA_WARP) {
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
                mma_commit(&ctl->kv_empty[j & 1]);  // K(j) may be overwritten once S(j) is done
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
                    // TS: S(j + 1) overwrites P(j - 1), the A operand of P V(j - 1);
                    // MMAs into different accumulators are not ordered, so wait
                    // for that product to complete
                    if (TS && j >= 1 && !mbar_wait(&ctl->o_full[(j - 1) & 1], ((j - 1) >> 1) & 1, DEV_ERR_ATT_MMA, abort))
                        break;
                    tc_fence_after();
                    issue_s(j + 1);
                }
                // P(j) written by the softmax warps (and O(j - 2) already folded).
                // TS: the softmax warps do not wait for P V(j) before writing
                // P(j + 1), so the two tile parities arrive on separate barriers
                // (a warp cannot run two tiles ahead: P(j + 2) follows its fold
                // of O_t(j), which needs every warp's P(j))
                if (!mbar_wait(TS ? &ctl->p_full[j & 1] : &ctl->p_full[0], TS ? (j >> 1) & 1 : j & 1, DEV_ERR_ATT_MMA,
                               abort))
                    break;
                if (!mbar_wait(&ctl->v_full[j & 1], (j >> 1) & 1, DEV_ERR_ATT_MMA, abort)) break;
                tc_fence_after();
                const uint32_t v_addr = smem_u32(sV(j & 1));
#pragma unroll
                for (int kb = 0; kb < 4; ++kb)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t vd = smem_desc(v_addr + kb * 8192 + kk * 1024, 4096, 512, 1);
                        if constexpr (TS)  // P(j) in place of S(j): keys kb * 32 + kk * 8 .. + 7
                            mma_tf32_ts(tmem + (uint32_t)(2 * AK + (j & 1) * AHS),
                                        tmem + (uint32_t)((j & 1) * AK + kb * 32 + kk * 8), vd, idesc_o,
                                        (kb | kk) != 0);
                        else
                            mma_tf32(tmem + (uint32_t)(2 * AK + (j & 1) * AHS),
                                     smem_desc(p_addr + kb * (P_BYTES / 4) + kk * 32, 16, 1024, 2), vd, idesc_o,
                                     (kb | kk) != 0);
                    }
                mma_commit(&ctl->o_full[j & 1]);
                mma_commit(&ctl->v_empty[j & 1]);
            }
        }
    } else {
        // -------------------------- softmax: row = thread, 32 key columns per warp
        const int quarter = warp & 3, cs = warp >> 2;
        const int r = quarter * 32 + lane, q = q0 + r;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        float o[16];
#pragma unroll
        for (int d = 0; d < 16; ++d) o[d] = 0.f;
        float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
        bool ok = true;
        if constexpr (TS) {
            // P(j) overwrites S(j) in TMEM and is the A operand of P V(j), so
            // the exponentials of tile j + 1 overlap P V(j) on the tensor
            // cores. The row max is exchanged through shared memory (one
            // partial per column slice, double-buffered by tile parity); every
            // warp passes the same named barriers whatever happens, so a
            // timed-out wait cannot strand the rest of its lane quarter.
            float *pmax = (float *)(base + SM_P + 4 * AQ * sizeof(float));  // [2][4][AQ]
            auto fold = [&](int j) -> bool {  // O = O * alpha_prev + O_t(j), this warp's 16 columns
                if (!mbar_wait(&ctl->o_full[j & 1], (j >> 1) & 1, DEV_ERR_ATT_SOFTMAX, abort)) return false;
                tc_fence_after();
                float v[16];
                tmem_ld_32x32b_x16(tmem + lane_off + (uint32_t)(2 * AK + (j & 1) * AHS + cs * 16), v);
#pragma unroll
                for (int i = 0; i < 16; ++i) o[i] = o[i] * alpha_prev + v[i];
                return true;
            };
            for (int j = 0; j < nkv; ++j) {
                const int buf = j & 1;
                ok = ok && mbar_wait(&ctl->s_full[buf], (j >> 1) & 1, DEV_ERR_ATT_SOFTMAX, abort);
                ok = __all_sync(0xffffffffu, ok);
                const bool diag = (j == qt);
                const int kfirst = j * AK + cs * 32;
                const uint32_t s_addr = tmem + lane_off + (uint32_t)(buf * AK + cs * 32);
                float pm = -INFINITY;  // max of this slice's unscaled, unmasked scores
                if (ok) {
                    float v[32];
                    tc_fence_after();
                    tmem_ld_32x32b_x32(s_addr, v);
                    if (diag) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (kfirst + i <= q) pm = fmaxf(pm, v[i]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) pm = fmaxf(pm, v[i]);
                    }
                }
                float *pb = pmax + buf * 4 * AQ;
                pb[cs * AQ + r] = pm;
                asm volatile("bar.sync %0, 128;" ::"r"(1 + quarter) : "memory");
                if (!ok) continue;
                const float mraw = fmaxf(fmaxf(pb[r], pb[AQ + r]), fmaxf(pb[2 * AQ + r], pb[3 * AQ + r]));
                const float m_new = fmaxf(m, mraw * sl2);  // sl2 > 0: max commutes with the scale
                const float alpha = ex2f(m - m_new);
                // P over S in two halves of 16 columns, the scores read again
                // from TMEM (fewer live registers than holding all 32 across
                // the barrier); the row sum keeps column order
                float rs = 0.f;
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    float v[16];
                    tmem_ld_32x32b_x16(s_addr + (uint32_t)(hf * 16), v);
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float p = (diag && kfirst + hf * 16 + i > q) ? 0.f : ex2f(v[i] * sl2 - m_new);
                        v[i] = p;
                        rs += p;
                    }
                    tmem_st_32x32b_x16_nowait(s_addr + (uint32_t)(hf * 16), v);
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ctl->p_full[buf]);
                l = l * alpha + rs;
                m = m_new;
                if (j > 0) ok = __all_sync(0xffffffffu, fold(j - 1));
                alpha_prev = alpha;
            }
            ok = ok && fold(nkv - 1);
        } else {
            uint8_t *pblk = base + SM_P + cs * (P_BYTES / 4) + (r >> 3) * 1024 + (r & 7) * 128;
            auto fold = [&](int j) -> bool {  // O = O * alpha_prev + O_t(j), this warp's 16 columns
                if (!mbar_wait(&ctl->o_full[j & 1], (j >> 1) & 1, DEV_ERR_ATT_SOFTMAX, abort)) return false;
                tc_fence_after();
                float v[32];
                tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)(2 * AK + (j & 1) * AHS + (cs >> 1) * 32), v);
                if (cs & 1) {
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[i] = o[i] * alpha_prev + v[16 + i];
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) o[i] = o[i] * alpha_prev + v[i];
                }
                return true;
            };
            for (int j = 0; j < nkv; ++j) {
                if (!mbar_wait(&ctl->s_full[j & 1], (j >> 1) & 1, DEV_ERR_ATT_SOFTMAX, abort)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const bool diag = (j == qt);
                const int kb0 = j * AK;
                float own[32];
                float mraw = -INFINITY;  // max of the unscaled, unmasked scores
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float v[32];
                    tmem_ld_32x32b_x32(tmem + lane_off + (uint32_t)((j & 1) * AK + c * 32), v);
                    if (diag) {
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (kb0 + c * 32 + i <= q) mraw = fmaxf(mraw, v[i]);
                    } else {
#pragma unroll
                        for (int i = 0; i < 32; ++i) mraw = fmaxf(mraw, v[i]);
                    }
                    if (c == cs) {
#pragma unroll
                        for (int i = 0; i < 32; ++i) own[i] = v[i];
                    }
                }
                const float m_new = fmaxf(m, mraw * sl2);  // sl2 > 0: max commutes with the scale
                const float alpha = ex2f(m - m_new);
                // P(j) may only be written once P V of tile j - 1 has read P
                if (j > 0 && !fold(j - 1)) {
                    ok = false;
                    break;
                }
                const int kfirst = kb0 + cs * 32;
                float rs = 0.f;
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {
                    float p4[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int i = ch * 4 + e;
                        p4[e] = (diag && kfirst + i > q) ? 0.f : ex2f(own[i] * sl2 - m_new);
                        rs += p4[e];
                    }
                    *(float4 *)(pblk + ((ch ^ (r & 7)) << 4)) = make_float4(p4[0], p4[1], p4[2], p4[3]);
                }
                l = l * alpha + rs;
                m = m_new;
                alpha_prev = alpha;
                // generic-proxy P writes -> visible to the tensor core
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&ctl->p_full[0]);
            }
            ok = ok && fold(nkv - 1);
        }
        // row sums: the four column slices of each row, added in slice order,
        // exchanged through the P buffer (free once the last P V completed)
        float *lsum = (float *)(base + SM_P);
        lsum[cs * AQ + r] = l;
        asm volatile("bar.sync %0, 128;" ::"r"(1 + quarter) : "memory");
        if (ok && q < T) {
            const float lt = ((lsum[r] + lsum[AQ + r]) + lsum[2 * AQ + r]) + lsum[3 * AQ + r];
            const float inv = 1.0f / lt;
            float *orow = out + (long)(row_base + q) * C + h * AHS + cs * 16;
#pragma unroll
            for (int d = 0; d < 16; d += 4)
                *(float4 *)(orow + d) = make_float4(o[d] * inv, o[d + 1] * inv, o[d + 2] * inv, o[d + 3] * inv);
            if (lse && cs == 0) lse[(long)bh * T + q] = m * LN2f + logf(lt);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        tmem_dealloc(tmem, ATT_TMEM_COLS);
    }
}


// ================================================================ backward
// Both passes recompute P = exp2(S * scale * log2e - lse * log2e) from the
// saved row log-sum-exp, form dS = P (dP - D) with D = rowsum(dO * O), and
// accumulate in TMEM across their loop - no atomics, deterministic:
//   attn_bwd_dkdv_tc_kernel  one CTA per (128-key tile, sequence * head),
//     steps of 64 queries q >= first key: S^T = K Q^T and dP^T = V dO^T
//     (keys on the TMEM lanes), then dV += P^T dO and dK += dS^T Q with P^T /
//     dS^T written by the compute warps into shared memory (K-major) and Q,
//     dO read a second time in the MN-major layout as the B operands;
//   attn_bwd_dq_tc_kernel  one CTA per (128-query tile, sequence * head),
//     steps of 64 keys <= the tile's last query: S = Q K^T, dP = dO V^T, then
//     dQ += dS K (K read MN-major).
// 16 compute warps (thread = TMEM lane row, 16 of the 64 step columns per
// warp), one TMA warp, one MMA warp; every wait bounded.
constexpr int BQS = 64;                               // step width (queries or keys)
constexpr int BT_HALF = BQS * 64 * 4;                 // 16 KB: a 64-row x 64-dim operand
constexpr int BT_FULL = 128 * 64 * 4;                 // 32 KB: a 128-row operand
constexpr int BT_DS = 128 * BQS * 4;                  // 32 KB: P^T / dS^T or dS tile
// dK/dV: K, V resident; stages of {Q, dO} K-major + {Q, dO} MN-major
constexpr int KV_SM_K = 0, KV_SM_V = BT_FULL, KV_SM_STAGE = 2 * BT_FULL, KV_STAGE = 4 * BT_HALF;
constexpr int KV_SM_DS = KV_SM_STAGE + 2 * KV_STAGE, KV_SM_CTL = KV_SM_DS + BT_DS;
constexpr int KV_SMEM = KV_SM_CTL + 256 + 1024;
// dQ: Q, dO resident; stages of {K, V} K-major + K MN-major
constexpr int DQ_SM_Q = 0, DQ_SM_DO = BT_FULL, DQ_SM_STAGE = 2 * BT_FULL, DQ_STAGE = 3 * BT_HALF;
constexpr int DQ_SM_DS = DQ_SM_STAGE + 2 * DQ_STAGE, DQ_SM_CTL = DQ_SM_DS + BT_DS;
constexpr int DQ_SMEM = DQ_SM_CTL + 256 + 1024;
constexpr int BWD_WARPS = 16, BWD_TMA = 16, BWD_MMA = 17, BWD_THREADS = 18 * 32;
constexpr float LOG2Ef = 1.4426950408889634f;

struct BwdCtl {
    // st_*: ring of the K-major step operands (free once S / dP are done);
    // mn_*: ring of the MN-major step operands (free once the accumulating
    // MMAs that read them are done). With P^T / dS in TMEM the compute warps
    // arrive on a_full for even steps and b_full for odd ones.
    uint64_t in_full, st_full[2], st_empty[2], mn_full[2], mn_empty[2], sp_full[2], a_full, a_done, b_full,
        b_done, acc_done;
    uint32_t tmem_base;
    int abort;
};
static_assert(sizeof(BwdCtl) <= 256, "control block");

enum : int { DEV_ERR_ATTB_TMA = 311, DEV_ERR_ATTB_MMA = 312, DEV_ERR_ATTB_CMP = 313 };

__device__ __forceinline__ void bwd_init(BwdCtl *ctl) {
    mbar_init(&ctl->in_full, 1);
    for (int s = 0; s < 2; ++s) {
        mbar_init(&ctl->st_full[s], 1);
        mbar_init(&ctl->st_empty[s], 1);
        mbar_init(&ctl->mn_full[s], 1);
        mbar_init(&ctl->mn_empty[s], 1);
        mbar_init(&ctl->sp_full[s], 1);
    }
    mbar_init(&ctl->a_full, BWD_WARPS);
    mbar_init(&ctl->a_done, 1);
    mbar_init(&ctl->b_full, BWD_WARPS);
    mbar_init(&ctl->b_done, 1);
    mbar_init(&ctl->acc_done, 1);
    ctl->abort = 0;
    fence_mbar_init();
}

// 16 values of one row into the K-major 128B-swizzled tile (rows of 128 B =
// 32 floats; this writes floats [col0, col0 + 16) of row r, col0 % 16 == 0)
__device__ __forceinline__ void put_row16(uint8_t *tile, int r, int col0, const float (&v)[16]) {
    uint8_t *row = tile + (col0 >> 5) * (128 * 128) + (r >> 3) * 1024 + (r & 7) * 128;
    const int ch0 = (col0 & 31) >> 2;
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *(float4 *)(row + (((ch0 + c) ^ (r & 7)) << 4)) = make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

// D (+)= A B^T over K = 64 (two 32-wide k-blocks, four tf32 MMAs each)
// A: 128 rows K-major at a (k-block stride a_kb); B: K-major rows at b
// (k-block stride b_kb) or MN-major at b (k-block stride 8192, dim atoms 4096)
__device__ __forceinline__ void mma_k64(uint32_t d, uint32_t a, int a_kb, uint32_t b, int b_kb, bool b_mn,
                                        uint32_t idesc, bool acc) {
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint64_t da = smem_desc(a + kb * a_kb + kk * 32, 16, 1024, 2);
            const uint64_t db = b_mn ? smem_desc(b + kb * 8192 + kk * 1024, 4096, 512, 1)
                                     : smem_desc(b + kb * b_kb + kk * 32, 16, 1024, 2);
            mma_tf32(d, da, db, idesc, (acc || kb || kk) ? 1u : 0u);
        }
}

// D (+)= A B^T over K = 64 with A in TMEM (128 lanes, columns a .. a + 63,
// one fp32 element per column) and B MN-major at b (k-block stride 8192, dim
// atoms 4096)
__device__ __forceinline__ void mma_k64_ts(uint32_t d, uint32_t a, uint32_t b, uint32_t idesc, bool acc) {
#pragma unroll
    for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
            mma_tf32_ts(d, a + (uint32_t)(kb * 32 + kk * 8), smem_desc(b + kb * 8192 + kk * 1024, 4096, 512, 1),
                        idesc, (acc || kb || kk) ? 1u : 0u);
}

template <bool TS>
__global__ void __launch_bounds__(BWD_THREADS, 1)
attn_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmQK128, const __grid_constant__ CUtensorMap tmQK64,
                        const __grid_constant__ CUtensorMap tmMN, const __grid_constant__ CUtensorMap tmDO64,
                        const __grid_constant__ CUtensorMap tmDOMN, const float *__restrict__ lse,
                        const float *__restrict__ Dd, float *__restrict__ dqkv, int T, int C, int H, float sl2,
                        float scale) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    BwdCtl *ctl = (BwdCtl *)(base + KV_SM_CTL);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nkt = (T + 127) / 128, BH = gridDim.x / nkt;
    const int kt = (int)(blockIdx.x / BH), bh = blockIdx.x % BH;  // light tiles (late keys) last
    const int b = bh / H, h = bh % H, row_base = b * T, k0 = kt * 128;
    const int ns = (T - k0 + BQS - 1) / BQS;  // query steps q0 = k0 + 64 s
    volatile int *abort = &ctl->abort;
    auto stage = [&](int st) { return base + KV_SM_STAGE + st * KV_STAGE; };  // Qk, dOk, Qmn, dOmn
    if (threadIdx.x == 0) bwd_init(ctl);
    if (warp == BWD_MMA) {
        tmem_alloc(&ctl->tmem_base, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    // TMEM: S^T[2] at 0 / 64, dP^T[2] at 128 / 192, dV at 256, dK at 320
    if (warp == BWD_TMA) {
        if (lane == 0) {
            mbar_arrive_expect_tx(&ctl->in_full, 2 * BT_FULL);
            for (int kb = 0; kb < 2; ++kb) {
                tma_load_2d(base + KV_SM_K + kb * (BT_FULL / 2), &tmQK128, &ctl->in_full, C + h * 64 + 32 * kb,
                            row_base + k0);
                tma_load_2d(base + KV_SM_V + kb * (BT_FULL / 2), &tmQK128, &ctl->in_full, 2 * C + h * 64 + 32 * kb,
                            row_base + k0);
            }
            for (int s = 0; s < ns; ++s) {
                const int st = s & 1;
                if (!mbar_wait(&ctl->st_empty[st], ((s >> 1) & 1) ^ 1u, DEV_ERR_ATTB_TMA, abort)) break;
                mbar_arrive_expect_tx(&ctl->st_full[st], 2 * BT_HALF);
                const int q0 = row_base + k0 + s * BQS;
                uint8_t *sg = stage(st);
                for (int kb = 0; kb < 2; ++kb) {
                    tma_load_2d(sg + kb * (BT_HALF / 2), &tmQK64, &ctl->st_full[st], h * 64 + 32 * kb, q0);
                    tma_load_2d(sg + BT_HALF + kb * (BT_HALF / 2), &tmDO64, &ctl->st_full[st], h * 64 + 32 * kb, q0);
                }
            }
        } else if (lane == 1) {
            for (int s = 0; s < ns; ++s) {
                const int st = s & 1;
                if (!mbar_wait(&ctl->mn_empty[st], ((s >> 1) & 1) ^ 1u, DEV_ERR_ATTB_TMA, abort)) break;
                mbar_arrive_expect_tx(&ctl->mn_full[st], 2 * BT_HALF);
                const int q0 = row_base + k0 + s * BQS;
                uint8_t *sg = stage(st);
                for (int kb = 0; kb < 2; ++kb)
                    for (int d = 0; d < 2; ++d) {
                        tma_load_2d(sg + 2 * BT_HALF + kb * 8192 + d * 4096, &tmMN, &ctl->mn_full[st],
                                    h * 64 + 32 * d, q0 + 32 * kb);
                        tma_load_2d(sg + 3 * BT_HALF + kb * 8192 + d * 4096, &tmDOMN, &ctl->mn_full[st],
                                    h * 64 + 32 * d, q0 + 32 * kb);
                    }
            }
        }
    } else if (warp == BWD_MMA) {
        if (lane == 0) {
            constexpr uint32_t id_sp = idesc_tf32(128, BQS, false, false);
            constexpr uint32_t id_acc = idesc_tf32(128, 64, false, true);
            const uint32_t ka = smem_u32(base + KV_SM_K), va = smem_u32(base + KV_SM_V), dsa = smem_u32(base + KV_SM_DS);
            auto issue_sp = [&](int s) {
                const uint32_t sg = smem_u32(stage(s & 1));
                mma_k64(tmem + (s & 1) * 64, ka, BT_FULL / 2, sg, BT_HALF / 2, false, id_sp, false);
                mma_k64(tmem + 128 + (s & 1) * 64, va, BT_FULL / 2, sg + BT_HALF, BT_HALF / 2, false, id_sp, false);
                mma_commit(&ctl->sp_full[s & 1]);
                mma_commit(&ctl->st_empty[s & 1]);
            };
            bool ok = mbar_wait(&ctl->in_full, 0, DEV_ERR_ATTB_MMA, abort) &&
                      mbar_wait(&ctl->st_full[0], 0, DEV_ERR_ATTB_MMA, abort);
            if (ok) {
                tc_fence_after();
                issue_sp(0);
            }
            for (int s = 0; ok && s < ns; ++s) {
                if (s + 1 < ns) {
                    if (!mbar_wait(&ctl->st_full[(s + 1) & 1], ((s + 1) >> 1) & 1, DEV_ERR_ATTB_MMA, abort)) break;
                    // TS: step s + 1 overwrites the TMEM operands of step s - 1's
                    // accumulating MMAs (not ordered against them): wait for those
                    if (TS && s >= 1 &&
                        !mbar_wait(&ctl->mn_empty[(s - 1) & 1], ((s - 1) >> 1) & 1, DEV_ERR_ATTB_MMA, abort))
                        break;
                    tc_fence_after();
                    issue_sp(s + 1);
                }
                const uint32_t sg = smem_u32(stage(s & 1));
                if (TS ? !mbar_wait((s & 1) ? &ctl->b_full : &ctl->a_full, (s >> 1) & 1, DEV_ERR_ATTB_MMA, abort)
                       : !mbar_wait(&ctl->a_full, s & 1, DEV_ERR_ATTB_MMA, abort))
                    break;  // P^T (TS: and dS^T) written
                if (!mbar_wait(&ctl->mn_full[s & 1], (s >> 1) & 1, DEV_ERR_ATTB_MMA, abort)) break;
                tc_fence_after();
                if constexpr (TS) {  // P^T, dS^T in place of S^T, dP^T
                    mma_k64_ts(tmem + 256, tmem + (s & 1) * 64, sg + 3 * BT_HALF, id_acc, s > 0);        // dV += P^T dO
                    mma_k64_ts(tmem + 320, tmem + 128 + (s & 1) * 64, sg + 2 * BT_HALF, id_acc, s > 0);  // dK += dS^T Q
                    mma_commit(&ctl->mn_empty[s & 1]);
                    continue;
                }
                mma_k64(tmem + 256, dsa, BT_DS / 2, sg + 3 * BT_HALF, 0, true, id_acc, s > 0);  // dV += P^T dO
                mma_commit(&ctl->a_done);
                if (!mbar_wait(&ctl->b_full, s & 1, DEV_ERR_ATTB_MMA, abort)) break;  // dS^T written
                tc_fence_after();
                mma_k64(tmem + 320, dsa, BT_DS / 2, sg + 2 * BT_HALF, 0, true, id_acc, s > 0);  // dK += dS^T Q
                mma_commit(&ctl->b_done);
                mma_commit(&ctl->mn_empty[s & 1]);
            }
            mma_commit(&ctl->acc_done);
        }
    } else {
        const int quarter = warp & 3, cq = warp >> 2;
        const int r = quarter * 32 + lane, key = k0 + r;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        uint8_t *ds = base + KV_SM_DS;
        const float *lse_bh = lse + (long)bh * T, *D_bh = Dd + (long)bh * T;
        // lse and D of this warp's 16 queries of a step: one load per lane
        // (lanes 0-15 lse, 16-31 D), handed out by shuffles; the next step's
        // load is issued before this step's wait so its latency is hidden
        auto lse_d = [&](int s) {
            const int ql = k0 + s * BQS + cq * 16 + (lane & 15);
            return ql < T ? ((lane < 16) ? lse_bh[ql] : D_bh[ql]) : 0.f;
        };
        float raw_next = lse_d(0);
        bool ok = true;
        for (int s = 0; s < ns; ++s) {
            const float raw = raw_next;
            if (s + 1 < ns) raw_next = lse_d(s + 1);
            if (!mbar_wait(&ctl->sp_full[s & 1], (s >> 1) & 1, DEV_ERR_ATTB_CMP, abort)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[16], dp[16], pv[16], dsv[16];
            tmem_ld_32x32b_x16(tmem + lane_off + (uint32_t)((s & 1) * 64 + cq * 16), sv);
            tmem_ld_32x32b_x16(tmem + lane_off + (uint32_t)(128 + (s & 1) * 64 + cq * 16), dp);
            const int qf = k0 + s * BQS + cq * 16;
            const float ld_ = (lane < 16) ? raw * LOG2Ef : raw;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const int q = qf + c;
                const bool valid = key <= q && q < T;
                const float l2 = __shfl_sync(0xffffffffu, ld_, c), dd = __shfl_sync(0xffffffffu, ld_, 16 + c);
                pv[c] = valid ? ex2f(sv[c] * sl2 - l2) : 0.f;
                dsv[c] = pv[c] * (dp[c] - dd);
            }
            if constexpr (TS) {
                // in place: S^T(s), dP^T(s) are not read again, and step s + 2
                // overwrites them only after this step's dV / dK MMAs
                tmem_st_32x32b_x16_nowait(tmem + lane_off + (uint32_t)((s & 1) * 64 + cq * 16), pv);
                tmem_st_32x32b_x16_nowait(tmem + lane_off + (uint32_t)(128 + (s & 1) * 64 + cq * 16), dsv);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                // even / odd steps on separate barriers: nothing here waits for
                // this step's MMAs, but step s + 2 needs them complete
                if (lane == 0) mbar_arrive((s & 1) ? &ctl->b_full : &ctl->a_full);
                continue;
            }
            // the dS^T of the previous step must have been read (dK MMA done)
            if (s > 0 && !mbar_wait(&ctl->b_done, (s - 1) & 1, DEV_ERR_ATTB_CMP, abort)) {
                ok = false;
                break;
            }
            put_row16(ds, r, cq * 16, pv);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->a_full);
            if (!mbar_wait(&ctl->a_done, s & 1, DEV_ERR_ATTB_CMP, abort)) {  // dV MMA read P^T
                ok = false;
                break;
            }
            put_row16(ds, r, cq * 16, dsv);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->b_full);
        }
        if (ok && mbar_wait(&ctl->acc_done, 0, DEV_ERR_ATTB_CMP, abort)) {
            tc_fence_after();
            float dv[16], dk[16];
            tmem_ld_32x32b_x16(tmem + lane_off + (uint32_t)(256 + cq * 16), dv);
            tmem_ld_32x32b_x16(tmem + lane_off + (uint32_t)(320 + cq * 16), dk);
            if (key < T) {
                float *row = dqkv + (long)(row_base + key) * 3 * C + h * 64 + cq * 16;
#pragma unroll
                for (int c = 0; c < 16; c += 4) {
                    *(float4 *)(row + C + c) = make_float4(dk[c] * scale, dk[c + 1] * scale, dk[c + 2] * scale,
                                                           dk[c + 3] * scale);
                    *(float4 *)(row + 2 * C + c) = make_float4(dv[c], dv[c + 1], dv[c + 2], dv[c + 3]);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == BWD_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <bool TS>
__global__ void __launch_bounds__(BWD_THREADS, 1)
attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmQK128, const __grid_constant__ CUtensorMap tmQK64,
                      const __grid_constant__ CUtensorMap tmMN, const __grid_constant__ CUtensorMap tmDO128,
                      const float *__restrict__ lse, const float *__restrict__ Dd, float *__restrict__ dqkv, int T,
                      int C, int H, float sl2, float scale) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *base = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    BwdCtl *ctl = (BwdCtl *)(base + DQ_SM_CTL);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqt = (T + 127) / 128, BH = gridDim.x / nqt;
    const int qt = nqt - 1 - (int)(blockIdx.x / BH), bh = blockIdx.x % BH;  // heavy tiles first
    const int b = bh / H, h = bh % H, row_base = b * T, q0 = qt * 128;
    const int ns = (min(T, q0 + 128) + BQS - 1) / BQS;  // key steps k0 = 64 s
    volatile int *abort = &ctl->abort;
    auto stage = [&](int st) { return base + DQ_SM_STAGE + st * DQ_STAGE; };  // Kk, Vk, Kmn
    if (threadIdx.x == 0) bwd_init(ctl);
    if (warp == BWD_MMA) {
        tmem_alloc(&ctl->tmem_base, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = ctl->tmem_base;
    // TMEM: S[2] at 0 / 64, dP[2] at 128 / 192, dQ at 256
    if (warp == BWD_TMA) {
        if (lane == 0) {
            mbar_arrive_expect_tx(&ctl->in_full, 2 * BT_FULL);
            for (int kb = 0; kb < 2; ++kb) {
                tma_load_2d(base + DQ_SM_Q + kb * (BT_FULL / 2), &tmQK128, &ctl->in_full, h * 64 + 32 * kb,
                            row_base + q0);
                tma_load_2d(base + DQ_SM_DO + kb * (BT_FULL / 2), &tmDO128, &ctl->in_full, h * 64 + 32 * kb,
                            row_base + q0);
            }
            for (int s = 0; s < ns; ++s) {
                const int st = s & 1;
                if (!mbar_wait(&ctl->st_empty[st], ((s >> 1) & 1) ^ 1u, DEV_ERR_ATTB_TMA, abort)) break;
                mbar_arrive_expect_tx(&ctl->st_full[st], 2 * BT_HALF);
                const int k0 = row_base + s * BQS;
                uint8_t *sg = stage(st);
                for (int kb = 0; kb < 2; ++kb) {
                    tma_load_2d(sg + kb * (BT_HALF / 2), &tmQK64, &ctl->st_full[st], C + h * 64 + 32 * kb, k0);
                    tma_load_2d(sg + BT_HALF + kb * (BT_HALF / 2), &tmQK64, &ctl->st_full[st],
                                2 * C + h * 64 + 32 * kb, k0);
                }
            }
        } else if (lane == 1) {
            for (int s = 0; s < ns; ++s) {
                const int st = s & 1;
                if (!mbar_wait(&ctl->mn_empty[st], ((s >> 1) & 1) ^ 1u, DEV_ERR_ATTB_TMA, abort)) break;
                mbar_arrive_expect_tx(&ctl->mn_full[st], BT_HALF);
                const int k0 = row_base + s * BQS;
                uint8_t *sg = stage(st);
                for (int kb = 0; kb < 2; ++kb)
                    for (int d = 0; d < 2; ++d)
                        tma_load_2d(sg + 2 * BT_HALF + kb * 8192 + d * 4096, &tmMN, &ctl->mn_full[st],
                                    C + h * 64 + 32 * d, k0 + 32 * kb);
            }
        }
    } else if (warp == BWD_MMA) {
        if (lane == 0) {
            constexpr uint32_t id_sp = idesc_tf32(128, BQS, false, false);
            constexpr uint32_t id_acc = idesc_tf32(128, 64, false, true);
            const uint32_t qa = smem_u32(base + DQ_SM_Q), doa = smem_u32(base + DQ_SM_DO);
            const uint32_t dsa = smem_u32(base + DQ_SM_DS);
            auto issue_sp = [&](int s) {
                const uint32_t sg = smem_u32(stage(s & 1));
                mma_k64(tmem + (s & 1) * 64, qa, BT_FULL / 2, sg, BT_HALF / 2, false, id_sp, false);
                mma_k64(tmem + 128 + (s & 1) * 64, doa, BT_FULL / 2, sg + BT_HALF, BT_HALF / 2, false, id_sp, false);
                mma_commit(&ctl->sp_full[s & 1]);
                mma_commit(&ctl->st_empty[s & 1]);
            };
            bool ok = mbar_wait(&ctl->in_full, 0, DEV_ERR_ATTB_MMA, abort) &&
                      mbar_wait(&ctl->st_full[0], 0, DEV_ERR_ATTB_MMA, abort);
            if (ok) {
                tc_fence_after();
                issue_sp(0);
            }
            for (int s = 0; ok && s < ns; ++s) {
                if (s + 1 < ns) {
                    if (!mbar_wait(&ctl->st_full[(s + 1) & 1], ((s + 1) >> 1) & 1, DEV_ERR_ATTB_MMA, abort)) break;
                    // TS: step s + 1 overwrites the TMEM operands of step s - 1's
                    // accumulating MMAs (not ordered against them): wait for those
                    if (TS && s >= 1 &&
                        !mbar_wait(&ctl->mn_empty[(s - 1) & 1], ((s - 1) >> 1) & 1, DEV_ERR_ATTB_MMA, abort))
                        break;
                    tc_fence_after();
                    issue_sp(s + 1);
                }
                if (TS ? !mbar_wait((s & 1) ? &ctl->b_full : &ctl->a_full, (s >> 1) & 1, DEV_ERR_ATTB_MMA, abort)
                       : !mbar_wait(&ctl->a_full, s & 1, DEV_ERR_ATTB_MMA, abort))
                    break;  // dS written
                if (!mbar_wait(&ctl->mn_full[s & 1], (s >> 1) & 1, DEV_ERR_ATTB_MMA, abort)) break;
                tc_fence_after();
                if constexpr (TS)  // dS in place of dP
                    mma_k64_ts(tmem + 256, tmem + 128 + (s & 1) * 64, smem_u32(stage(s & 1)) + 2 * BT_HALF, id_acc,
                               s > 0);
                else
                    mma_k64(tmem + 256, dsa, BT_DS / 2, smem_u32(stage(s & 1)) + 2 * BT_HALF, 0, true, id_acc, s > 0);
                mma_commit(&ctl->a_done);
                mma_commit(&ctl->mn_empty[s & 1]);
            }
            mma_commit(&ctl->acc_done);
        }
    } else {
        const int quarter = warp & 3, cq = warp >> 2;
        const int r = quarter * 32 + lane, q = q0 + r;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        uint8_t *ds = base + DQ_SM_DS;
        const bool qv = q < T;
        const float l2 = qv ? lse[(long)bh * T + q] * LOG2Ef : 0.f, dd = qv ? Dd[(long)bh * T + q] : 0.f;
        bool ok = true;
        for (int s = 0; s < ns; ++s) {
            if (!mbar_wait(&ctl->sp_full[s & 1], (s >> 1) & 1, DEV_ERR_ATTB_CMP, abort)) {
                ok = false;
                break;
            }
            tc_fence_after();
            float sv[16], dp[16], dsv[16];
            tmem_ld_32x32b_x16(tmem + lane_off + (uint32_t)((s & 1) * 64 + cq * 16), sv);
            tmem_ld_32x32b_x16(tmem + lane_off + (uint32_t)(128 + (s & 1) * 64 + cq * 16), dp);
            const int kf = s * BQS + cq * 16;
#pragma unroll
            for (int c = 0; c < 16; ++c) {
                const bool valid = qv && kf + c <= q;
                const float p = valid ? ex2f(sv[c] * sl2 - l2) : 0.f;
                dsv[c] = p * (dp[c] - dd);
            }
            if constexpr (TS) {
                tmem_st_32x32b_x16_nowait(tmem + lane_off + (uint32_t)(128 + (s & 1) * 64 + cq * 16), dsv);
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                // even / odd steps on separate barriers: nothing here waits for
                // this step's MMAs, but step s + 2 needs them complete
                if (lane == 0) mbar_arrive((s & 1) ? &ctl->b_full : &ctl->a_full);
                continue;
            }
            if (s > 0 && !mbar_wait(&ctl->a_done, (s - 1) & 1, DEV_ERR_ATTB_CMP, abort)) {  // dQ MMA read dS
                ok = false;
                break;
            }
            put_row16(ds, r, cq * 16, dsv);
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&ctl->a_full);
        }
        if (ok && mbar_wait(&ctl->acc_done, 0, DEV_ERR_ATTB_CMP, abort)) {
            tc_fence_after();
            float dq[16];
            tmem_ld_32x32b_x16(tmem + lane_off + (uint32_t)(256 + cq * 16), dq);
            if (qv) {
                float *row = dqkv + (long)(row_base + q) * 3 * C + h * 64 + cq * 16;
#pragma unroll
                for (int c = 0; c < 16; c += 4)
                    *(float4 *)(row + c) = make_float4(dq[c] * scale, dq[c + 1] * scale, dq[c + 2] * scale,
                                                       dq[c + 3] * scale);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == BWD_MMA) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

}  // namespace

CG_DEV_ERROR_ACCESSORS(attn_tc_take_dev_error, attn_tc_set_wait_limit)

// TF32 causal attention forward on tcgen05; returns ERR_ARG (nothing
// launched) when the shapes or alignment do not fit, so the caller can take
// another kernel.
// The forward and backward kernels keep P (and dS) in tensor memory, in place
// of the scores they come from, and read them there as the A operand of the
// following MMA; CNGPT_CUDA_ATTN_P_TMEM=0 stages them in shared memory instead
// (the forward's output is bit-identical either way)
static bool fwd_p_in_tmem() {
    static int on = -1;
    if (on < 0) {
        const char *e = getenv("CNGPT_CUDA_ATTN_P_TMEM");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

int attention_fwd_tc(const float *qkv, float *out, float *lse, int B, int T, int C, int H, cudaStream_t s) {
    if (C / H != AHS || C % H != 0 || ((uintptr_t)qkv % 16) != 0 || ((uintptr_t)out % 16) != 0 ||
        (3L * C) % 4 != 0 || C % 4 != 0)
        return ERR_ARG;
    CUtensorMap tqk, tv;
    CG_TRY(make_tensor_map(&tqk, qkv, 3L * C, (long)B * T, 3L * C, 32, AQ, false));
    CG_TRY(make_tensor_map(&tv, qkv, 3L * C, (long)B * T, 3L * C, 32, 32, true));
    static bool attr = false;
    if (!attr) {
        CG_CUDA(cudaFuncSetAttribute(attn_fwd_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM));
        CG_CUDA(cudaFuncSetAttribute(attn_fwd_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM));
        attr = true;
    }
    const int nqt = (T + AQ - 1) / AQ;
    const float sl2 = (1.0f / sqrtf((float)AHS)) * 1.4426950408889634f;
    if (fwd_p_in_tmem())
        attn_fwd_tc_kernel<true><<<nqt * B * H, ATT_THREADS, ATT_SMEM, s>>>(tqk, tv, out, lse, T, C, H, sl2);
    else
        attn_fwd_tc_kernel<false><<<nqt * B * H, ATT_THREADS, ATT_SMEM, s>>>(tqk, tv, out, lse, T, C, H, sl2);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    return OK;
}

// TF32 causal attention backward on tcgen05 (head size 64): D must already
// hold rowsum(dO * O) per (sequence * head, row). ERR_ARG without launching
// when the shapes or alignment do not fit.
int attention_bwd_tc(const float *qkv, const float *dout, const float *lse, const float *D, float *dqkv, int B,
                     int T, int C, int H, cudaStream_t s) {
    auto al = [](const void *p) { return ((uintptr_t)p % 16) == 0; };
    if (C / H != 64 || C % H != 0 || C % 4 != 0 || !al(qkv) || !al(dout) || !al(dqkv)) return ERR_ARG;
    CUtensorMap qk128, qk64, mn, do128, do64, domn;
    const long rows = (long)B * T;
    CG_TRY(make_tensor_map(&qk128, qkv, 3L * C, rows, 3L * C, 32, 128, false));
    CG_TRY(make_tensor_map(&qk64, qkv, 3L * C, rows, 3L * C, 32, 64, false));
    CG_TRY(make_tensor_map(&mn, qkv, 3L * C, rows, 3L * C, 32, 32, true));
    CG_TRY(make_tensor_map(&do128, dout, C, rows, C, 32, 128, false));
    CG_TRY(make_tensor_map(&do64, dout, C, rows, C, 32, 64, false));
    CG_TRY(make_tensor_map(&domn, dout, C, rows, C, 32, 32, true));
    static bool attr = false;
    if (!attr) {
        CG_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, KV_SMEM));
        CG_CUDA(cudaFuncSetAttribute(attn_bwd_dkdv_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, KV_SMEM));
        CG_CUDA(cudaFuncSetAttribute(attn_bwd_dq_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, DQ_SMEM));
        CG_CUDA(cudaFuncSetAttribute(attn_bwd_dq_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, DQ_SMEM));
        attr = true;
    }
    const int nt = (T + 127) / 128;
    const float scale = 0.125f, sl2 = scale * LOG2Ef;  // 1 / sqrt(64)
    const bool ts = fwd_p_in_tmem();
    auto dkdv = ts ? attn_bwd_dkdv_tc_kernel<true> : attn_bwd_dkdv_tc_kernel<false>;
    auto dq = ts ? attn_bwd_dq_tc_kernel<true> : attn_bwd_dq_tc_kernel<false>;
    dkdv<<<nt * B * H, BWD_THREADS, KV_SMEM, s>>>(qk128, qk64, mn, do64, domn, lse, D, dqkv, T, C, H, sl2, scale);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    dq<<<nt * B * H, BWD_THREADS, DQ_SMEM, s>>>(qk128, qk64, mn, do128, lse, D, dqkv, T, C, H, sl2, scale);
    ++g_launch_count;
    CG_CUDA(cudaGetLastError());
    return OK;
}

}  // namespace cg
