// attention.cu - fused causal self-attention (reference: src/model.c:514-563
// forward, src/model.c:742-822 backward, src/fast.c:264-298 inference).
//
// The reference materialises S = QK^T/sqrt(hs), masks, softmaxes into P and
// multiplies P V per (batch, head). Here every (batch, head, 64-query tile)
// runs as one block that streams 64-key tiles through shared memory with an
// online softmax, so no T x T matrix is written. The backward recomputes P
// from the saved row log-sum-exp in two deterministic passes (dK/dV by key
// tile, dQ by query tile) instead of accumulating dQ with atomics.
//
// Head size 64 (every BASELINE config) uses the tensor cores through
// mma.sync m16n8k8 TF32; in 3xTF32 mode each product is split as
// hi*hi + hi*lo + lo*hi. Other head sizes (the reference's unit tests use
// hs = 8) take a CUDA-core kernel with one warp per query row.
#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace cg {

CG_DEV_ERROR_ACCESSORS(attn_take_dev_error, attn_set_wait_limit)

namespace {

constexpr int HS = 64;
constexpr int TQ = 64, TK = 64;  // query / key tile
constexpr int LDS = HS + 4;      // smem row pitch (floats)

__device__ __forceinline__ uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void mma8(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// d += a * b with fp32 operands. TF32 mode passes the fp32 bit patterns
// straight to the tensor core, which reads them as tf32 (dropping the low 13
// mantissa bits); 3xTF32 mode splits each operand into rna-rounded hi/lo
// parts and issues lo*hi + hi*lo + hi*hi.
template <bool SPLIT>
__device__ __forceinline__ void mma_f32(float (&d)[4], const float (&a)[4], const float (&b)[2]) {
    uint32_t ah[4], bh[2];
    if constexpr (!SPLIT) {
#pragma unroll
        for (int i = 0; i < 4; ++i) ah[i] = __float_as_uint(a[i]);
#pragma unroll
        for (int i = 0; i < 2; ++i) bh[i] = __float_as_uint(b[i]);
        mma8(d, ah, bh);
    } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) ah[i] = to_tf32(a[i]);
#pragma unroll
        for (int i = 0; i < 2; ++i) bh[i] = to_tf32(b[i]);
        uint32_t al[4], bl[2];
#pragma unroll
        for (int i = 0; i < 4; ++i) al[i] = to_tf32(a[i] - __uint_as_float(ah[i]));
#pragma unroll
        for (int i = 0; i < 2; ++i) bl[i] = to_tf32(b[i] - __uint_as_float(bh[i]));
        mma8(d, al, bh);
        mma8(d, ah, bl);
        mma8(d, ah, bh);
    }
}

// Key order inside an 8-wide n-tile: accumulator column n holds key sig(n), so
// a thread's C-fragment columns (2t, 2t+1) are keys (t, t+4) - exactly the
// A-fragment columns it needs when the result feeds the next product.
__device__ __forceinline__ int sig(int n) { return (n >> 1) + 4 * (n & 1); }

// Load a [rows x 64] tile with row pitch `ld` (floats) into smem [rows][LDS]
// with cp.async (16 bytes per copy; rows >= valid are zero-filled), so the
// copy of the next tile overlaps the math on the current one.
__device__ __forceinline__ void load_tile_async(float *dst, const float *src, long ld, int rows,
                                                int valid) {
    for (int i = threadIdx.x; i < rows * (HS / 4); i += blockDim.x) {
        const int r = i / (HS / 4), c4 = i % (HS / 4);
        const bool ok = r < valid;
        const float *g = src + (long)(ok ? r : 0) * ld + c4 * 4;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                     ::"r"(smem_u32(dst + r * LDS + c4 * 4)), "l"(g), "r"(ok ? 16 : 0) : "memory");
    }
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// ldmatrix.x4: four 8x(16-byte) matrices; lane l gives the address of row
// l % 8 of matrix l / 8 and receives, from each matrix, the 32-bit word at
// (row l / 4, word l % 4) - which for 32-bit data is a tf32 mma fragment
// element. Rows are 272 bytes apart (LDS = 68 floats): conflict-free.
__device__ __forceinline__ void ldsm4(float (&r)[4], const float *p) {
    uint32_t x0, x1, x2, x3;
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(x0), "=r"(x1), "=r"(x2), "=r"(x3) : "r"(smem_u32(p)));
    r[0] = __uint_as_float(x0);
    r[1] = __uint_as_float(x1);
    r[2] = __uint_as_float(x2);
    r[3] = __uint_as_float(x3);
}

// A fragment (16 rows x 8 cols starting at row r0, col k0) from smem [.][LDS]:
// matrices (rows 0-7, cols 0-3), (rows 8-15, cols 0-3), (0-7, 4-7), (8-15, 4-7)
__device__ __forceinline__ void frag_a(float (&a)[4], const float *s, int r0, int k0, int lane) {
    const int mat = lane >> 3, rr = lane & 7;
    ldsm4(a, s + (r0 + rr + (mat & 1) * 8) * LDS + k0 + (mat >> 1) * 4);
}

// B fragments of two consecutive k-steps (k0 and k0+8) where the operand's n
// index runs over smem rows, permuted by sig, and k over smem columns:
// element (k, n) = s[n0 + sig(n)][k]. b[0..1] is the k0 step, b[2..3] k0+8.
__device__ __forceinline__ void frag_b_rows2(float (&b)[4], const float *s, int n0, int k0, int lane) {
    const int mat = lane >> 3, rr = lane & 7;
    ldsm4(b, s + (n0 + sig(rr)) * LDS + k0 + mat * 4);
}

// 2^x on the special-function unit (ex2.approx; |rel. err| ~ 2^-22)
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

// B fragment where k runs over smem rows and n over smem columns:
// element (k, n) = s[(k0 + k)][n0 + n].
__device__ __forceinline__ void frag_b_cols(float (&b)[2], const float *s, int k0, int n0, int g,
                                            int t) {
    b[0] = s[(k0 + t) * LDS + n0 + g];
    b[1] = s[(k0 + t + 4) * LDS + n0 + g];
}

// ------------------------------------------------------------- forward
// One block per (batch*head, 128-query tile), 8 warps of 16 query rows; key
// tiles of 64 stream through a double-buffered shared-memory ring.
constexpr int FQ = 128;

template <bool SPLIT>
__global__ void __launch_bounds__(256)
attn_fwd_mma_kernel(const float *__restrict__ qkv, float *__restrict__ out, float *__restrict__ lse,
                    int T, int C, int H, float scale) {
    extern __shared__ float sm[];
    float *sQ = sm;
    float *sK[2] = {sm + FQ * LDS, sm + (FQ + TK) * LDS};
    float *sV[2] = {sm + (FQ + 2 * TK) * LDS, sm + (FQ + 3 * TK) * LDS};
    const int nqt = (T + FQ - 1) / FQ;
    const int qt = nqt - 1 - blockIdx.x;  // heaviest tiles first
    const int bh = blockIdx.y, b = bh / H, h = bh % H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const long ld = 3L * C;
    const float *base = qkv + (long)b * T * ld;
    const int q0 = qt * FQ;
    const int nkt = (min(T, q0 + FQ) + TK - 1) / TK;
    load_tile_async(sQ, base + (long)q0 * ld + h * HS, ld, FQ, min(FQ, T - q0));
    load_tile_async(sK[0], base + C + h * HS, ld, TK, min(TK, T));
    load_tile_async(sV[0], base + 2 * C + h * HS, ld, TK, min(TK, T));
    cp_async_commit();

    float o[8][4] = {};
    float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
    const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;

    for (int kt = 0; kt < nkt; ++kt) {
        const int k0 = kt * TK, buf = kt & 1;
        if (kt + 1 < nkt) {
            const int k1 = k0 + TK;
            load_tile_async(sK[buf ^ 1], base + (long)k1 * ld + C + h * HS, ld, TK, min(TK, T - k1));
            load_tile_async(sV[buf ^ 1], base + (long)k1 * ld + 2 * C + h * HS, ld, TK, min(TK, T - k1));
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        if (k0 <= q0 + warp * 16 + 15) {  // else every key of the tile is in this warp's future
            const float *cK = sK[buf], *cV = sV[buf];
            float s[8][4] = {};
#pragma unroll
            for (int kk = 0; kk < HS / 8; kk += 2) {
                float a0[4], a1[4];
                frag_a(a0, sQ, warp * 16, kk * 8, lane);
                frag_a(a1, sQ, warp * 16, kk * 8 + 8, lane);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float bb[4];
                    frag_b_rows2(bb, cK, j * 8, kk * 8, lane);
                    const float b0[2] = {bb[0], bb[1]}, b1[2] = {bb[2], bb[3]};
                    mma_f32<SPLIT>(s[j], a0, b0);
                    mma_f32<SPLIT>(s[j], a1, b1);
                }
            }
            // scores in log2 units: s * scale * log2(e); the row max and the
            // probabilities use ex2 (the first processed tile, k0 = 0, always
            // holds key 0 <= row, so the running max is finite from then on)
            const float sl2 = scale * LOG2E;
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int key = k0 + j * 8 + t + ((e & 1) ? 4 : 0);
                    const int row = (e < 2) ? row0 : row1;
                    float v = s[j][e] * sl2;
                    if (key > row || key >= T) v = -INFINITY;
                    s[j][e] = v;
                    mx[e >> 1] = fmaxf(mx[e >> 1], v);
                }
            }
            float corr[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
                mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
                const float mnew = fmaxf(m_r[r], mx[r]);
                corr[r] = ex2(m_r[r] - mnew);
                m_r[r] = mnew;
            }
            float ls[2] = {0.f, 0.f};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float p = ex2(s[j][e] - m_r[e >> 1]);
                    s[j][e] = p;
                    ls[e >> 1] += p;
                }
            }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 1);
                ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 2);
                l_r[r] = l_r[r] * corr[r] + ls[r];
            }
#pragma unroll
            for (int dn = 0; dn < 8; ++dn) {
                o[dn][0] *= corr[0];
                o[dn][1] *= corr[0];
                o[dn][2] *= corr[1];
                o[dn][3] *= corr[1];
            }
            // O += P V ; P's C fragment of key tile j is the A fragment {c0, c2, c1, c3}
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float a[4] = {s[j][0], s[j][2], s[j][1], s[j][3]};
#pragma unroll
                for (int dn = 0; dn < 8; ++dn) {
                    float bb[2];
                    frag_b_cols(bb, cV, j * 8, dn * 8, g, t);
                    mma_f32<SPLIT>(o[dn], a, bb);
                }
            }
        }
        __syncthreads();  // the next iteration's prefetch overwrites this buffer
    }
    if (row0 >= T && row1 >= T) return;
    const float inv0 = 1.0f / l_r[0], inv1 = 1.0f / l_r[1];
#pragma unroll
    for (int dn = 0; dn < 8; ++dn) {
        const int col = h * HS + dn * 8 + 2 * t;
        if (row0 < T)
            *(float2 *)(out + ((long)b * T + row0) * C + col) = make_float2(o[dn][0] * inv0, o[dn][1] * inv0);
        if (row1 < T)
            *(float2 *)(out + ((long)b * T + row1) * C + col) = make_float2(o[dn][2] * inv1, o[dn][3] * inv1);
    }
    if (lse && t == 0) {  // natural-log units: (m2 + log2 l) * ln 2
        if (row0 < T) lse[(long)bh * T + row0] = m_r[0] * LN2 + logf(l_r[0]);
        if (row1 < T) lse[(long)bh * T + row1] = m_r[1] * LN2 + logf(l_r[1]);
    }
}

// ------------------------------------------------------------- backward
// D[bh, t] = sum_d dO[b,t,h*hs+d] * O[b,t,h*hs+d]
__global__ void attn_bwd_dot_kernel(const float *__restrict__ out, const float *__restrict__ dout,
                                    float *__restrict__ D, int B, int T, int C, int H, int hs) {
    const long rows = (long)B * H * T;
    const int lane = threadIdx.x & 31;
    for (long r = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; r < rows;
         r += ((long)gridDim.x * blockDim.x) >> 5) {
        const long bh = r / T;
        const int tt = (int)(r % T), b = (int)(bh / H), h = (int)(bh % H);
        const float *o = out + ((long)b * T + tt) * C + h * hs;
        const float *d = dout + ((long)b * T + tt) * C + h * hs;
        float s = 0.f;
        for (int i = lane; i < hs; i += 32) s += o[i] * d[i];
        s = warp_sum(s);
        if (lane == 0) D[r] = s;
    }
}

// Same for head size 64 with 16-byte loads: a warp takes a whole token row
// (b, t) of every head - lane l reads float4 l + 32 j of O and dO, which lie
// in head 2 j + l / 16 - so its loads are coalesced across the row, and each
// half-warp reduces one head's 16 float4 products.
__global__ void attn_bwd_dot64_kernel(const float *__restrict__ out, const float *__restrict__ dout,
                                      float *__restrict__ D, int B, int T, int C, int H) {
    const long rows = (long)B * T;
    const int lane = threadIdx.x & 31, C4 = C >> 2;
    for (long r = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; r < rows;
         r += ((long)gridDim.x * blockDim.x) >> 5) {
        const int b = (int)(r / T), tt = (int)(r % T);
        const float4 *o = (const float4 *)(out + r * C), *d = (const float4 *)(dout + r * C);
        for (int j = 0; 32 * j < C4; ++j) {
            const int f = lane + 32 * j;
            float s = 0.f;
            if (f < C4) {
                const float4 a = __ldcs(o + f), g = __ldcs(d + f);
                s = (a.x * g.x + a.y * g.y) + (a.z * g.z + a.w * g.w);
            }
#pragma unroll
            for (int k = 8; k > 0; k >>= 1) s += __shfl_xor_sync(0xffffffffu, s, k);
            const int h = 2 * j + (lane >> 4);
            if ((lane & 15) == 0 && h < H) D[((long)b * H + h) * T + tt] = s;
        }
    }
}

// dK, dV for one 64-key tile; loops over query tiles qt >= kt with the next
// Q / dO tile prefetched while the current one is used.
template <bool SPLIT>
__global__ void __launch_bounds__(128)
attn_bwd_dkdv_kernel(const float *__restrict__ qkv, const float *__restrict__ dout,
                     const float *__restrict__ lse, const float *__restrict__ Dd,
                     float *__restrict__ dqkv, int T, int C, int H, float scale) {
    extern __shared__ float sm[];
    float *sK = sm, *sV = sm + TK * LDS;
    float *sQ[2] = {sm + 2 * TK * LDS, sm + (2 * TK + TQ) * LDS};
    float *sO[2] = {sm + (2 * TK + 2 * TQ) * LDS, sm + (2 * TK + 3 * TQ) * LDS};
    float *sLD = sm + (2 * TK + 4 * TQ) * LDS;  // [2][2][TQ]: lse, D per buffer
    const int nkt = (T + TK - 1) / TK;
    const int kt = blockIdx.x;  // tile 0 has the most work: launched first
    const int bh = blockIdx.y, b = bh / H, h = bh % H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const long ld = 3L * C;
    const float *base = qkv + (long)b * T * ld;
    const float *dob = dout + (long)b * T * C;
    const int k0 = kt * TK;
    auto load_q = [&](int qt, int buf) {
        const int q0 = qt * TQ;
        load_tile_async(sQ[buf], base + (long)q0 * ld + h * HS, ld, TQ, min(TQ, T - q0));
        load_tile_async(sO[buf], dob + (long)q0 * C + h * HS, C, TQ, min(TQ, T - q0));
        for (int i = threadIdx.x; i < TQ; i += blockDim.x) {
            const int q = q0 + i;
            sLD[buf * 2 * TQ + i] = q < T ? lse[(long)bh * T + q] : 0.f;
            sLD[buf * 2 * TQ + TQ + i] = q < T ? Dd[(long)bh * T + q] : 0.f;
        }
    };
    load_tile_async(sK, base + (long)k0 * ld + C + h * HS, ld, TK, min(TK, T - k0));
    load_tile_async(sV, base + (long)k0 * ld + 2 * C + h * HS, ld, TK, min(TK, T - k0));
    load_q(kt, 0);
    cp_async_commit();
    float dk[8][4] = {}, dv[8][4] = {};
    const int key0 = k0 + warp * 16 + g, key1 = key0 + 8;
    for (int qt = kt; qt < nkt; ++qt) {
        const int q0 = qt * TQ, buf = (qt - kt) & 1;
        if (qt + 1 < nkt) {
            load_q(qt + 1, buf ^ 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float *cQ = sQ[buf], *cO = sO[buf], *cL = sLD + buf * 2 * TQ, *cD = cL + TQ;
        // S^T = K Q^T and dP^T = V dO^T  (rows: this warp's 16 keys, cols: 64 queries)
        float st[8][4] = {}, dpt[8][4] = {};
#pragma unroll
        for (int kk = 0; kk < HS / 8; kk += 2) {
            float ak0[4], ak1[4], av0[4], av1[4];
            frag_a(ak0, sK, warp * 16, kk * 8, lane);
            frag_a(ak1, sK, warp * 16, kk * 8 + 8, lane);
            frag_a(av0, sV, warp * 16, kk * 8, lane);
            frag_a(av1, sV, warp * 16, kk * 8 + 8, lane);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float bq[4], bo[4];
                frag_b_rows2(bq, cQ, j * 8, kk * 8, lane);
                frag_b_rows2(bo, cO, j * 8, kk * 8, lane);
                const float q0b[2] = {bq[0], bq[1]}, q1b[2] = {bq[2], bq[3]};
                const float o0b[2] = {bo[0], bo[1]}, o1b[2] = {bo[2], bo[3]};
                mma_f32<SPLIT>(st[j], ak0, q0b);
                mma_f32<SPLIT>(st[j], ak1, q1b);
                mma_f32<SPLIT>(dpt[j], av0, o0b);
                mma_f32<SPLIT>(dpt[j], av1, o1b);
            }
        }
        // P^T = exp(S^T*scale - lse[q]) (0 where q < key), dS^T = P^T (dP^T - D[q])
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int qi = j * 8 + t + ((e & 1) ? 4 : 0);
                const int q = q0 + qi;
                const int key = (e < 2) ? key0 : key1;
                float p = 0.f;
                if (q >= key && q < T && key < T) p = ex2((st[j][e] * scale - cL[qi]) * LOG2E);
                st[j][e] = p;
                dpt[j][e] = p * (dpt[j][e] - cD[qi]);
            }
        }
        // dV += P^T dO ; dK += dS^T Q
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float ap[4] = {st[j][0], st[j][2], st[j][1], st[j][3]};
            const float as[4] = {dpt[j][0], dpt[j][2], dpt[j][1], dpt[j][3]};
#pragma unroll
            for (int dn = 0; dn < 8; ++dn) {
                float bo[2], bq[2];
                frag_b_cols(bo, cO, j * 8, dn * 8, g, t);
                frag_b_cols(bq, cQ, j * 8, dn * 8, g, t);
                mma_f32<SPLIT>(dv[dn], ap, bo);
                mma_f32<SPLIT>(dk[dn], as, bq);
            }
        }
        __syncthreads();  // the next iteration's prefetch overwrites this buffer
    }
    float *dkb = dqkv + (long)b * T * ld + C + h * HS;
    float *dvb = dqkv + (long)b * T * ld + 2 * C + h * HS;
#pragma unroll
    for (int dn = 0; dn < 8; ++dn) {
        const int col = dn * 8 + 2 * t;
        if (key0 < T) {
            *(float2 *)(dkb + (long)key0 * ld + col) = make_float2(dk[dn][0] * scale, dk[dn][1] * scale);
            *(float2 *)(dvb + (long)key0 * ld + col) = make_float2(dv[dn][0], dv[dn][1]);
        }
        if (key1 < T) {
            *(float2 *)(dkb + (long)key1 * ld + col) = make_float2(dk[dn][2] * scale, dk[dn][3] * scale);
            *(float2 *)(dvb + (long)key1 * ld + col) = make_float2(dv[dn][2], dv[dn][3]);
        }
    }
}

// dQ for one 64-query tile; loops over key tiles kt <= qt with the next K / V
// tile prefetched while the current one is used.
template <bool SPLIT>
__global__ void __launch_bounds__(128)
attn_bwd_dq_kernel(const float *__restrict__ qkv, const float *__restrict__ dout,
                   const float *__restrict__ lse, const float *__restrict__ Dd,
                   float *__restrict__ dqkv, int T, int C, int H, float scale) {
    extern __shared__ float sm[];
    float *sQ = sm, *sO = sm + TQ * LDS;
    float *sK[2] = {sm + 2 * TQ * LDS, sm + (2 * TQ + TK) * LDS};
    float *sV[2] = {sm + (2 * TQ + 2 * TK) * LDS, sm + (2 * TQ + 3 * TK) * LDS};
    const int nqt = (T + TQ - 1) / TQ;
    const int qt = nqt - 1 - blockIdx.x;
    const int bh = blockIdx.y, b = bh / H, h = bh % H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const long ld = 3L * C;
    const float *base = qkv + (long)b * T * ld;
    const int q0 = qt * TQ;
    load_tile_async(sQ, base + (long)q0 * ld + h * HS, ld, TQ, min(TQ, T - q0));
    load_tile_async(sO, dout + ((long)b * T + q0) * C + h * HS, C, TQ, min(TQ, T - q0));
    load_tile_async(sK[0], base + C + h * HS, ld, TK, min(TK, T));
    load_tile_async(sV[0], base + 2 * C + h * HS, ld, TK, min(TK, T));
    cp_async_commit();
    const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;
    const float L0 = row0 < T ? lse[(long)bh * T + row0] : 0.f;
    const float L1 = row1 < T ? lse[(long)bh * T + row1] : 0.f;
    const float D0 = row0 < T ? Dd[(long)bh * T + row0] : 0.f;
    const float D1 = row1 < T ? Dd[(long)bh * T + row1] : 0.f;
    float dq[8][4] = {};
    for (int kt = 0; kt <= qt; ++kt) {
        const int k0 = kt * TK, buf = kt & 1;
        if (kt + 1 <= qt) {
            const int k1 = k0 + TK;
            load_tile_async(sK[buf ^ 1], base + (long)k1 * ld + C + h * HS, ld, TK, min(TK, T - k1));
            load_tile_async(sV[buf ^ 1], base + (long)k1 * ld + 2 * C + h * HS, ld, TK, min(TK, T - k1));
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const float *cK = sK[buf], *cV = sV[buf];
        float s[8][4] = {}, dp[8][4] = {};
#pragma unroll
        for (int kk = 0; kk < HS / 8; kk += 2) {
            float aq0[4], aq1[4], ao0[4], ao1[4];
            frag_a(aq0, sQ, warp * 16, kk * 8, lane);
            frag_a(aq1, sQ, warp * 16, kk * 8 + 8, lane);
            frag_a(ao0, sO, warp * 16, kk * 8, lane);
            frag_a(ao1, sO, warp * 16, kk * 8 + 8, lane);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float bk[4], bv[4];
                frag_b_rows2(bk, cK, j * 8, kk * 8, lane);
                frag_b_rows2(bv, cV, j * 8, kk * 8, lane);
                const float k0b[2] = {bk[0], bk[1]}, k1b[2] = {bk[2], bk[3]};
                const float v0b[2] = {bv[0], bv[1]}, v1b[2] = {bv[2], bv[3]};
                mma_f32<SPLIT>(s[j], aq0, k0b);
                mma_f32<SPLIT>(s[j], aq1, k1b);
                mma_f32<SPLIT>(dp[j], ao0, v0b);
                mma_f32<SPLIT>(dp[j], ao1, v1b);
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int key = k0 + j * 8 + t + ((e & 1) ? 4 : 0);
                const int row = (e < 2) ? row0 : row1;
                float p = 0.f;
                if (key <= row && key < T && row < T)
                    p = ex2((s[j][e] * scale - ((e < 2) ? L0 : L1)) * LOG2E);
                s[j][e] = p * (dp[j][e] - ((e < 2) ? D0 : D1));  // dS
            }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float a[4] = {s[j][0], s[j][2], s[j][1], s[j][3]};
#pragma unroll
            for (int dn = 0; dn < 8; ++dn) {
                float bk[2];
                frag_b_cols(bk, cK, j * 8, dn * 8, g, t);
                mma_f32<SPLIT>(dq[dn], a, bk);
            }
        }
        __syncthreads();
    }
    float *dqb = dqkv + (long)b * T * ld + h * HS;
#pragma unroll
    for (int dn = 0; dn < 8; ++dn) {
        const int col = dn * 8 + 2 * t;
        if (row0 < T) *(float2 *)(dqb + (long)row0 * ld + col) = make_float2(dq[dn][0] * scale, dq[dn][1] * scale);
        if (row1 < T) *(float2 *)(dqb + (long)row1 * ld + col) = make_float2(dq[dn][2] * scale, dq[dn][3] * scale);
    }
}

// ----------------------------------------------- CUDA-core kernels (any hs)
// One warp per query row; lanes hold head dims d = lane + 32*i (hs <= 128).
// Keys are processed in order with an online softmax.
__global__ void attn_fwd_simt_kernel(const float *__restrict__ qkv, float *__restrict__ out,
                                     float *__restrict__ lse, int B, int T, int C, int H, int hs,
                                     float scale, int q0) {
    const int lane = threadIdx.x & 31;
    const long rows = (long)B * H * (T - q0);
    for (long r = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; r < rows;
         r += ((long)gridDim.x * blockDim.x) >> 5) {
        const long bh = r / (T - q0);
        const int tq = q0 + (int)(r % (T - q0)), b = (int)(bh / H), h = (int)(bh % H);
        const long ld = 3L * C;
        const float *qr = qkv + ((long)b * T + tq) * ld + h * hs;
        float q[4], o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = (lane + 32 * i < hs) ? qr[lane + 32 * i] : 0.f;
        float m = -INFINITY, l = 0.f;
        for (int j = 0; j <= tq; ++j) {
            const float *kr = qkv + ((long)b * T + j) * ld + C + h * hs;
            const float *vr = kr + C;
            float d = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (lane + 32 * i < hs) d += q[i] * kr[lane + 32 * i];
            const float sc = warp_sum(d) * scale;
            const float mn = fmaxf(m, sc);
            const float corr = (m == -INFINITY) ? 0.f : expf(m - mn);
            const float p = expf(sc - mn);
            l = l * corr + p;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (lane + 32 * i < hs) o[i] = o[i] * corr + p * vr[lane + 32 * i];
            m = mn;
        }
        float *orow = out + ((long)b * T + tq) * C + h * hs;
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (lane + 32 * i < hs) orow[lane + 32 * i] = o[i] / l;
        if (lse && lane == 0) lse[bh * T + tq] = m + logf(l);
    }
}

// dQ rows (mode 0, one warp per query row) or dK/dV rows (mode 1, one warp
// per key row), recomputing P from the saved lse.
__global__ void attn_bwd_simt_kernel(const float *__restrict__ qkv, const float *__restrict__ dout,
                                     const float *__restrict__ lse, const float *__restrict__ Dd,
                                     float *__restrict__ dqkv, int B, int T, int C, int H, int hs,
                                     float scale, int mode) {
    const int lane = threadIdx.x & 31;
    const long rows = (long)B * H * T;
    const long ld = 3L * C;
    for (long r = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5; r < rows;
         r += ((long)gridDim.x * blockDim.x) >> 5) {
        const long bh = r / T;
        const int x = (int)(r % T), b = (int)(bh / H), h = (int)(bh % H);
        const float *qb = qkv + (long)b * T * ld + h * hs;
        const float *kb = qb + C, *vb = qb + 2 * C;
        const float *ob = dout + (long)b * T * C + h * hs;
        float acc0[4] = {0.f, 0.f, 0.f, 0.f}, acc1[4] = {0.f, 0.f, 0.f, 0.f};
        if (mode == 0) {  // x = query row
            const int lo = 0, hi = x;
            for (int j = lo; j <= hi; ++j) {
                float sd = 0.f, dpd = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int d = lane + 32 * i;
                    if (d < hs) {
                        sd += qb[(long)x * ld + d] * kb[(long)j * ld + d];
                        dpd += ob[(long)x * C + d] * vb[(long)j * ld + d];
                    }
                }
                const float p = expf(warp_sum(sd) * scale - lse[bh * T + x]);
                const float ds = p * (warp_sum(dpd) - Dd[bh * T + x]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int d = lane + 32 * i;
                    if (d < hs) acc0[i] += ds * kb[(long)j * ld + d];
                }
            }
            float *dq = dqkv + ((long)b * T + x) * ld + h * hs;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (lane + 32 * i < hs) dq[lane + 32 * i] = acc0[i] * scale;
        } else {  // x = key row
            for (int q = x; q < T; ++q) {
                float sd = 0.f, dpd = 0.f;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int d = lane + 32 * i;
                    if (d < hs) {
                        sd += qb[(long)q * ld + d] * kb[(long)x * ld + d];
                        dpd += ob[(long)q * C + d] * vb[(long)x * ld + d];
                    }
                }
                const float p = expf(warp_sum(sd) * scale - lse[bh * T + q]);
                const float ds = p * (warp_sum(dpd) - Dd[bh * T + q]);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int d = lane + 32 * i;
                    if (d < hs) {
                        acc0[i] += ds * qb[(long)q * ld + d];   // dK
                        acc1[i] += p * ob[(long)q * C + d];     // dV
                    }
                }
            }
            float *dk = dqkv + ((long)b * T + x) * ld + C + h * hs;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (lane + 32 * i < hs) {
                    dk[lane + 32 * i] = acc0[i] * scale;
                    dk[C + lane + 32 * i] = acc1[i];
                }
        }
    }
}

// Decode: one block per (sequence, head); scores for all cached positions in
// shared memory, then a block softmax and P V with threads over head dims.
__global__ void __launch_bounds__(256)
attn_decode_kernel(const float *__restrict__ q, long ldq, const float *__restrict__ kc,
                   const float *__restrict__ vc, long Tmax, int len, float *__restrict__ out,
                   int C, int H, int hs, float scale, int vec4, const int *__restrict__ pos_dev) {
    extern __shared__ float sm[];
    // with a device position the scores area is sized for the capacity Tmax
    float *sq = sm, *sp = sm + hs, *red = sp + (pos_dev ? (int)Tmax : len);  // red: 64 floats
    if (pos_dev) len = *pos_dev + 1;
    const int bh = blockIdx.x, b = bh / H, h = bh % H;
    const float *qr = q + (long)b * ldq + h * hs;
    for (int i = threadIdx.x; i < hs; i += blockDim.x) sq[i] = qr[i];
    __syncthreads();
    const float *kb = kc + (long)b * Tmax * C + h * hs;
    const float *vb = vc + (long)b * Tmax * C + h * hs;
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < len; j += blockDim.x) {
        const float *kr = kb + (long)j * C;
        float d = 0.f;
        if (vec4) {
            for (int i = 0; i < hs; i += 4) {
                const float4 kv = *(const float4 *)(kr + i);
                d += sq[i] * kv.x + sq[i + 1] * kv.y + sq[i + 2] * kv.z + sq[i + 3] * kv.w;
            }
        } else {
            for (int i = 0; i < hs; ++i) d += sq[i] * kr[i];
        }
        d *= scale;
        sp[j] = d;
        mx = fmaxf(mx, d);
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    mx = warp_max(mx);
    if (lane == 0) red[wid] = mx;
    __syncthreads();
    mx = red[0];
    for (int k = 1; k < nw; ++k) mx = fmaxf(mx, red[k]);
    __syncthreads();
    float s = 0.f;
    for (int j = threadIdx.x; j < len; j += blockDim.x) {
        const float p = expf(sp[j] - mx);
        sp[j] = p;
        s += p;
    }
    s = warp_sum(s);
    if (lane == 0) red[wid] = s;
    __syncthreads();
    s = 0.f;
    for (int k = 0; k < nw; ++k) s += red[k];
    const float inv = 1.0f / s;
    // P V: thread (group, d) sums keys j = group (mod G) for dim d
    const int G = blockDim.x / hs;
    const int d = threadIdx.x % hs, grp = threadIdx.x / hs;
    float acc = 0.f;
    if (grp < G)
        for (int j = grp; j < len; j += G) acc += sp[j] * vb[(long)j * C + d];
    __syncthreads();
    float *part = red + 64;  // G * hs floats
    if (grp < G) part[grp * hs + d] = acc;
    __syncthreads();
    if (threadIdx.x < hs) {
        float o = 0.f;
        for (int k = 0; k < G; ++k) o += part[k * hs + threadIdx.x];
        out[(long)b * C + h * hs + threadIdx.x] = o * inv;
    }
}

// Split-context decode for head size 64 (flash-decoding): block (b*H + h,
// split) scores keys [64*split, 64*split + 64) with a half-warp per key
// (float4 per lane, 4-step shuffle reduction) and forms the chunk's softmax
// partials (max m, sum l, unnormalised P V). The last block of a head to
// finish (integer ticket; the partials are made visible with a fence before
// the ticket is taken) merges every chunk of the head in chunk order, so the
// result does not depend on which block came last, and resets the ticket.
// Launched with programmatic dependent launch: nothing is read before
// griddepcontrol.wait.
constexpr int DEC_KEYS = 64, DEC_PART = 66;

__global__ void __launch_bounds__(128)
attn_decode_split_kernel(const float *__restrict__ q, long ldq, const float *__restrict__ kc,
                         const float *__restrict__ vc, long Tmax, int len, const int *__restrict__ pos_dev,
                         float *__restrict__ part, int *__restrict__ tickets, float *__restrict__ out,
                         int C, int H, int S, float scale) {
    pdl_trigger();
    pdl_wait();
    if (pos_dev) len = *pos_dev + 1;
    const int bh = blockIdx.x, split = blockIdx.y, b = bh / H, h = bh % H;
    const int j0 = split * DEC_KEYS;
    if (j0 >= len) return;  // uniform over the block: an empty chunk takes no ticket
    __shared__ float sc[DEC_KEYS], pr[DEC_KEYS], so[64], red[2], cm[64], cl[64];
    __shared__ int last;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, half = lane >> 4, l16 = lane & 15;
    const float4 qv = *(const float4 *)(q + (long)b * ldq + h * 64 + 4 * l16);
    const float *kb = kc + (long)b * Tmax * C + h * 64 + 4 * l16;
    float d[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int j = j0 + warp * 16 + 2 * i + half;
        float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < len) kv = *(const float4 *)(kb + (long)j * C);
        d[i] = qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w;
    }
    // V of this thread's 32 keys (thread (kh, dim): keys kh*32.., one
    // dimension), loaded while the scores are reduced
    const int dim = threadIdx.x & 63, kh = threadIdx.x >> 6;
    const int kend = min(DEC_KEYS, len - j0);
    const float *vb = vc + (long)b * Tmax * C + h * 64 + dim + (long)j0 * C;
    float vr[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) vr[i] = (kh * 32 + i < kend) ? vb[(long)(kh * 32 + i) * C] : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) d[i] += __shfl_xor_sync(0xffffffffu, d[i], o);
    if (l16 == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int jl = warp * 16 + 2 * i + half;
            sc[jl] = (j0 + jl < len) ? d[i] * scale : -INFINITY;
        }
    }
    __syncthreads();
    float m = -INFINITY;
    if (threadIdx.x < DEC_KEYS) m = sc[threadIdx.x];
    m = warp_max(m);
    if (lane == 0 && warp < 2) red[warp] = m;
    __syncthreads();
    m = fmaxf(red[0], red[1]);  // sc[0] is a valid key: m is finite
    __syncthreads();
    if (threadIdx.x < DEC_KEYS) {
        const float p = j0 + (int)threadIdx.x < len ? expf(sc[threadIdx.x] - m) : 0.f;
        pr[threadIdx.x] = p;
        const float w = warp_sum(p);
        if (lane == 0) red[warp] = w;
    }
    __syncthreads();
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) acc += pr[kh * 32 + i] * vr[i];
    if (kh == 1) so[dim] = acc;
    __syncthreads();
    float *pp = part + ((long)bh * S + split) * DEC_PART;
    if (kh == 0) {
        pp[2 + dim] = acc + so[dim];
        if (dim == 0) {
            pp[0] = m;
            pp[1] = red[0] + red[1];
        }
    }
    __threadfence();
    __syncthreads();
    const int ns = (len + DEC_KEYS - 1) / DEC_KEYS;
    if (threadIdx.x == 0) last = (atomicAdd(&tickets[bh], 1) == ns - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    // merge the chunks in chunk order: (max, sum) of every chunk first, then
    // each dimension's partial outputs (independent loads)
    const float *pb = part + (long)bh * S * DEC_PART;
    if ((int)threadIdx.x < ns) {
        cm[threadIdx.x] = __ldcg(pb + threadIdx.x * DEC_PART);
        cl[threadIdx.x] = __ldcg(pb + threadIdx.x * DEC_PART + 1);
    }
    __syncthreads();
    if (threadIdx.x < 64) {
        float M = -INFINITY;
        for (int k = 0; k < ns; ++k) M = fmaxf(M, cm[k]);
        float L = 0.f, O = 0.f;
#pragma unroll 4
        for (int k = 0; k < ns; ++k) {
            const float w = expf(cm[k] - M);
            L += cl[k] * w;
            O += __ldcg(pb + k * DEC_PART + 2 + threadIdx.x) * w;
        }
        out[(long)b * C + h * 64 + threadIdx.x] = O / L;
        if (threadIdx.x == 0) tickets[bh] = 0;
    }
}

template <typename K>
int set_smem(K kern, int bytes) {
    CG_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
    return OK;
}

}  // namespace

#define LAUNCH_CHECK() do { ++g_launch_count; CG_CUDA(cudaGetLastError()); } while (0)

namespace {
// The tensor-core kernels move rows with 16-byte cp.async / ldmatrix and store
// 8-byte pairs: every base must be 16-byte aligned and every row pitch (3C and
// C floats) a multiple of 16 bytes. Activation-arena slots are not aligned
// when B*T is odd (the mean/rstd slots before them hold B*T floats each), so
// this is checked per call and such calls take the CUDA-core kernels.
bool mma_ok(int C, std::initializer_list<const void *> ptrs) {
    if (C % 4 != 0) return false;
    for (const void *p : ptrs)
        if (p && ((uintptr_t)p % 16) != 0) return false;
    return true;
}
}  // namespace

// CNGPT_CUDA_ATTN_TC=0 keeps the TF32 forward on the mma.sync kernel
bool tc_attention_enabled() {
    static int on = -1;
    if (on < 0) {
        const char *e = getenv("CNGPT_CUDA_ATTN_TC");
        on = (e && e[0] == '0') ? 0 : 1;
    }
    return on == 1;
}

int attention_fwd(const float *qkv, float *out, float *lse, int B, int T, int C, int H,
                  cudaStream_t s) {
    if (B <= 0 || T <= 0) return OK;
    const int hs = C / H;
    const float scale = 1.0f / sqrtf((float)hs);
    if (precision() == PREC_TF32 && tc_attention_enabled() && attention_fwd_tc(qkv, out, lse, B, T, C, H, s) == OK)
        return OK;
    if (hs == HS && precision() != PREC_FP32 && mma_ok(C, {qkv, out})) {
        const int smem = (FQ + 4 * TK) * LDS * sizeof(float);
        dim3 grid((T + FQ - 1) / FQ, B * H);
        if (precision() == PREC_3XTF32) {
            static bool a = false;
            if (!a) { CG_TRY(set_smem(attn_fwd_mma_kernel<true>, smem)); a = true; }
            attn_fwd_mma_kernel<true><<<grid, 256, smem, s>>>(qkv, out, lse, T, C, H, scale);
        } else {
            static bool a = false;
            if (!a) { CG_TRY(set_smem(attn_fwd_mma_kernel<false>, smem)); a = true; }
            attn_fwd_mma_kernel<false><<<grid, 256, smem, s>>>(qkv, out, lse, T, C, H, scale);
        }
        LAUNCH_CHECK();
        return OK;
    }
    if (hs > 128) {
        set_last_error(ERR_ARG, "attention: head size %d > 128 unsupported", hs);
        return ERR_ARG;
    }
    const long rows = (long)B * H * T;
    attn_fwd_simt_kernel<<<(int)std::min<long>((rows + 7) / 8, 148L * 64), 256, 0, s>>>(
        qkv, out, lse, B, T, C, H, hs, scale, 0);
    LAUNCH_CHECK();
    return OK;
}

int attention_fwd_rows(const float *qkv, float *out, int B, int T, int C, int H, int q0,
                       cudaStream_t s) {
    const int hs = C / H;
    if (hs > 128) {
        set_last_error(ERR_ARG, "attention: head size %d > 128 unsupported", hs);
        return ERR_ARG;
    }
    const long rows = (long)B * H * (T - q0);
    if (rows <= 0) return OK;
    attn_fwd_simt_kernel<<<(int)std::min<long>((rows + 7) / 8, 148L * 64), 256, 0, s>>>(
        qkv, out, nullptr, B, T, C, H, hs, 1.0f / sqrtf((float)hs), q0);
    LAUNCH_CHECK();
    return OK;
}

size_t attention_bwd_scratch_bytes(int B, int T, int H) { return (size_t)B * H * T * sizeof(float); }

int attention_bwd(const float *qkv, const float *out, const float *dout, const float *lse,
                  float *dqkv, float *scratch, int B, int T, int C, int H, cudaStream_t s) {
    if (B <= 0 || T <= 0) return OK;
    const int hs = C / H;
    const float scale = 1.0f / sqrtf((float)hs);
    float *D = scratch;
    const long rows = (long)B * H * T;
    if (hs == 64 && C % 128 == 0 && ((uintptr_t)out % 16) == 0 && ((uintptr_t)dout % 16) == 0) {
        const long trows = (long)B * T;
        attn_bwd_dot64_kernel<<<(int)std::min<long>((trows + 7) / 8, 148L * 16), 256, 0, s>>>(out, dout, D, B, T,
                                                                                            C, H);
    } else {
        attn_bwd_dot_kernel<<<(int)std::min<long>((rows + 7) / 8, 148L * 64), 256, 0, s>>>(out, dout, D, B, T, C,
                                                                                          H, hs);
    }
    LAUNCH_CHECK();
    if (precision() == PREC_TF32 && tc_attention_enabled() &&
        attention_bwd_tc(qkv, dout, lse, D, dqkv, B, T, C, H, s) == OK)
        return OK;
    if (hs == HS && precision() != PREC_FP32 && mma_ok(C, {qkv, out, dout, dqkv})) {
        const int nt = (T + 63) / 64;
        const int smem_kv = ((2 * TK + 4 * TQ) * LDS + 4 * TQ) * sizeof(float);
        const int smem_q = (2 * TQ + 4 * TK) * LDS * sizeof(float);
        dim3 grid(nt, B * H);
        if (precision() == PREC_3XTF32) {
            static bool a = false;
            if (!a) {
                CG_TRY(set_smem(attn_bwd_dkdv_kernel<true>, smem_kv));
                CG_TRY(set_smem(attn_bwd_dq_kernel<true>, smem_q));
                a = true;
            }
            attn_bwd_dkdv_kernel<true><<<grid, 128, smem_kv, s>>>(qkv, dout, lse, D, dqkv, T, C, H, scale);
            LAUNCH_CHECK();
            attn_bwd_dq_kernel<true><<<grid, 128, smem_q, s>>>(qkv, dout, lse, D, dqkv, T, C, H, scale);
        } else {
            static bool a = false;
            if (!a) {
                CG_TRY(set_smem(attn_bwd_dkdv_kernel<false>, smem_kv));
                CG_TRY(set_smem(attn_bwd_dq_kernel<false>, smem_q));
                a = true;
            }
            attn_bwd_dkdv_kernel<false><<<grid, 128, smem_kv, s>>>(qkv, dout, lse, D, dqkv, T, C, H, scale);
            LAUNCH_CHECK();
            attn_bwd_dq_kernel<false><<<grid, 128, smem_q, s>>>(qkv, dout, lse, D, dqkv, T, C, H, scale);
        }
        LAUNCH_CHECK();
        return OK;
    }
    if (hs > 128) {
        set_last_error(ERR_ARG, "attention: head size %d > 128 unsupported", hs);
        return ERR_ARG;
    }
    const int grid = (int)std::min<long>((rows + 7) / 8, 148L * 64);
    attn_bwd_simt_kernel<<<grid, 256, 0, s>>>(qkv, dout, lse, D, dqkv, B, T, C, H, hs, scale, 0);
    LAUNCH_CHECK();
    attn_bwd_simt_kernel<<<grid, 256, 0, s>>>(qkv, dout, lse, D, dqkv, B, T, C, H, hs, scale, 1);
    LAUNCH_CHECK();
    return OK;
}

int attention_decode_impl(const float *q, long ldq, const float *kcache, const float *vcache,
                          long Tmax, int len, const int *pos_dev, float *out, int B, int C, int H,
                          float *part, cudaStream_t s) {
    const int hs = C / H;
    const int cap = pos_dev ? (int)Tmax : len;
    if (hs > 256 || cap <= 0) {
        set_last_error(ERR_ARG, "attention_decode: unsupported hs=%d len=%d", hs, cap);
        return ERR_ARG;
    }
    const float scale = 1.0f / sqrtf((float)hs);
    const bool vec4 = (C % 4 == 0) && (ldq % 4 == 0) && ((uintptr_t)kcache % 16) == 0 &&
                      ((uintptr_t)vcache % 16) == 0 && ((uintptr_t)q % 16) == 0;
    if (part && hs == 64 && vec4 && cap <= 64 * DEC_KEYS) {
        const int S = (cap + DEC_KEYS - 1) / DEC_KEYS;
        int *tickets = (int *)(part + (size_t)B * H * S * DEC_PART);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(B * H, S);
        cfg.blockDim = dim3(128);
        cfg.stream = s;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        CG_CUDA(cudaLaunchKernelEx(&cfg, attn_decode_split_kernel, q, ldq, kcache, vcache, Tmax, len, pos_dev,
                                   part, tickets, out, C, H, S, scale));
        ++g_launch_count;
        return OK;
    }
    const int G = 256 / hs;
    const size_t smem = (size_t)(hs + cap + 64 + G * hs) * sizeof(float);
    if (smem > 200 * 1024) {
        set_last_error(ERR_ARG, "attention_decode: context %d too long", cap);
        return ERR_ARG;
    }
    static bool a = false;
    if (!a) { CG_TRY(set_smem(attn_decode_kernel, 200 * 1024 + 4096)); a = true; }
    attn_decode_kernel<<<B * H, 256, smem, s>>>(q, ldq, kcache, vcache, Tmax, len, out, C, H, hs, scale,
                                                (C % 4 == 0) && ((uintptr_t)kcache % 16) == 0, pos_dev);
    LAUNCH_CHECK();
    return OK;
}

size_t attention_decode_scratch_floats(int B, int H, long Tmax) {
    // partials, then one int ticket per (sequence, head)
    return (size_t)B * H * ((Tmax + DEC_KEYS - 1) / DEC_KEYS) * DEC_PART + (size_t)B * H;
}

int attention_decode(const float *q, long ldq, const float *kcache, const float *vcache, long Tmax,
                     int len, float *out, int B, int C, int H, float *part, cudaStream_t s) {
    return attention_decode_impl(q, ldq, kcache, vcache, Tmax, len, nullptr, out, B, C, H, part, s);
}

int attention_decode_at(const float *q, long ldq, const float *kcache, const float *vcache, long Tmax,
                        const int *pos_dev, float *out, int B, int C, int H, float *part, cudaStream_t s) {
    return attention_decode_impl(q, ldq, kcache, vcache, Tmax, 0, pos_dev, out, B, C, H, part, s);
}

}  // namespace cg
