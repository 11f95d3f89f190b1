// kernels.cu - the non-GEMM device kernels of the hot path.
//
// All reductions have a fixed order (per-thread sequential sums, fixed-shape
// tree or partial-buffer reductions), so every kernel here is bit-for-bit
// deterministic run to run; no floating-point atomics are used.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace cg {

namespace {

inline int grid_for(long n, int threads, int cap = 148 * 16) {
    long g = (n + threads - 1) / threads;
    return (int)std::max(1L, std::min(g, (long)cap));
}

// ---------------------------------------------------------------- LayerNorm
// One warp per row; eps 1e-5; biased variance; two passes over the row as in
// src/ops.c:231-247 (mean first, then the sum of squared deviations).
__global__ void layernorm_fwd_kernel(const float *__restrict__ x, long ldx,
                                     const float *__restrict__ w, const float *__restrict__ b,
                                     float *__restrict__ out, long ldo, float *__restrict__ mean,
                                     float *__restrict__ rstd, int T, int C) {
    pdl_trigger();  // a GEMV launched after this may start prefetching its weights
    const int warps = blockDim.x >> 5;
    const int lane = threadIdx.x & 31;
    for (long t = (long)blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += (long)gridDim.x * warps) {
        const float *xr = x + t * ldx;
        float s = 0.f;
        for (int c = lane; c < C; c += 32) s += xr[c];
        const float m = warp_sum(s) / (float)C;
        float v = 0.f;
        for (int c = lane; c < C; c += 32) {
            float d = xr[c] - m;
            v += d * d;
        }
        const float rs = 1.0f / sqrtf(warp_sum(v) / (float)C + 1e-5f);
        if (lane == 0) {
            if (mean) mean[t] = m;
            if (rstd) rstd[t] = rs;
        }
        float *orow = out + t * ldo;
        for (int c = lane; c < C; c += 32) orow[c] = (xr[c] - m) * rs * w[c] + b[c];
    }
}

// Same for C = 128 NJ with 16-byte rows: a warp holds its row in registers
// (lane l: float4 l + 32 j), so x is read from memory once; the mean, then
// the sum of squared deviations about it, as above.
template <int NJ>
__global__ void __launch_bounds__(256)
layernorm_fwd4_kernel(const float *__restrict__ x, long ldx, const float *__restrict__ w, const float *__restrict__ b,
                      float *__restrict__ out, long ldo, float *__restrict__ mean, float *__restrict__ rstd, int T) {
    pdl_trigger();
    constexpr int C = 128 * NJ;
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (long t = (long)blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += (long)gridDim.x * warps) {
        const float4 *xr = (const float4 *)(x + t * ldx);
        float4 v[NJ];
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            v[j] = __ldg(xr + lane + 32 * j);
            s += (v[j].x + v[j].y) + (v[j].z + v[j].w);
        }
        const float m = warp_sum(s) / (float)C;
        float q = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const float a = v[j].x - m, bb = v[j].y - m, c = v[j].z - m, d = v[j].w - m;
            q += (a * a + bb * bb) + (c * c + d * d);
        }
        const float rs = 1.0f / sqrtf(warp_sum(q) / (float)C + 1e-5f);
        if (lane == 0) {
            if (mean) mean[t] = m;
            if (rstd) rstd[t] = rs;
        }
        float4 *orow = (float4 *)(out + t * ldo);
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const float4 g = __ldg((const float4 *)w + lane + 32 * j), bv = __ldg((const float4 *)b + lane + 32 * j);
            orow[lane + 32 * j] = make_float4((v[j].x - m) * rs * g.x + bv.x, (v[j].y - m) * rs * g.y + bv.y,
                                              (v[j].z - m) * rs * g.z + bv.z, (v[j].w - m) * rs * g.w + bv.w);
        }
    }
}

// dx += rstd (dn - mean(dn) - xhat mean(dn xhat)) per row (src/ops.c:305-329),
// dn = dout * w, xhat = (x - mean) * rstd: one warp per row, two passes.
__global__ void __launch_bounds__(256)
layernorm_bwd_dx_kernel(const float *__restrict__ dout, const float *__restrict__ x,
                        const float *__restrict__ w, const float *__restrict__ mean,
                        const float *__restrict__ rstd, float *__restrict__ dx, int T, int C) {
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (long t = (long)blockIdx.x * warps + (threadIdx.x >> 5); t < T; t += (long)gridDim.x * warps) {
        const float *dr = dout + t * C, *xr = x + t * C;
        const float m = mean[t], rs = rstd[t];
        float s1 = 0.f, s2 = 0.f;
#pragma unroll 4
        for (int c = lane; c < C; c += 32) {
            const float dn = dr[c] * w[c];
            s1 += dn;
            s2 += dn * ((xr[c] - m) * rs);
        }
        s1 = warp_sum(s1) / (float)C;
        s2 = warp_sum(s2) / (float)C;
        float *dxr = dx + t * C;
#pragma unroll 4
        for (int c = lane; c < C; c += 32) {
            const float xh = (xr[c] - m) * rs, dn = dr[c] * w[c];
            dxr[c] += rs * (dn - s1 - xh * s2);
        }
    }
}

// Column partials of dw = sum_t dout * xhat and db = sum_t dout over a chunk
// of rows: thread = column (coalesced across the warp), rows in order.
// part layout [chunk][2][C]; layernorm_bwd_reduce adds them in chunk order.
__global__ void __launch_bounds__(256)
layernorm_bwd_dwdb_kernel(const float *__restrict__ dout, const float *__restrict__ x,
                          const float *__restrict__ mean, const float *__restrict__ rstd,
                          float *__restrict__ part, int T, int C, int rows_per_chunk) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const long r0 = (long)blockIdx.y * rows_per_chunk;
    const long r1 = std::min<long>(T, r0 + rows_per_chunk);
    float a = 0.f, b = 0.f;
#pragma unroll 8
    for (long t = r0; t < r1; ++t) {
        const float d = dout[t * C + c];
        a += d * ((x[t * C + c] - mean[t]) * rstd[t]);
        b += d;
    }
    part[((long)blockIdx.y * 2 + 0) * C + c] = a;
    part[((long)blockIdx.y * 2 + 1) * C + c] = b;
}

// dw/db += sum of the per-block partials, in block order. One block per 32
// columns; warp w sums blocks k = w, w+8, ... and the 8 warp sums are added
// in warp order, so the result is independent of scheduling.
__global__ void __launch_bounds__(256)
layernorm_bwd_reduce(const float *__restrict__ part, int nblocks, int C, float *__restrict__ dw,
                     float *__restrict__ db) {
    __shared__ float red[8][2][32];
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = blockIdx.x * 32 + lane;
    float a = 0.f, b = 0.f;
    if (c < C)
        for (int k = wid; k < nblocks; k += 8) {
            a += part[((long)k * 2 + 0) * C + c];
            b += part[((long)k * 2 + 1) * C + c];
        }
    red[wid][0][lane] = a;
    red[wid][1][lane] = b;
    __syncthreads();
    if (wid == 0 && c < C) {
        float sa = 0.f, sb = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            sa += red[k][0][lane];
            sb += red[k][1][lane];
        }
        dw[c] += sa;
        db[c] += sb;
    }
}

// Fused LayerNorm backward of the training step, one pass over the rows:
//   dx[t, c] += rstd (dn - mean(dn) - xhat mean(dn xhat)), dn = dout w
//   (src/ops.c:305-329), with the column sums that follow it folded in:
//   dw += sum_t dout xhat, db += sum_t dout (src/ops.c:322-327) and, when cs
//   is given, cs += sum_t dx_new - the bias gradient of the linear layer
//   whose output gradient the updated dx is (src/ops.c:145-148).
// C = 128 NJ: lane l of a warp owns the float4 columns 4 (l + 32 j). Warp w of
// a block takes rows r0 + w, r0 + w + 8, ... of the block's row range and adds
// its column terms into its own shared-memory partials (no two lanes share a
// column); the block's 8 partials are then summed in warp order into
// part[block][3][C], and ln_bwd_part_reduce adds the blocks in block order -
// a fixed order, so the result is deterministic.
template <int NJ>
__global__ void __launch_bounds__(256, 2)
ln_bwd_fused_kernel(const float *__restrict__ dout, const float *__restrict__ x, const float *__restrict__ w,
                    const float *__restrict__ mean, const float *__restrict__ rstd, float *__restrict__ dx, int T,
                    int rows_per_block, float *__restrict__ part, int want_cs) {
    constexpr int C = 128 * NJ;
    extern __shared__ float4 ln_sp[];  // [8 warps][3][C / 4]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float4 *my = ln_sp + warp * 3 * (C / 4);
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
        my[lane + 32 * j] = z;
        my[C / 4 + lane + 32 * j] = z;
        my[2 * (C / 4) + lane + 32 * j] = z;
    }
    const float4 *wv = (const float4 *)w;  // read through L1 at each use (3 KB, every row)
    const long r0 = (long)blockIdx.x * rows_per_block;
    const long r1 = std::min<long>(T, r0 + rows_per_block);
    const float invC = 1.0f / (float)C;
    for (long t = r0 + warp; t < r1; t += 8) {
        const float4 *d4 = (const float4 *)(dout + t * C), *x4 = (const float4 *)(x + t * C);
        float4 *o4 = (float4 *)(dx + t * C);
        float4 d[NJ], xh[NJ], o[NJ];
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            d[j] = __ldcs(d4 + lane + 32 * j);
            xh[j] = __ldcs(x4 + lane + 32 * j);
            o[j] = __ldcs(o4 + lane + 32 * j);
        }
        const float m = mean[t], rs = rstd[t];
        float s1 = 0.f, s2 = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            xh[j] = make_float4((xh[j].x - m) * rs, (xh[j].y - m) * rs, (xh[j].z - m) * rs, (xh[j].w - m) * rs);
            const float4 wj = __ldg(wv + lane + 32 * j);
            const float4 dn = make_float4(d[j].x * wj.x, d[j].y * wj.y, d[j].z * wj.z, d[j].w * wj.w);
            s1 += (dn.x + dn.y) + (dn.z + dn.w);
            s2 += (dn.x * xh[j].x + dn.y * xh[j].y) + (dn.z * xh[j].z + dn.w * xh[j].w);
        }
        s1 = warp_sum(s1) * invC;
        s2 = warp_sum(s2) * invC;
#pragma unroll
        for (int j = 0; j < NJ; ++j) {
            const float4 dv = d[j], xv = xh[j], wj = __ldg(wv + lane + 32 * j);
            float4 n = o[j];
            n.x += rs * (dv.x * wj.x - s1 - xv.x * s2);
            n.y += rs * (dv.y * wj.y - s1 - xv.y * s2);
            n.z += rs * (dv.z * wj.z - s1 - xv.z * s2);
            n.w += rs * (dv.w * wj.w - s1 - xv.w * s2);
            __stcs(o4 + lane + 32 * j, n);
            float4 &pw = my[lane + 32 * j], &pb = my[C / 4 + lane + 32 * j];
            pw.x += dv.x * xv.x; pw.y += dv.y * xv.y; pw.z += dv.z * xv.z; pw.w += dv.w * xv.w;
            pb.x += dv.x; pb.y += dv.y; pb.z += dv.z; pb.w += dv.w;
            if (want_cs) {
                float4 &pc = my[2 * (C / 4) + lane + 32 * j];
                pc.x += n.x; pc.y += n.y; pc.z += n.z; pc.w += n.w;
            }
        }
    }
    __syncthreads();
    const float *spf = (const float *)ln_sp;
    for (int c = threadIdx.x; c < 3 * C; c += blockDim.x) {
        float v = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) v += spf[k * 3 * C + c];
        part[(long)blockIdx.x * 3 * C + c] = v;
    }
}

// dw, db (and cs) += the blocks' partials part[nb][3][C]: one block per 32 of
// the 3C sums, lane = sum, warp w adds the partials of blocks w, w + 16, ...
// in order, then the 16 warp totals are added in warp order (fixed order).
__global__ void __launch_bounds__(512)
ln_bwd_part_reduce(const float *__restrict__ part, int nb, int C, float *__restrict__ dw, float *__restrict__ db,
                   float *__restrict__ cs) {
    __shared__ float red[16][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int j = blockIdx.x * 32 + lane;  // index into [3][C]
    float v = 0.f;
    if (j < 3 * C)
#pragma unroll 4
        for (int b = warp; b < nb; b += 16) v += part[(long)b * 3 * C + j];
    red[warp][lane] = v;
    __syncthreads();
    if (warp == 0 && j < 3 * C) {
        float t = 0.f;
#pragma unroll
        for (int w = 0; w < 16; ++w) t += red[w][lane];
        const int k = j / C, c = j - k * C;  // 0: dw, 1: db, 2: cs
        float *dst = k == 0 ? dw : (k == 1 ? db : cs);
        if (dst) dst[c] += t;
    }
}

// ---------------------------------------------------------------- GELU
__global__ void gelu_fwd_kernel(const float *__restrict__ x, float *__restrict__ out, long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        out[i] = gelu_tanh(x[i]);
}

__global__ void gelu_bwd_kernel(const float *__restrict__ dout, const float *__restrict__ x,
                                float *__restrict__ dx, long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        dx[i] += dout[i] * gelu_tanh_grad(x[i]);
}

// ---------------------------------------------------------------- softmax
// One block per row: max, sum of exp, normalise (src/ops.c:464-480).
__device__ __forceinline__ float block_reduce(float v, bool is_max, float *sh) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = is_max ? warp_max(v) : warp_sum(v);
    __syncthreads();
    if (lane == 0) sh[wid] = v;
    __syncthreads();
    float r = lane < nw ? sh[lane] : (is_max ? -INFINITY : 0.f);
    r = is_max ? warp_max(r) : warp_sum(r);
    return r;
}

__global__ void softmax_rows_kernel(float *__restrict__ x, int cols) {
    __shared__ float sh[32];
    float *row = x + (long)blockIdx.x * cols;
    float mx = -INFINITY;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) mx = fmaxf(mx, row[c]);
    mx = block_reduce(mx, true, sh);
    float s = 0.f;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) {
        float e = expf(row[c] - mx);
        row[c] = e;
        s += e;
    }
    s = block_reduce(s, false, sh);
    const float inv = 1.0f / s;
    for (int c = threadIdx.x; c < cols; c += blockDim.x) row[c] *= inv;
}

__global__ void causal_mask_kernel(float *__restrict__ s, int T) {
    const long n = (long)T * T;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const long r = i / T, c = i % T;
        if (c > r) s[i] = -1e9f;
    }
}

// ---------------------------------------------------------------- cross-entropy
// (max, sum exp(x - max)) pairs, merged with rescaling (online softmax)
__device__ __forceinline__ void ms_merge(float &m, float &sum, float m2, float s2) {
    if (m2 == -INFINITY) return;
    if (m == -INFINITY) { m = m2; sum = s2; return; }
    if (m2 > m) { sum = sum * expf(m - m2) + s2; m = m2; }
    else sum += s2 * expf(m2 - m);
}

// One block per row of logits [rows, V] (pitch ldl). One pass computes the
// row max and sum of exp(x - max) together; a second writes probs (optional,
// pitch ldp) and dlogits = scale * (probs - onehot) (optional, pitch ldd, pad
// columns [V, ldd) zeroed), and the row's NLL term (l[tgt] - max) - log(sum)
// goes to rowterm[row] (src/ops.c:551-570). The block reduction has a fixed
// shape, so the result is deterministic.
__global__ void __launch_bounds__(512)
ce_fwd_kernel(const float *__restrict__ logits, long ldl, const int *__restrict__ targets,
              float *__restrict__ probs, long ldp, float *__restrict__ dlogits, long ldd,
              float scale, float *__restrict__ rowterm, int V) {
    // Each thread handles columns v = tid + 512 u in groups of CE_U, loading a
    // whole group before using it so that CE_U loads per thread are in flight
    // (the rows are HBM-resident and their pitch V is odd, so no float4).
    constexpr int CE_U = 8, NT = 512;
    __shared__ float shm[16], shs[16];
    const long r = blockIdx.x;
    const float *lg = logits + r * ldl;
    float m = -INFINITY, sum = 0.f;
    for (int v0 = threadIdx.x; v0 < V; v0 += NT * CE_U) {
        float x[CE_U];
#pragma unroll
        for (int u = 0; u < CE_U; ++u) {
            const int v = v0 + u * NT;
            x[u] = v < V ? __ldcs(lg + v) : -INFINITY;
        }
        float mx = x[0];
#pragma unroll
        for (int u = 1; u < CE_U; ++u) mx = fmaxf(mx, x[u]);
        if (mx == -INFINITY) continue;
        const float mn = fmaxf(m, mx);
        float add = 0.f;
#pragma unroll
        for (int u = 0; u < CE_U; ++u) add += expf(x[u] - mn);
        sum = (m == -INFINITY ? 0.f : sum * expf(m - mn)) + add;
        m = mn;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, sum, o);
        ms_merge(m, sum, m2, s2);
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) { shm[wid] = m; shs[wid] = sum; }
    __syncthreads();
    m = shm[0];
    sum = shs[0];
    for (int k = 1; k < nw; ++k) ms_merge(m, sum, shm[k], shs[k]);
    const float inv = 1.0f / sum;
    const int tgt = targets ? targets[r] : -1;
    if (probs || dlogits) {
        float *pr = probs ? probs + r * ldp : nullptr;
        float *dl = dlogits ? dlogits + r * ldd : nullptr;
        for (int v0 = threadIdx.x; v0 < V; v0 += NT * CE_U) {
            float x[CE_U];
#pragma unroll
            for (int u = 0; u < CE_U; ++u) {
                const int v = v0 + u * NT;
                x[u] = v < V ? __ldcs(lg + v) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < CE_U; ++u) {
                const int v = v0 + u * NT;
                if (v < V) {
                    const float p = expf(x[u] - m) * inv;
                    if (pr) __stcs(pr + v, p);
                    if (dl) __stcs(dl + v, scale * (p - (v == tgt ? 1.0f : 0.0f)));
                }
            }
        }
        if (dl)
            for (long v = V + threadIdx.x; v < ldd; v += blockDim.x) dl[v] = 0.f;
    }
    if (threadIdx.x == 0 && rowterm) rowterm[r] = tgt >= 0 ? (lg[tgt] - m) - logf(sum) : 0.f;
}

// Fused cross-entropy, second half (the LM-head GEMM's epilogue formed the
// per-64-column (max, sum exp) pairs of every logits row): one block per row
// merges the row's pairs in a fixed order into (max, sum), keeps the row's
// NLL term (l[tgt] - max) - log(sum) (src/ops.c:551-570), then overwrites the
// logits row in place with dlogits = scale * (softmax - onehot)
// (src/ops.c:576-590 into the zeroed buffer of src/model.c:644), pad columns
// [V, ldd) zeroed. Rows are 16-byte aligned (ldd % 4 == 0).
__global__ void __launch_bounds__(512)
ce_fused_rows_kernel(float *__restrict__ rows_io, long ldd, const float2 *__restrict__ part, int ce_ld,
                     const int *__restrict__ targets, float scale, float *__restrict__ rowterm, int V) {
    constexpr int NT = 512;
    __shared__ float shm[16], shs[16];
    const long r = blockIdx.x;
    float m = -INFINITY, sum = 0.f;
    for (int g = threadIdx.x; g < ce_ld; g += NT) {
        const float2 p = part[r * ce_ld + g];
        ms_merge(m, sum, p.x, p.y);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o), s2 = __shfl_xor_sync(0xffffffffu, sum, o);
        ms_merge(m, sum, m2, s2);
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) { shm[wid] = m; shs[wid] = sum; }
    __syncthreads();
    m = shm[0];
    sum = shs[0];
    for (int k = 1; k < NT / 32; ++k) ms_merge(m, sum, shm[k], shs[k]);
    float *row = rows_io + r * ldd;
    const int tgt = targets[r];
    if (threadIdx.x == 0) rowterm[r] = (row[tgt] - m) - logf(sum);
    __syncthreads();  // the target's logit is read before the row is overwritten
    const float inv = 1.0f / sum;
    float4 *row4 = (float4 *)row;
    const int n4 = (int)(ldd >> 2);
    for (int i = threadIdx.x; i < n4; i += NT) {
        const float4 x = __ldcs(row4 + i);
        const float xv[4] = {x.x, x.y, x.z, x.w};
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int v = 4 * i + j;
            o[j] = v < V ? scale * (expf(xv[j] - m) * inv - (v == tgt ? 1.0f : 0.0f)) : 0.0f;
        }
        __stcs(row4 + i, make_float4(o[0], o[1], o[2], o[3]));
    }
}

// loss = -(sum of the row terms) / rows: 1024 threads each sum a fixed
// strided subset, then a fixed-shape tree (deterministic; the reference sums
// in row order in one float, src/ops.c:503,548,573).
__global__ void __launch_bounds__(1024) ce_loss_kernel(const float *__restrict__ rowterm, int rows,
                                                       float *__restrict__ loss) {
    __shared__ float sh[1024];
    float acc = 0.f;
    for (int r = threadIdx.x; r < rows; r += 1024) acc += rowterm[r];
    sh[threadIdx.x] = acc;
    __syncthreads();
    for (int w = 512; w > 0; w >>= 1) {
        if ((int)threadIdx.x < w) sh[threadIdx.x] += sh[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) *loss = -sh[0] / (float)rows;
}

__global__ void ce_bwd_kernel(float *__restrict__ dlogits, const float *__restrict__ probs,
                              const int *__restrict__ targets, float scale, int rows, int V) {
    const long n = (long)rows * V;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const long r = i / V;
        const int v = (int)(i % V);
        dlogits[i] += scale * (probs[i] - (v == targets[r] ? 1.0f : 0.0f));
    }
}

// dlogits[r, v] = scale * (probs[r, v] - onehot) with pitch ldd (pad zeroed):
// the reference's calloc + cross_entropy_bwd (src/model.c:644,665).
__global__ void ce_grad_kernel(const float *__restrict__ probs, long ldp, const int *__restrict__ targets,
                               float scale, float *__restrict__ dl, long ldd, int V) {
    const long r = blockIdx.x;
    const int tgt = targets[r];
    for (long v = threadIdx.x; v < ldd; v += blockDim.x)
        dl[r * ldd + v] = v < V ? scale * (probs[r * ldp + v] - (v == tgt ? 1.0f : 0.0f)) : 0.0f;
}

// kc[b, pos0 + t, :] = qkv[b*T + t, C:2C], vc likewise from [2C:3C]
__global__ void kv_append_kernel(const float *__restrict__ qkv, float *__restrict__ kc,
                                 float *__restrict__ vc, int B, int T, long Tmax, int pos0, int C,
                                 const int *__restrict__ pos_dev) {
    if (pos_dev) pos0 += *pos_dev;
    const long n = (long)B * T * C;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const long r = i / C;
        const int c = (int)(i % C), b = (int)(r / T), t = (int)(r % T);
        const float *src = qkv + r * 3L * C;
        const long dst = ((long)b * Tmax + pos0 + t) * C + c;
        kc[dst] = src[C + c];
        vc[dst] = src[2 * C + c];
    }
}

// dst[b, :] = src[b*T + T-1, :]
__global__ void gather_last_kernel(const float *__restrict__ src, float *__restrict__ dst, int B, int T,
                                   int C) {
    const long n = (long)B * C;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const long b = i / C;
        const int c = (int)(i % C);
        dst[i] = src[(b * T + T - 1) * C + c];
    }
}

// ---------------------------------------------------------------- misc
__global__ void axpy_kernel(float *__restrict__ dst, const float *__restrict__ src, long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        dst[i] += src[i];
}

__global__ void add3_kernel(float *__restrict__ dst, const float *__restrict__ a,
                            const float *__restrict__ b, long n) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        dst[i] = a[i] + b[i];
}

__global__ void scale_kernel(float *__restrict__ x, long n, const float *__restrict__ sp, float s) {
    const float f = sp ? *sp : s;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        x[i] *= f;
}

__global__ void mask_mul_kernel(float *__restrict__ x, const unsigned char *__restrict__ mask,
                                long n, float scale) {
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        x[i] *= mask[i] ? scale : 0.0f;
}

// sum of squares, double accumulation: per-block partials then a fixed-order
// final pass.
__global__ void sumsq_partial_kernel(const float *__restrict__ g, long n, double *__restrict__ part) {
    __shared__ double sh[32];
    double s = 0.0;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        s += (double)g[i] * (double)g[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < (int)(blockDim.x >> 5); ++k) t += sh[k];
        part[blockIdx.x] = t;
    }
}

// norm = sqrt(sum part); if clip > 0: factor = norm > clip ? clip / norm : 1
__global__ void norm_final_kernel(const double *__restrict__ part, int nparts, float *__restrict__ norm,
                                  float *__restrict__ clip_factor, float clip) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    double s = 0.0;
    for (int k = 0; k < nparts; ++k) s += part[k];
    const float nv = (float)sqrt(s);
    if (norm) *norm = nv;
    if (clip_factor) *clip_factor = (clip > 0.f && nv > clip) ? clip / nv : 1.0f;
}

// ---------------------------------------------------------------- embeddings
// emb[i] = wte[tok[i]] + wpe[i % T] (src/model.c:460-470)
__global__ void embed_fwd_kernel(const int *__restrict__ tok, const float *__restrict__ wte,
                                 const float *__restrict__ wpe, float *__restrict__ out, int BT,
                                 int T, int C, int pos0, const int *__restrict__ pos_dev) {
    if (pos_dev) pos0 += *pos_dev;
    const long n = (long)BT * C;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const long r = i / C;
        const int c = (int)(i % C);
        const int t = (int)(r % T) + pos0;
        out[i] = wte[(long)tok[r] * C + c] + wpe[(long)t * C + c];
    }
}

// d_wpe[t] += sum_b dx[b, t] in b order (src/model.c:853-857)
__global__ void embed_bwd_wpe_kernel(const float *__restrict__ dx, float *__restrict__ dwpe, int B,
                                     int T, int C) {
    const long n = (long)T * C;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        float acc = dwpe[i];
        for (int b = 0; b < B; ++b) acc += dx[(long)b * n + i];
        dwpe[i] = acc;
    }
}

// d_wte[tok[i]] += dx[i], positions applied in increasing i as in
// src/model.c:861-867. One warp per position; a position whose token occurs
// earlier is skipped, the first occurrence ("leader") accumulates all later
// occurrences in order into registers. Tokens are staged in shared memory.
template <int CPL>
__global__ void __launch_bounds__(256)
embed_bwd_wte_kernel(const int *__restrict__ tok, const float *__restrict__ dx,
                     float *__restrict__ dwte, int BT, int C) {
    extern __shared__ int stok[];
    for (int i = threadIdx.x; i < BT; i += blockDim.x) stok[i] = tok[i];
    __syncthreads();
    const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
    for (int i = blockIdx.x * warps + (threadIdx.x >> 5); i < BT; i += gridDim.x * warps) {
        const int v = stok[i];
        bool leader = true;
        for (int base = 0; base < i; base += 32) {
            const int j = base + lane;
            if (__any_sync(0xffffffffu, j < i && stok[j] == v)) { leader = false; break; }
        }
        if (!leader) continue;
        float *row = dwte + (long)v * C;
        float acc[CPL];
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
            const int c = lane + 32 * q;
            acc[q] = c < C ? row[c] + dx[(long)i * C + c] : 0.f;
        }
        for (int base = i + 1; base < BT; base += 32) {
            const int j = base + lane;
            unsigned mk = __ballot_sync(0xffffffffu, j < BT && stok[j] == v);
            while (mk) {
                const int jj = base + __ffs(mk) - 1;
                mk &= mk - 1;
#pragma unroll
                for (int q = 0; q < CPL; ++q) {
                    const int c = lane + 32 * q;
                    if (c < C) acc[q] += dx[(long)jj * C + c];
                }
            }
        }
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
            const int c = lane + 32 * q;
            if (c < C) row[c] = acc[q];
        }
    }
}

// ---------------------------------------------------------------- AdamW
// One fused pass (src/model.c:901-920): grads are first multiplied by the
// clip factor computed on the device (identity when no clipping applies).
// Four parameters per thread per iteration (16-byte loads and stores).
__device__ __forceinline__ void adamw_one(float &p, float &g, float &m, float &v, unsigned char d,
                                          float cf, bool scale, float lr, float b1, float b2,
                                          float eps, float wd, float bc1, float bc2) {
    if (scale) g *= cf;
    m = b1 * m + (1.0f - b1) * g;
    v = b2 * v + (1.0f - b2) * g * g;
    const float mh = m / bc1, vh = v / bc2;
    const float ewd = d ? wd : 0.0f;
    p = p * (1.0f - lr * ewd) - lr * mh / (sqrtf(vh) + eps);
}

__global__ void adamw_kernel(float *__restrict__ p, float *__restrict__ g, float *__restrict__ m,
                             float *__restrict__ v, const unsigned char *__restrict__ decay, long n,
                             const float *__restrict__ clip_factor, float lr, float b1, float b2,
                             float eps, float wd, float bc1, float bc2) {
    const float cf = clip_factor ? *clip_factor : 1.0f;
    const bool scale = cf != 1.0f;
    const long n4 = n / 4;
    const long stride = (long)gridDim.x * blockDim.x;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 P = ((float4 *)p)[i], G = ((float4 *)g)[i], Mm = ((float4 *)m)[i], Vv = ((float4 *)v)[i];
        const uchar4 D = ((const uchar4 *)decay)[i];
        adamw_one(P.x, G.x, Mm.x, Vv.x, D.x, cf, scale, lr, b1, b2, eps, wd, bc1, bc2);
        adamw_one(P.y, G.y, Mm.y, Vv.y, D.y, cf, scale, lr, b1, b2, eps, wd, bc1, bc2);
        adamw_one(P.z, G.z, Mm.z, Vv.z, D.z, cf, scale, lr, b1, b2, eps, wd, bc1, bc2);
        adamw_one(P.w, G.w, Mm.w, Vv.w, D.w, cf, scale, lr, b1, b2, eps, wd, bc1, bc2);
        ((float4 *)p)[i] = P;
        if (scale) ((float4 *)g)[i] = G;
        ((float4 *)m)[i] = Mm;
        ((float4 *)v)[i] = Vv;
    }
    for (long i = n4 * 4 + blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += stride) {
        float pp = p[i], gg = g[i], mm = m[i], vv = v[i];
        adamw_one(pp, gg, mm, vv, decay[i], cf, scale, lr, b1, b2, eps, wd, bc1, bc2);
        p[i] = pp;
        g[i] = gg;
        m[i] = mm;
        v[i] = vv;
    }
}

// ---------------------------------------------------------------- column sums
// db[n] += sum_m dY[m, n]: row-chunk partials then an in-order final pass.
__global__ void colsum_partial_kernel(const float *__restrict__ y, long ldy, int M, int N,
                                      int rows_per_chunk, float *__restrict__ part) {
    const int n = blockIdx.x * blockDim.x + threadIdx.x;
    if (n >= N) return;
    const long r0 = (long)blockIdx.y * rows_per_chunk;
    const long r1 = std::min<long>(M, r0 + rows_per_chunk);
    float s = 0.f;
#pragma unroll 8
    for (long r = r0; r < r1; ++r) s += y[r * ldy + n];
    part[(long)blockIdx.y * N + n] = s;
}

// db[n] += sum of the chunk partials, in chunk order per warp: one block per
// 32 columns, warp w sums chunks k = w, w+8, ... and the 8 warp sums are
// added in warp order (fixed shape, deterministic)
__global__ void __launch_bounds__(256) colsum_final_kernel(const float *__restrict__ part, int chunks, int N,
                                                           float *__restrict__ db) {
    __shared__ float red[8][32];
    const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31, n = blockIdx.x * 32 + lane;
    float s = 0.f;
    if (n < N)
        for (int k = wid; k < chunks; k += 8) s += part[(long)k * N + n];
    red[wid][lane] = s;
    __syncthreads();
    if (wid == 0 && n < N) {
        float t = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) t += red[k][lane];
        db[n] += t;
    }
}

// ---------------------------------------------------------------- argmax
// Greedy token per row: largest logit, lowest index on ties (the first index
// whose CDF exceeds r in src/model.c:982-985 with top_k = 1).
__global__ void argmax_kernel(const float *__restrict__ x, long ldx, int V, int *__restrict__ out,
                              float *__restrict__ outval, int *__restrict__ log,
                              const int *__restrict__ step_dev) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const float *row = x + (long)blockIdx.x * ldx;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const float f = row[v];
        if (f > best) { best = f; bi = v; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float f = __shfl_xor_sync(0xffffffffu, best, o);
        const int j = __shfl_xor_sync(0xffffffffu, bi, o);
        if (f > best || (f == best && j < bi)) { best = f; bi = j; }
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) { sv[wid] = best; si[wid] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int k = 1; k < (int)(blockDim.x >> 5); ++k)
            if (sv[k] > best || (sv[k] == best && si[k] < bi)) { best = sv[k]; bi = si[k]; }
        out[blockIdx.x] = bi;
        if (outval) outval[blockIdx.x] = best;
        if (log) log[(long)(*step_dev) * gridDim.x + blockIdx.x] = bi;
    }
}

__device__ __forceinline__ unsigned long long greedy_key(float v, int col) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)col);
}

__global__ void argmax_keys_kernel(const float *__restrict__ x, long ldx, int V, unsigned long long *keys) {
    __shared__ unsigned long long sk[32];
    const float *row = x + (long)blockIdx.x * ldx;
    unsigned long long best = 0;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
        const unsigned long long k = greedy_key(row[v], v);
        best = k > best ? k : best;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
        best = k > best ? k : best;
    }
    if ((threadIdx.x & 31) == 0) sk[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) best = sk[w] > best ? sk[w] : best;
        atomicMax(keys + blockIdx.x, best);
    }
}

__global__ void greedy_finalize_kernel(unsigned long long *keys, int rows, int *next, int *log, const int *step,
                                       int *pair, int *ctr) {
    const int t = threadIdx.x;
    if (t < rows) {
        const unsigned long long k = keys[t];
        keys[t] = 0ull;
        const uint32_t ord = (uint32_t)(k >> 32);
        const int col = (int)(0xFFFFFFFFu - (uint32_t)k);
        const uint32_t u = (ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord;
        if (next) next[t] = col;
        if (log) log[(long)(*step) * rows + t] = col;
        if (pair) {
            pair[t] = (int)u;
            pair[rows + t] = col;
        }
    }
    __syncthreads();
    if (ctr && t == 0) {
        ctr[0] += 1;
        ctr[1] += 1;
    }
}

}  // namespace

// ========================================================== launchers

#define LAUNCH_CHECK() do { ++g_launch_count; CG_CUDA(cudaGetLastError()); } while (0)

int layernorm_fwd(const float *x, long ldx, const float *w, const float *b, float *out, long ldo,
                  float *mean, float *rstd, int T, int C, cudaStream_t s) {
    if (T <= 0) return OK;
    const int warps = 8;
    const uintptr_t al = (uintptr_t)x | (uintptr_t)w | (uintptr_t)b | (uintptr_t)out;
    if (C % 128 == 0 && C <= 1024 && ldx % 4 == 0 && ldo % 4 == 0 && al % 16 == 0) {
        const int g = grid_for(T, warps, 148 * 8);
        switch (C / 128) {
#define LNF4(N) case N: layernorm_fwd4_kernel<N><<<g, warps * 32, 0, s>>>(x, ldx, w, b, out, ldo, mean, rstd, T); break;
            LNF4(1) LNF4(2) LNF4(3) LNF4(4) LNF4(5) LNF4(6) LNF4(7) LNF4(8)
#undef LNF4
        }
        LAUNCH_CHECK();
        return OK;
    }
    layernorm_fwd_kernel<<<grid_for(T, warps, 148 * 8), warps * 32, 0, s>>>(x, ldx, w, b, out, ldo,
                                                                           mean, rstd, T, C);
    LAUNCH_CHECK();
    return OK;
}

constexpr int kLnBwdRowsPerChunk = 128;

// Rows per dw/db partial chunk: the requested count, raised where needed so
// that the chunks fit the grid's y dimension (65535).
static int ln_bwd_chunk_rows(int T, int rows_per_chunk) {
    if (rows_per_chunk <= 0) rows_per_chunk = kLnBwdRowsPerChunk;
    const int min_rows = (int)(((long)T + 65534) / 65535);
    return std::max(rows_per_chunk, min_rows);
}

size_t layernorm_bwd_scratch_bytes(int T, int C, int rows_per_chunk) {
    rows_per_chunk = ln_bwd_chunk_rows(T, rows_per_chunk);
    const long chunks = ((long)T + rows_per_chunk - 1) / rows_per_chunk;
    return (size_t)chunks * 2 * C * sizeof(float);
}

size_t layernorm_bwd_scratch_bytes(int T, int C) { return layernorm_bwd_scratch_bytes(T, C, kLnBwdRowsPerChunk); }

int layernorm_bwd(const float *dout, const float *x, const float *w, const float *mean, const float *rstd,
                  float *dx, float *dw, float *db, int T, int C, float *scratch, cudaStream_t s,
                  int rows_per_chunk) {
    if (T <= 0) return OK;
    rows_per_chunk = ln_bwd_chunk_rows(T, rows_per_chunk);
    layernorm_bwd_dx_kernel<<<grid_for(T, 8, 148 * 16), 256, 0, s>>>(dout, x, w, mean, rstd, dx, T, C);
    LAUNCH_CHECK();
    const int chunks = (int)(((long)T + rows_per_chunk - 1) / rows_per_chunk);
    dim3 g((C + 255) / 256, chunks);
    layernorm_bwd_dwdb_kernel<<<g, 256, 0, s>>>(dout, x, mean, rstd, scratch, T, C, rows_per_chunk);
    LAUNCH_CHECK();
    layernorm_bwd_reduce<<<(C + 31) / 32, 256, 0, s>>>(scratch, chunks, C, dw, db);
    LAUNCH_CHECK();
    return OK;
}

int layernorm_bwd(const float *dout, const float *x, const float *w, const float *mean,
                  const float *rstd, float *dx, float *dw, float *db, int T, int C, float *scratch,
                  cudaStream_t s) {
    return layernorm_bwd(dout, x, w, mean, rstd, dx, dw, db, T, C, scratch, s, kLnBwdRowsPerChunk);
}

namespace {
int ln_bwd_fused_blocks(int T) { return std::max(1, std::min((T + 7) / 8, 148 * 2)); }

template <int NJ>
int launch_ln_bwd_fused(const float *dout, const float *x, const float *w, const float *mean, const float *rstd,
                        float *dx, int T, int nb, int rpb, float *part, bool want_cs, cudaStream_t s) {
    constexpr int smem = 8 * 3 * 128 * NJ * 4;
    static bool attr = false;
    if (!attr) {
        CG_CUDA(cudaFuncSetAttribute(ln_bwd_fused_kernel<NJ>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        attr = true;
    }
    ln_bwd_fused_kernel<NJ><<<nb, 256, smem, s>>>(dout, x, w, mean, rstd, dx, T, rpb, part, want_cs ? 1 : 0);
    LAUNCH_CHECK();
    return OK;
}
}  // namespace

bool layernorm_bwd_fused_ok(int C, const void *dout, const void *x, const void *w, const void *dx) {
    const uintptr_t a = (uintptr_t)dout | (uintptr_t)x | (uintptr_t)w | (uintptr_t)dx;
    return C > 0 && C % 128 == 0 && C <= 1024 && (a % 16) == 0;
}

size_t layernorm_bwd_fused_scratch_bytes(int T, int C) {
    return (size_t)ln_bwd_fused_blocks(T) * 3 * C * sizeof(float);
}

int layernorm_bwd_fused(const float *dout, const float *x, const float *w, const float *mean, const float *rstd,
                        float *dx, float *dw, float *db, float *cs, int T, int C, float *scratch, cudaStream_t s) {
    if (T <= 0) return OK;
    if (!layernorm_bwd_fused_ok(C, dout, x, w, dx)) {
        set_last_error(ERR_ARG, "layernorm_bwd_fused: C=%d needs C %% 128 == 0, C <= 1024, aligned rows", C);
        return ERR_ARG;
    }
    const int nb = ln_bwd_fused_blocks(T), rpb = (T + nb - 1) / nb;
    switch (C / 128) {
        case 1: CG_TRY(launch_ln_bwd_fused<1>(dout, x, w, mean, rstd, dx, T, nb, rpb, scratch, cs, s)); break;
        case 2: CG_TRY(launch_ln_bwd_fused<2>(dout, x, w, mean, rstd, dx, T, nb, rpb, scratch, cs, s)); break;
        case 3: CG_TRY(launch_ln_bwd_fused<3>(dout, x, w, mean, rstd, dx, T, nb, rpb, scratch, cs, s)); break;
        case 4: CG_TRY(launch_ln_bwd_fused<4>(dout, x, w, mean, rstd, dx, T, nb, rpb, scratch, cs, s)); break;
        case 5: CG_TRY(launch_ln_bwd_fused<5>(dout, x, w, mean, rstd, dx, T, nb, rpb, scratch, cs, s)); break;
        case 6: CG_TRY(launch_ln_bwd_fused<6>(dout, x, w, mean, rstd, dx, T, nb, rpb, scratch, cs, s)); break;
        case 7: CG_TRY(launch_ln_bwd_fused<7>(dout, x, w, mean, rstd, dx, T, nb, rpb, scratch, cs, s)); break;
        default: CG_TRY(launch_ln_bwd_fused<8>(dout, x, w, mean, rstd, dx, T, nb, rpb, scratch, cs, s)); break;
    }
    ln_bwd_part_reduce<<<(3 * C + 31) / 32, 512, 0, s>>>(scratch, nb, C, dw, db, cs);
    LAUNCH_CHECK();
    return OK;
}

int gelu_fwd(const float *x, float *out, long n, cudaStream_t s) {
    if (n <= 0) return OK;
    gelu_fwd_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, out, n);
    LAUNCH_CHECK();
    return OK;
}

int gelu_bwd(const float *dout, const float *x, float *dx, long n, cudaStream_t s) {
    if (n <= 0) return OK;
    gelu_bwd_kernel<<<grid_for(n, 256), 256, 0, s>>>(dout, x, dx, n);
    LAUNCH_CHECK();
    return OK;
}

int softmax_rows(float *x, int rows, int cols, cudaStream_t s) {
    if (rows <= 0 || cols <= 0) return OK;
    const int th = cols >= 1024 ? 512 : (cols >= 128 ? 128 : 32);
    softmax_rows_kernel<<<rows, th, 0, s>>>(x, cols);
    LAUNCH_CHECK();
    return OK;
}

int causal_mask(float *scores, int T, cudaStream_t s) {
    if (T <= 1) return OK;
    causal_mask_kernel<<<grid_for((long)T * T, 256), 256, 0, s>>>(scores, T);
    LAUNCH_CHECK();
    return OK;
}

int cross_entropy_rows(const float *logits, long ldl, const int *targets, float *probs, long ldp,
                       float *dlogits, long ldd, float scale, float *rowterm, int rows, int V,
                       cudaStream_t s) {
    if (rows <= 0) return OK;
    ce_fwd_kernel<<<rows, 512, 0, s>>>(logits, ldl, targets, probs, ldp, dlogits, ldd, scale,
                                       rowterm, V);
    LAUNCH_CHECK();
    return OK;
}

int cross_entropy_fused(float *rows_io, long ldd, const float2 *part, int ce_ld, const int *targets, float scale,
                        float *rowterm, int rows, int V, cudaStream_t s) {
    if (rows <= 0) return OK;
    if (ldd % 4 != 0 || ((uintptr_t)rows_io % 16) != 0 || ldd < V) {
        set_last_error(ERR_ARG, "cross_entropy_fused: rows need a 16-byte aligned pitch >= V");
        return ERR_ARG;
    }
    ce_fused_rows_kernel<<<rows, 512, 0, s>>>(rows_io, ldd, part, ce_ld, targets, scale, rowterm, V);
    LAUNCH_CHECK();
    return OK;
}

int cross_entropy_loss(const float *rowterm, int rows, float *loss, cudaStream_t s) {
    ce_loss_kernel<<<1, 1024, 0, s>>>(rowterm, rows, loss);
    LAUNCH_CHECK();
    return OK;
}

int cross_entropy_bwd(float *dlogits, const float *probs, const int *targets, float scale, int rows,
                      int V, cudaStream_t s) {
    if (rows <= 0) return OK;
    ce_bwd_kernel<<<grid_for((long)rows * V, 256), 256, 0, s>>>(dlogits, probs, targets, scale, rows, V);
    LAUNCH_CHECK();
    return OK;
}

int axpy1(float *dst, const float *src, long n, cudaStream_t s) {
    if (n <= 0) return OK;
    axpy_kernel<<<grid_for(n, 256), 256, 0, s>>>(dst, src, n);
    LAUNCH_CHECK();
    return OK;
}

int add3(float *dst, const float *a, const float *b, long n, cudaStream_t s) {
    if (n <= 0) return OK;
    add3_kernel<<<grid_for(n, 256), 256, 0, s>>>(dst, a, b, n);
    LAUNCH_CHECK();
    return OK;
}

int scale(float *x, long n, const float *dev_factor, float factor, cudaStream_t s) {
    if (n <= 0) return OK;
    scale_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, n, dev_factor, factor);
    LAUNCH_CHECK();
    return OK;
}

int mask_mul(float *x, const unsigned char *mask, long n, float sc, cudaStream_t s) {
    if (n <= 0) return OK;
    mask_mul_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, mask, n, sc);
    LAUNCH_CHECK();
    return OK;
}

size_t norm_scratch_bytes() { return 1024 * sizeof(double); }

int grad_norm(const float *g, long n, double *scratch, float *norm, float *clip_factor, float clip,
              cudaStream_t s) {
    const int nb = std::max(1, std::min(1024, (int)((n + 255) / 256)));
    sumsq_partial_kernel<<<nb, 256, 0, s>>>(g, n, scratch);
    LAUNCH_CHECK();
    norm_final_kernel<<<1, 32, 0, s>>>(scratch, nb, norm, clip_factor, clip);
    LAUNCH_CHECK();
    return OK;
}

int embed_fwd(const int *tok, const float *wte, const float *wpe, float *out, int BT, int T, int C,
              int pos0, cudaStream_t s) {
    if (BT <= 0) return OK;
    embed_fwd_kernel<<<grid_for((long)BT * C, 256), 256, 0, s>>>(tok, wte, wpe, out, BT, T, C, pos0,
                                                                 nullptr);
    LAUNCH_CHECK();
    return OK;
}

int embed_bwd(const int *tok, const float *dx, float *dwte, float *dwpe, int B, int T, int C,
              cudaStream_t s) {
    const int BT = B * T;
    if (BT <= 0) return OK;
    embed_bwd_wpe_kernel<<<grid_for((long)T * C, 256), 256, 0, s>>>(dx, dwpe, B, T, C);
    LAUNCH_CHECK();
    const size_t sm = (size_t)BT * sizeof(int);
    if (sm > 200 * 1024) {
        set_last_error(ERR_ARG, "embed_bwd: B*T=%d exceeds the staged-token limit", BT);
        return ERR_ARG;
    }
    if (C > 2048) {
        set_last_error(ERR_ARG, "embed_bwd: C=%d > 2048 unsupported", C);
        return ERR_ARG;
    }
    const int grid = std::min(num_sms() * 2, (BT + 7) / 8), cpl = (C + 31) / 32;
#define EBW(N)                                                                                \
    do {                                                                                      \
        static bool attr = false;                                                             \
        if (!attr) {                                                                          \
            CG_CUDA(cudaFuncSetAttribute(embed_bwd_wte_kernel<N>,                             \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, 204800)); \
            attr = true;                                                                      \
        }                                                                                     \
        embed_bwd_wte_kernel<N><<<grid, 256, sm, s>>>(tok, dx, dwte, BT, C);                  \
    } while (0)
    if (cpl <= 8) EBW(8);
    else if (cpl <= 16) EBW(16);
    else if (cpl <= 24) EBW(24);
    else if (cpl <= 32) EBW(32);
    else if (cpl <= 50) EBW(50);
    else EBW(64);
#undef EBW
    LAUNCH_CHECK();
    return OK;
}

int adamw(float *p, float *g, float *m, float *v, const unsigned char *decay, long n,
          const float *clip_factor, float lr, float b1, float b2, float eps, float wd, float bc1,
          float bc2, cudaStream_t s) {
    if (n <= 0) return OK;
    if (((uintptr_t)p | (uintptr_t)g | (uintptr_t)m | (uintptr_t)v) % 16 || (uintptr_t)decay % 4) {
        set_last_error(ERR_ARG, "adamw: arenas must be 16-byte aligned");
        return ERR_ARG;
    }
    adamw_kernel<<<grid_for(n / 4 + 1, 256, 148 * 16), 256, 0, s>>>(p, g, m, v, decay, n, clip_factor, lr, b1,
                                                            b2, eps, wd, bc1, bc2);
    LAUNCH_CHECK();
    return OK;
}

// 32-row chunks (at most 256): enough blocks to keep every SM's loads in
// flight; the chunk sums are added in chunk order
size_t colsum_scratch_bytes(int M, int N) {
    const int chunks = std::max(1, std::min(256, (M + 31) / 32));
    return (size_t)chunks * N * sizeof(float);
}

int colsum_add(const float *y, long ldy, int M, int N, float *db, float *scratch, cudaStream_t s) {
    if (M <= 0 || N <= 0) return OK;
    const int chunks = std::max(1, std::min(256, (M + 31) / 32));
    const int rpc = (M + chunks - 1) / chunks;
    dim3 g((N + 255) / 256, chunks);
    colsum_partial_kernel<<<g, 256, 0, s>>>(y, ldy, M, N, rpc, scratch);
    LAUNCH_CHECK();
    colsum_final_kernel<<<(N + 31) / 32, 256, 0, s>>>(scratch, chunks, N, db);
    LAUNCH_CHECK();
    return OK;
}

int ce_grad(const float *probs, long ldp, const int *targets, float sc, float *dl, long ldd, int rows,
            int V, cudaStream_t s) {
    if (rows <= 0) return OK;
    ce_grad_kernel<<<rows, 512, 0, s>>>(probs, ldp, targets, sc, dl, ldd, V);
    LAUNCH_CHECK();
    return OK;
}

int kv_append(const float *qkv, float *kc, float *vc, int B, int T, long Tmax, int pos0, int C,
              cudaStream_t s) {
    if (B * T <= 0) return OK;
    kv_append_kernel<<<grid_for((long)B * T * C, 256), 256, 0, s>>>(qkv, kc, vc, B, T, Tmax, pos0, C,
                                                                    nullptr);
    LAUNCH_CHECK();
    return OK;
}

int gather_last(const float *src, float *dst, int B, int T, int C, cudaStream_t s) {
    if (B <= 0) return OK;
    gather_last_kernel<<<grid_for((long)B * C, 256), 256, 0, s>>>(src, dst, B, T, C);
    LAUNCH_CHECK();
    return OK;
}

// Decode-step variants: positions and the step index come from device
// counters ctr[0] (position of the incoming token) and ctr[1] (step), so one
// captured CUDA graph serves every step.
__global__ void decode_advance_kernel(int *ctr) {
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        ctr[0] += 1;
        ctr[1] += 1;
    }
}

int embed_fwd_at(const int *tok, const float *wte, const float *wpe, float *out, int B, int C,
                 const int *pos_dev, cudaStream_t s) {
    embed_fwd_kernel<<<grid_for((long)B * C, 256), 256, 0, s>>>(tok, wte, wpe, out, B, 1, C, 0, pos_dev);
    LAUNCH_CHECK();
    return OK;
}

int kv_append_at(const float *qkv, float *kc, float *vc, int B, long Tmax, int C, const int *pos_dev,
                 cudaStream_t s) {
    kv_append_kernel<<<grid_for((long)B * C, 256), 256, 0, s>>>(qkv, kc, vc, B, 1, Tmax, 0, C, pos_dev);
    LAUNCH_CHECK();
    return OK;
}

int argmax_log(const float *x, long ldx, int rows, int V, int *cur, int *log, const int *step_dev,
               cudaStream_t s) {
    argmax_kernel<<<rows, 512, 0, s>>>(x, ldx, V, cur, nullptr, log, step_dev);
    LAUNCH_CHECK();
    return OK;
}

int decode_advance(int *ctr, cudaStream_t s) {
    decode_advance_kernel<<<1, 32, 0, s>>>(ctr);
    LAUNCH_CHECK();
    return OK;
}

int argmax_rows(const float *x, long ldx, int rows, int V, int *out, float *outval, cudaStream_t s) {
    if (rows <= 0) return OK;
    argmax_kernel<<<rows, 512, 0, s>>>(x, ldx, V, out, outval, nullptr, nullptr);
    LAUNCH_CHECK();
    return OK;
}

int argmax_keys(const float *x, long ldx, int rows, int V, unsigned long long *keys, cudaStream_t s) {
    if (rows <= 0) return OK;
    argmax_keys_kernel<<<rows, 512, 0, s>>>(x, ldx, V, keys);
    LAUNCH_CHECK();
    return OK;
}

int greedy_finalize(unsigned long long *keys, int rows, int *next, int *log, const int *step, int *pair,
                    int *ctr, cudaStream_t s) {
    if (rows > 1024) {
        set_last_error(ERR_ARG, "greedy_finalize: %d rows", rows);
        return ERR_ARG;
    }
    greedy_finalize_kernel<<<1, rows < 32 ? 32 : ((rows + 31) / 32) * 32, 0, s>>>(keys, rows, next, log, step,
                                                                                   pair, ctr);
    LAUNCH_CHECK();
    return OK;
}

}  // namespace cg
