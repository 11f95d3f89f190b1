// decode_mk.cu - one greedy decode step of up to 8 sequences as a single
// persistent kernel.
//
// The decode step of src/fast.c:227-333 (one new row per sequence, K/V of the
// earlier positions from the cache) is a chain of small, HBM-bound products:
// per layer LN1 -> qkv -> attention over the cache -> c_proj + residual ->
// LN2 -> fc + GELU -> proj + residual, then LN_f -> LM head -> argmax. As
// separate kernels each link pays a launch ramp and a tail, which at batch 1
// costs as much as streaming the weights. Here one cooperative launch (one
// block per SM, all co-resident) runs every phase of the step and separates
// them with a grid barrier:
//
//   P1  every block normalises the rows (LN1) into shared memory; the blocks'
//       warps then take rows of c_attn_w (two at a time, lanes splitting K)
//       and append K and V to the cache at the current position
//   P2  attention: (sequence, head, 64-key chunk) items, two per block at a
//       time; the last chunk of a head merges the chunks in chunk order
//   P3  c_proj over the attention rows, residual added in place
//   P4  LN2, fc, GELU
//   P5  proj, residual added in place
//   P6  LN_f, LM head (logits written), row maxima folded into 64-bit keys
//       (value bits above the inverted column: ties go to the lowest column)
//   P7  block 0 turns the keys into the next tokens and advances the counters
//
// Before each barrier a block prefetches into L2 the weight rows it will
// stream in the next product, so the barrier's wait overlaps the HBM stream.
// Every barrier wait is bounded (the library's wait limit); a block that gives
// up records DEV_ERR_DECODE_BARRIER and raises an abort word that ends the
// other blocks' waits, and the step writes no token.
//
// The arithmetic is the GEMV path's (fp32 FMA, K split over lanes, fixed
// reduction order), so a step is deterministic.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>

#include "common.cuh"
#include "decode_mk.h"

namespace cg {

CG_DEV_ERROR_ACCESSORS(mk_take_dev_error, mk_set_wait_limit)

namespace {

constexpr int MK_THREADS = 512, MK_WARPS = MK_THREADS / 32;
constexpr int MK_KEYS = 64, MK_PART = 66;  // keys per attention chunk; partial = (max, sum, 64 outputs)

// ------------------------------------------------------------ grid barrier
// Monotone arrival counter (reset to 0 before each launch): the n-th barrier
// of the launch completes when the counter reaches n * gridDim.x.
__device__ __forceinline__ bool mk_barrier(unsigned long long *bar, int *abort, unsigned long long &target) {
    __shared__ int ok;
    __syncthreads();
    target += gridDim.x;
    if (threadIdx.x == 0) {
        ok = 1;
        // arrive: a release reduction at GPU scope (cumulative over the
        // block's writes ordered before it by the CTA barrier), no return value
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(bar) : "memory");
        const uint64_t t0 = globaltimer_ns();
        const uint64_t limit = *(volatile unsigned long long *)&g_cngpt_wait_limit_ns;
        for (unsigned it = 0;; ++it) {
            unsigned long long v;
            asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(bar) : "memory");
            if (v >= target) break;
            if ((it & 63u) == 63u) {
                if (*(volatile int *)abort) {
                    ok = 0;
                    break;
                }
                if (globaltimer_ns() - t0 > limit) {
                    record_error(DEV_ERR_DECODE_BARRIER);
                    atomicExch(abort, 1);
                    ok = 0;
                    break;
                }
            }
        }
    }
    __syncthreads();
    return ok != 0;
}

// ------------------------------------------------------------ row staging
// xs[m][k] = src[m][k] for m < B (global, read through L2: other blocks wrote
// it in the previous phase), normalised by LayerNorm when lnw is given (eps
// 1e-5, biased variance, two passes: src/ops.c:231-247).
template <int MT>
__device__ void mk_stage(float *xs, const float *src, long lds, int B, int K, const float *lnw, const float *lnb,
                         float *red) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, K4 = K >> 2;
    float4 *x4 = (float4 *)xs;
    for (int i = t; i < B * K4; i += MK_THREADS) {
        const int m = i / K4, k = i - m * K4;
        x4[i] = __ldcg((const float4 *)(src + (long)m * lds) + k);
    }
    if (!lnw) {
        __syncthreads();
        return;
    }
    __syncthreads();
    float mu[MT], rs[MT];
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
        float ps[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) ps[m] = 0.f;
        for (int k = t; k < K4; k += MK_THREADS) {
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m < B) {
                    const float4 v = x4[m * K4 + k];
                    if (pass == 0) {
                        ps[m] += (v.x + v.y) + (v.z + v.w);
                    } else {
                        const float a = v.x - mu[m], b = v.y - mu[m], c = v.z - mu[m], d = v.w - mu[m];
                        ps[m] += (a * a + b * b) + (c * c + d * d);
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const float v = warp_sum(ps[m]);
            if (lane == 0) red[warp * MT + m] = v;
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < MK_WARPS; ++w) v += red[w * MT + m];
            if (pass == 0) mu[m] = v / (float)K;
            else rs[m] = 1.0f / sqrtf(v / (float)K + 1e-5f);
        }
        __syncthreads();
    }
    for (int k = t; k < K4; k += MK_THREADS) {
        const float4 g = __ldg((const float4 *)lnw + k), b = __ldg((const float4 *)lnb + k);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m < B) {
                float4 v = x4[m * K4 + k];
                v.x = (v.x - mu[m]) * rs[m] * g.x + b.x;
                v.y = (v.y - mu[m]) * rs[m] * g.y + b.y;
                v.z = (v.z - mu[m]) * rs[m] * g.z + b.z;
                v.w = (v.w - mu[m]) * rs[m] * g.w + b.w;
                x4[m * K4 + k] = v;
            }
        }
    }
    __syncthreads();
}

// named barrier of the 128-thread group g of a block (ids 1..4)
__device__ __forceinline__ void group_sync(int g) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + g), "r"(128) : "memory");
}

// ------------------------------------------------------------ block GEMV
// Rows of W [N, K] (row pitch ldw) owned by this block: [lo, hi), R at a time.
// Each thread has R * KI 16-byte loads of W in flight before it multiplies;
// the R * MT partial sums are reduced across each warp by recursive halving
// and across the warps through shared memory in warp order (fixed order), and
// the epilogue gets (sequence m, row n, total).
template <int NV>
__device__ __forceinline__ void halve(float *a, int lane, int o, int &idx) {
    constexpr int h = NV / 2;
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
        const float send = up ? a[i] : a[i + h];
        const float keep = up ? a[i + h] : a[i];
        a[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
    if (up) idx += h;
}

template <int NV>
__device__ __forceinline__ int warp_reduce_vec(float *a, int lane) {
    int idx = 0, o = 16;
    if constexpr (NV >= 32) { halve<32>(a, lane, o, idx); o >>= 1; }
    if constexpr (NV >= 16) { halve<16>(a, lane, o, idx); o >>= 1; }
    if constexpr (NV >= 8) { halve<8>(a, lane, o, idx); o >>= 1; }
    if constexpr (NV >= 4) { halve<4>(a, lane, o, idx); o >>= 1; }
    if constexpr (NV >= 2) { halve<2>(a, lane, o, idx); o >>= 1; }
    for (; o > 0; o >>= 1) a[0] += __shfl_xor_sync(0xffffffffu, a[0], o);
    return ((lane & (32 / NV - 1)) == 0) ? idx : -1;
}

// rows of a product owned by block b: contiguous, a multiple of R each
template <int R>
__device__ __forceinline__ void mk_rows(int N, int &lo, int &hi) {
    const int per = (((N + (int)gridDim.x - 1) / (int)gridDim.x) + R - 1) / R * R;
    lo = min(N, (int)blockIdx.x * per);
    hi = min(N, lo + per);
}

// The block's four teams of 128 threads take R-row groups in turn, so three
// teams' loads are in flight while one reduces; within a team the threads
// split K (KI steps of 128 float4 at most) and reduce through the team's own
// shared partials (red + 128 * team) in warp order. A team is the same
// thread range as an attention group and uses the same named barrier.
//
// A team's first group of W does not depend on the previous phase, so it is
// loaded (WTile::load) before the grid barrier that ends that phase: the
// barrier's wait overlaps the first HBM round trip of the next product.
template <int R, int KI>
struct WTile {
    float4 v[KI][R];
    __device__ __forceinline__ void load(const float *__restrict__ W, long ldw, int N, int K) {
        constexpr int TT = 128;
        const int t = threadIdx.x & (TT - 1), K4 = K >> 2;
        int lo, hi;
        mk_rows<R>(N, lo, hi);
        const int n0 = lo + (int)(threadIdx.x >> 7) * R;
#pragma unroll
        for (int i = 0; i < KI; ++i) {
            const int k = t + i * TT;
#pragma unroll
            for (int r = 0; r < R; ++r)
                v[i][r] = (k < K4 && n0 < hi) ? __ldcs((const float4 *)(W + (long)min(n0 + r, N - 1) * ldw) + k)
                                              : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
};

template <int MT, int R, int KI, class Epi>
__device__ void mk_gemv(const float *xs, int B, int K, const float *__restrict__ W, long ldw, int N, Epi epi,
                        float *red, WTile<R, KI> &wv) {
    constexpr int NV = R * MT, TT = 128;
    static_assert(NV <= 32, "partial sums per thread");
    const int team = threadIdx.x >> 7, t = threadIdx.x & (TT - 1), lane = t & 31, warp = t >> 5, K4 = K >> 2;
    float *tred = red + team * TT;
    const float4 *x4 = (const float4 *)xs;
    int lo, hi;
    mk_rows<R>(N, lo, hi);
    for (int n0 = lo + team * R; n0 < hi; n0 += 4 * R) {
        if (n0 != lo + team * R) {  // the first group was loaded before the barrier
#pragma unroll
            for (int i = 0; i < KI; ++i) {
                const int k = t + i * TT;
#pragma unroll
                for (int r = 0; r < R; ++r)
                    wv.v[i][r] = k < K4 ? __ldcs((const float4 *)(W + (long)min(n0 + r, N - 1) * ldw) + k)
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        float acc[NV];
#pragma unroll
        for (int j = 0; j < NV; ++j) acc[j] = 0.f;
#pragma unroll
        for (int i = 0; i < KI; ++i) {
            const int k = t + i * TT;
            if (k < K4) {
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m < B) {
                        const float4 xv = x4[m * K4 + k];
#pragma unroll
                        for (int r = 0; r < R; ++r)
                            acc[r * MT + m] += wv.v[i][r].x * xv.x + wv.v[i][r].y * xv.y + wv.v[i][r].z * xv.z +
                                               wv.v[i][r].w * xv.w;
                    }
                }
            }
        }
        const int idx = warp_reduce_vec<NV>(acc, lane);
        if (idx >= 0) tred[warp * 32 + idx] = acc[0];
        group_sync(team);
        if (t < NV) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < TT / 32; ++w) v += tred[w * 32 + t];
            const int r = t / MT, m = t - r * MT, n = n0 + r;
            if (m < B && n < hi) epi(m, n, v);
        }
        group_sync(team);
    }
}

// L2 prefetch of the rows [lo, hi) of W [N, K] that this block streams next
// (at most the first 256 KB of them: the LM head's rows would not stay in L2)
template <int RW>
__device__ __forceinline__ void mk_prefetch(const float *W, int N, int K) {
    int lo, hi;
    mk_rows<RW>(N, lo, hi);
    const long lines = min((long)(hi - lo) * K / 32, 2048L);  // 128-byte lines
    const char *base = (const char *)(W + (long)lo * K);
    for (long i = threadIdx.x; i < lines; i += MK_THREADS)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(base + i * 128));
}

// ------------------------------------------------------------ attention
// One (sequence b, head h, 64-key chunk ch) item on a group of 128 threads
// (four groups per block, each synchronised by its own named barrier): scores
// of the chunk's keys (a half-warp per key, float4 of the head's 64
// dimensions per lane), V of the chunk loaded while the scores reduce, softmax
// terms, P V (two key halves per dimension), and the chunk's (max, sum,
// outputs) to `part`; the last chunk of (b, h) to finish (integer ticket)
// merges every chunk in chunk order into att.

constexpr int MK_GROUP_FLOATS = 64 * 5 + 4;

__device__ void mk_attention_item(const MkArgs &a, const float *kc_l, const float *vc_l, int b, int h, int ch,
                                  int len, int nch, float *sm, int g) {
    const int t = threadIdx.x & 127, C = a.C;
    float *sc = sm, *pr = sm + 64, *so = sm + 128, *cm = sm + 192, *cl = sm + 256, *misc = sm + 320;
    const int warp = t >> 5, lane = t & 31, half = lane >> 4, l16 = lane & 15;
    const int j0 = ch * MK_KEYS, kend = min(MK_KEYS, len - j0);
    const long brow = (long)b * a.Tmax * C + h * 64;
    const float4 qv = __ldcg((const float4 *)(a.qkv + (long)b * 3 * C + h * 64) + l16);
    float d[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int jl = warp * 16 + 2 * i + half;
        float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (jl < kend) kv = __ldcg((const float4 *)(kc_l + brow + (long)(j0 + jl) * C) + l16);
        d[i] = qv.x * kv.x + qv.y * kv.y + qv.z * kv.z + qv.w * kv.w;
    }
    // V of this thread's 32 keys (thread (kh, dim): keys 32 kh .., one dimension)
    const int dim = t & 63, kh = t >> 6;
    float vr[32];
#pragma unroll
    for (int i = 0; i < 32; ++i)
        vr[i] = (kh * 32 + i < kend) ? __ldcg(vc_l + brow + (long)(j0 + kh * 32 + i) * C + dim) : 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) d[i] += __shfl_xor_sync(0xffffffffu, d[i], o);
    if (l16 == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int jl = warp * 16 + 2 * i + half;
            sc[jl] = jl < kend ? d[i] * a.scale : -INFINITY;
        }
    }
    group_sync(g);
    if (warp < 2) {
        // warps 0 and 1 each take 32 of the scores; the maximum of all 64
        // (sc[0] is a valid key, so it is finite) and the softmax terms
        float m = fmaxf(sc[lane], sc[lane + 32]);
        m = warp_max(m);
        const float p = expf(sc[warp * 32 + lane] - m);
        pr[warp * 32 + lane] = p;
        const float w = warp_sum(p);
        if (lane == 0) {
            misc[warp] = w;
            misc[2] = m;
        }
    }
    group_sync(g);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < 32; ++i) acc += pr[kh * 32 + i] * vr[i];
    if (kh == 1) so[dim] = acc;
    group_sync(g);
    const int bh = b * a.H + h;
    float *pp = a.part + ((long)bh * a.S + ch) * MK_PART;
    if (kh == 0) {
        pp[2 + dim] = acc + so[dim];
        if (dim == 0) {
            pp[0] = misc[2];
            pp[1] = misc[0] + misc[1];
        }
    }
    __threadfence();
    group_sync(g);
    if (t == 0) misc[3] = (atomicAdd(&a.tickets[bh], 1) == nch - 1) ? 1.f : 0.f;
    group_sync(g);
    if (misc[3] != 0.f) {
        __threadfence();
        const float *pb = a.part + (long)bh * a.S * MK_PART;
        for (int k = t; k < nch; k += 128) {
            cm[k] = __ldcg(pb + k * MK_PART);
            cl[k] = __ldcg(pb + k * MK_PART + 1);
        }
        group_sync(g);
        if (t < 64) {
            float M = -INFINITY;
            for (int k = 0; k < nch; ++k) M = fmaxf(M, cm[k]);
            float L = 0.f, O = 0.f;
#pragma unroll 4
            for (int k = 0; k < nch; ++k) {
                const float w = expf(cm[k] - M);
                L += cl[k] * w;
                O += __ldcg(pb + k * MK_PART + 2 + t) * w;
            }
            a.att[(long)b * C + h * 64 + t] = O / L;
            if (t == 0) a.tickets[bh] = 0;
        }
    }
    group_sync(g);
}

// ------------------------------------------------------------ the step
template <int MT>
__global__ void __launch_bounds__(MK_THREADS, 1) decode_step_kernel(MkArgs a) {
    extern __shared__ float4 mk_smem4[];
    float *xs = (float *)mk_smem4;                  // [B][4C] staged rows
    float *red = xs + (size_t)MT * 4 * a.C;         // [16 warps][32] partial sums
    float *att_sm = red + MK_WARPS * 32;            // 4 attention groups
    __shared__ unsigned long long kmax[MT];
    const int C = a.C, B = a.B, L = a.L;
    const int pos = a.ctr[0], len = pos + 1;
    unsigned long long target = 0;
    int phase = 0;
    // phase trace (diagnostics): block 0 stamps the global timer after every barrier
    auto stamp = [&]() {
        if (a.trace && blockIdx.x == 0 && threadIdx.x == 0) a.trace[phase] = globaltimer_ns();
        ++phase;
    };
    stamp();
    const long LF = 12L * C * C + 13L * C;
    const float *layer0 = a.params + (long)a.V * C + (long)a.block * C;
    auto P = [&](int l) { return layer0 + (long)l * LF; };
    // parameter views of layer l in the reference's order (src/model.c:54-83)
    auto ln1_w = [&](int l) { return P(l); };
    auto ln1_b = [&](int l) { return P(l) + C; };
    auto attn_w = [&](int l) { return P(l) + 2L * C; };
    auto attn_b = [&](int l) { return P(l) + 2L * C + 3L * C * C; };
    auto proj1_w = [&](int l) { return attn_b(l) + 3L * C; };
    auto proj1_b = [&](int l) { return proj1_w(l) + (long)C * C; };
    auto ln2_w = [&](int l) { return proj1_b(l) + C; };
    auto ln2_b = [&](int l) { return ln2_w(l) + C; };
    auto fc_w = [&](int l) { return ln2_b(l) + C; };
    auto fc_b = [&](int l) { return fc_w(l) + 4L * C * C; };
    auto proj2_w = [&](int l) { return fc_b(l) + 4L * C; };
    auto proj2_b = [&](int l) { return proj2_w(l) + 4L * C * C; };
    const float *lnf_w = layer0 + (long)L * LF, *lnf_b = lnf_w + C;
    // rows per pass: R * MT <= 32 partial sums per thread, at most 16 loads of
    // W in flight per thread; K = C takes four 128-wide steps of K per thread
    // (C <= 2048), K = 4C sixteen
    constexpr int RC = MT <= 2 ? 4 : 2, R4 = 1;
    // embedding of the incoming tokens at position pos (src/model.c:460-470)
    for (int i = blockIdx.x * MK_THREADS + threadIdx.x; i < B * C; i += gridDim.x * MK_THREADS) {
        const int m = i / C, c = i - m * C;
        a.x[i] = __ldg(a.wte + (long)a.next[m] * C + c) + __ldg(a.wpe + (long)pos * C + c);
    }
    WTile<RC, 4> wc;   // first group of a K = C product, loaded before the barrier
    WTile<R4, 16> w4;  // first group of the K = 4C product
    mk_prefetch<RC>(attn_w(0), 3 * C, C);
    wc.load(attn_w(0), C, 3 * C, C);
    if (!mk_barrier(a.bar, a.abort, target)) return;
    stamp();
    for (int l = 0; l < L; ++l) {
        float *kc_l = a.kc + (long)l * a.B * a.Tmax * C, *vc_l = a.vc + (long)l * a.B * a.Tmax * C;
        // P1: LN1, qkv (+ bias), K and V appended at pos
        mk_stage<MT>(xs, a.x, C, B, C, ln1_w(l), ln1_b(l), red);
        {
            const float *bias = attn_b(l);
            mk_gemv<MT, RC, 4>(xs, B, C, attn_w(l), C, 3 * C, [&](int m, int n, float v) {
                v += __ldg(bias + n);
                a.qkv[(long)m * 3 * C + n] = v;
                const long at = ((long)m * a.Tmax + pos) * C;
                if (n >= 2 * C) vc_l[at + n - 2 * C] = v;
                else if (n >= C) kc_l[at + n - C] = v;
            }, red, wc);
        }
        mk_prefetch<RC>(proj1_w(l), C, C);
        if (!mk_barrier(a.bar, a.abort, target)) return;
        stamp();
        // P2: attention over positions [0, pos], four groups of 128 threads per block
        {
            const int nch = (len + MK_KEYS - 1) / MK_KEYS, items = B * a.H * nch, g = threadIdx.x >> 7;
            for (int it = 4 * blockIdx.x + g; it < items; it += 4 * gridDim.x) {
                const int ch = it % nch, bh = it / nch;
                mk_attention_item(a, kc_l, vc_l, bh / a.H, bh % a.H, ch, len, nch, att_sm + g * MK_GROUP_FLOATS,
                                  g);
            }
        }
        mk_prefetch<RC>(fc_w(l), 4 * C, C);
        wc.load(proj1_w(l), C, C, C);
        if (!mk_barrier(a.bar, a.abort, target)) return;
        stamp();
        // P3: c_proj, x += attn_proj + b
        mk_stage<MT>(xs, a.att, C, B, C, nullptr, nullptr, red);
        {
            const float *bias = proj1_b(l);
            mk_gemv<MT, RC, 4>(xs, B, C, proj1_w(l), C, C, [&](int m, int n, float v) {
                a.x[(long)m * C + n] += v + __ldg(bias + n);
            }, red, wc);
        }
        mk_prefetch<R4>(proj2_w(l), C, 4 * C);
        wc.load(fc_w(l), C, 4 * C, C);
        if (!mk_barrier(a.bar, a.abort, target)) return;
        stamp();
        // P4: LN2, fc, GELU
        mk_stage<MT>(xs, a.x, C, B, C, ln2_w(l), ln2_b(l), red);
        {
            const float *bias = fc_b(l);
            mk_gemv<MT, RC, 4>(xs, B, C, fc_w(l), C, 4 * C, [&](int m, int n, float v) {
                a.hid[(long)m * 4 * C + n] = gelu_tanh(v + __ldg(bias + n), a.fast_act != 0);
            }, red, wc);
        }
        if (l + 1 < L) mk_prefetch<RC>(attn_w(l + 1), 3 * C, C);
        w4.load(proj2_w(l), 4L * C, C, 4 * C);
        if (!mk_barrier(a.bar, a.abort, target)) return;
        stamp();
        // P5: proj, x += mlp_proj + b
        mk_stage<MT>(xs, a.hid, 4L * C, B, 4 * C, nullptr, nullptr, red);
        {
            const float *bias = proj2_b(l);
            mk_gemv<MT, R4, 16>(xs, B, 4 * C, proj2_w(l), 4L * C, C, [&](int m, int n, float v) {
                a.x[(long)m * C + n] += v + __ldg(bias + n);
            }, red, w4);
        }
        if (l + 1 == L) mk_prefetch<RC>(a.wte, a.V, C);
        if (l + 1 < L) wc.load(attn_w(l + 1), C, 3 * C, C);
        else wc.load(a.wte, C, a.V, C);
        if (!mk_barrier(a.bar, a.abort, target)) return;
        stamp();
    }
    // P6: LN_f, LM head, greedy keys
    mk_stage<MT>(xs, a.x, C, B, C, lnf_w, lnf_b, red);
    if (threadIdx.x < MT) kmax[threadIdx.x] = 0ull;
    __syncthreads();
    mk_gemv<MT, RC, 4>(xs, B, C, a.wte, C, a.V, [&](int m, int n, float v) {
        a.logits[(long)m * a.ldlog + n] = v;
        const uint32_t u = __float_as_uint(v);
        const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
        atomicMax(&kmax[m], ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)n));
    }, red, wc);
    __syncthreads();
    if (threadIdx.x < B && kmax[threadIdx.x]) atomicMax(a.am_key + threadIdx.x, kmax[threadIdx.x]);
    if (!mk_barrier(a.bar, a.abort, target)) return;
    stamp();
    // P7: tokens (next input, step log), keys cleared, counters advanced
    if (blockIdx.x == 0) {
        const int t = threadIdx.x;
        if (t < B) {
            const unsigned long long k = __ldcg(a.am_key + t);
            a.am_key[t] = 0ull;
            const int col = (int)(0xFFFFFFFFu - (uint32_t)k);
            a.next[t] = col;
            if (a.gen) a.gen[(long)a.ctr[1] * B + t] = col;
        }
        __syncthreads();
        if (t == 0) {
            a.ctr[0] = pos + 1;
            a.ctr[1] += 1;
        }
    }
}

template <int MT>
int launch_mk(const MkArgs &args, cudaStream_t s) {
    const size_t smem = mk_smem_bytes(args.C, MT);
    static size_t attr_bytes = 0;
    if (smem > attr_bytes) {
        CG_CUDA(cudaFuncSetAttribute(decode_step_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        int per_sm = 0;
        CG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel<MT>, MK_THREADS, smem));
        if (per_sm < 1) {
            set_last_error(ERR_ARG, "decode step kernel: a block does not fit on an SM (%zu B shared memory)", smem);
            return ERR_ARG;
        }
        attr_bytes = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms());  // one block per SM, all resident (cooperative launch)
    cfg.blockDim = dim3(MK_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    // the barrier counter and the abort word start at zero in every step
    CG_CUDA(cudaMemsetAsync(args.bar, 0, 16, s));
    CG_CUDA(cudaLaunchKernelEx(&cfg, decode_step_kernel<MT>, args));
    ++g_launch_count;
    return OK;
}

}  // namespace

size_t mk_smem_bytes(int C, int MT) {
    return ((size_t)MT * 4 * C + MK_WARPS * 32 + 4 * MK_GROUP_FLOATS) * sizeof(float);
}

namespace {
// off unless CNGPT_CUDA_DECODE_STEP_KERNEL=1 or cngpt_cuda_set_decode_step_kernel(1): measured on
// B200 it does not beat the kernel chain yet (grid barriers and latency-bound phases)
int g_mk_on = -1;
}  // namespace

void set_decode_step_kernel(bool on) { g_mk_on = on ? 1 : 0; }

bool decode_step_kernel_on() {
    if (g_mk_on < 0) {
        const char *e = getenv("CNGPT_CUDA_DECODE_STEP_KERNEL");
        g_mk_on = (e && e[0] == '1') ? 1 : 0;
    }
    return g_mk_on == 1;
}

bool mk_decode_ok(int B, int C, int H, long Tmax) {
    const int mt = B <= 1 ? 1 : B <= 2 ? 2 : B <= 4 ? 4 : 8;
    return decode_step_kernel_on() && B >= 1 && B <= 8 && H > 0 && C == 64 * H && C <= 2048 && Tmax > 0 &&
           Tmax <= 64 * MK_KEYS && mk_smem_bytes(C, mt) + 1024 <= 227 * 1024;
}

size_t mk_part_floats(int B, int H, long Tmax) {
    return (size_t)B * H * ((Tmax + MK_KEYS - 1) / MK_KEYS) * MK_PART;
}

int decode_step_mk(const MkArgs &args, cudaStream_t s) {
    if (args.B <= 1) return launch_mk<1>(args, s);
    if (args.B <= 2) return launch_mk<2>(args, s);
    if (args.B <= 4) return launch_mk<4>(args, s);
    return launch_mk<8>(args, s);
}

}  // namespace cg
