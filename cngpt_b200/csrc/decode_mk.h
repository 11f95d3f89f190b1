// decode_mk.h - the single-launch greedy decode step (decode_mk.cu), internal.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>

#include "internal.h"

namespace cg {

// Everything one decode step of B <= 8 sequences reads and writes. The
// parameters are the reference's single arena (params, wte, wpe views of it);
// the step embeds next[m] at position ctr[0], runs every layer (appending K
// and V at ctr[0]), writes logits [B, V], the greedy tokens to next[] and to
// gen[ctr[1] * B + m] (gen may be null), then advances both counters.
struct MkArgs {
    const float *params = nullptr, *wte = nullptr, *wpe = nullptr;
    int L = 0, C = 0, H = 0, V = 0, block = 0, B = 0;
    long Tmax = 0;
    float scale = 0.f;
    float *x = nullptr, *qkv = nullptr, *att = nullptr, *hid = nullptr;  // [B,C] [B,3C] [B,C] [B,4C]
    float *logits = nullptr;  // [B, ldlog]
    long ldlog = 0;
    float *kc = nullptr, *vc = nullptr;  // [L][B][Tmax][C]
    float *part = nullptr;               // attention chunk partials [B*H][S][66]
    int *tickets = nullptr;              // [B*H], zero between steps
    int S = 0;                           // chunk slots per (sequence, head)
    int *next = nullptr, *gen = nullptr, *ctr = nullptr;
    unsigned long long *am_key = nullptr;  // [B], zero between steps
    unsigned long long *bar = nullptr;     // 16 bytes: barrier counter and abort word, cleared per launch
    int *abort = nullptr;
    int fast_act = 0;
    // diagnostics: when set, block 0 writes the global timer (ns) at the start
    // and after every barrier: 2 + 5 L + 1 stamps
    unsigned long long *trace = nullptr;
};

// whether the single-launch step is enabled and handles this shape
bool mk_decode_ok(int B, int C, int H, long Tmax);
void set_decode_step_kernel(bool on);
bool decode_step_kernel_on();
size_t mk_smem_bytes(int C, int MT);
// attention partial floats for B sequences, H heads, Tmax positions (the ticket
// ints follow them in the same buffer)
size_t mk_part_floats(int B, int H, long Tmax);
int decode_step_mk(const MkArgs &args, cudaStream_t s);

}  // namespace cg
