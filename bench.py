"""Benchmark: GPT-2 small training step (fwd + bwd + AdamW) through libcngpt_cuda.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: GPT-2 small 124M (12L / 12H / 768C, V=50257,
block 1024), random-init fp32 weights (the reference's init from the C
library's rand() stream), B=8 x T=1024 token ids per GPU from the reference
bench's LCG (uniform over [0, 50257)), next-token targets, cosine LR with
warmup, AdamW (betas 0.9/0.95, eps 1e-8, wd 0.1, clip 1.0). N > 1 GPUs run
data parallel (one process per GPU under torchrun, NCCL gradient average):
weak scaling, global batch 8N.

One JSON line on rank 0:
  value   tokens/s of the whole job with token ids already in HBM (device
          timed with CUDA events, max over ranks), TF32 tensor-core mode
  e2e     the same through cngpt_cuda_train_step with pinned host token
          buffers: H2D of the ids and D2H of the loss inside every step
  roofline  the tcgen05 GEMM kernel, replaying one step's GEMM shapes alone
  cpu_baseline  the reference's own CPU build (oracle/_ref) on this host
--impl reference times only the reference's CPU build (all host threads).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import math
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

L_, H_, C_, V_, BLOCK = 12, 12, 768, 50257, 1024
B_, T_ = 8, 1024
LR, LR_MIN, WARMUP_LR, TOTAL_ITERS = 3e-4, 1e-5, 100, 5000
METRIC = "GPT-2 small tokens/sec (train step: fwd+bwd+AdamW)"
BASELINE_METRIC = "GPT-2 tokens/sec (train step, prefill, decode); GEMM % of TF32/HBM roofline"


def bench_config(world: int) -> dict:
    return {"workload": "GPT-2 small 124M training step (fwd+bwd+AdamW), B=8 T=1024 per GPU "
                        "(BASELINE configs[1])", "global_batch": B_ * world, "seq_len": T_,
            "parallelism": f"dp{world}", "l2": "inputs larger than L2 (17 GB of activations per step)",
            "baseline_metric": BASELINE_METRIC}


def lr_schedule(step: int) -> float:
    """cosine schedule with linear warmup (src/cngpt.c:68-78)"""
    if step < WARMUP_LR:
        return LR * (step + 1) / WARMUP_LR
    if step >= TOTAL_ITERS:
        return LR_MIN
    p = (step - WARMUP_LR) / (TOTAL_ITERS - WARMUP_LR)
    return LR_MIN + 0.5 * (LR - LR_MIN) * (1.0 + math.cos(3.14159265 * p))


def lcg_tokens(n: int, vocab: int, seed: int) -> np.ndarray:
    """the reference bench's generator (src/cngpt.c:338-342), vectorised"""
    out = np.empty(n, dtype=np.int64)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = (s >> 8) % vocab
    return out.astype(np.int32)


def step_flops(B: int, T: int) -> dict:
    """algorithmic FLOPs of one training step (causal attention counted once
    per (query, key<=query) pair; no recompute; backward = 2x forward)"""
    BT = B * T
    lin = 2 * BT * C_ * (12 * C_) * L_                 # qkv + proj + fc + mlp_proj
    head = 2 * BT * V_ * C_
    attn = 2 * 2 * B * H_ * (T * (T + 1) // 2) * (C_ // H_) * L_   # QK^T and PV
    return {"gemm": 3 * (lin + head), "attn": 3 * attn, "total": 3 * (lin + head + attn)}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region"""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.window = None  # (start, end) of the timed region, monotonic seconds

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def mark(self, start: float, end: float):
        self.window = (start, end)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        """Samples taken inside the timed region; when it was shorter than the
        sampling period, the samples of the warm-up steps just before it (the
        same load) with `samples_in_window` saying so."""
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        lines = [ln for _, ln in self.lines]
        inside = lines
        if self.window:
            inside = [ln for t, ln in self.lines if self.window[0] <= t <= self.window[1] + 0.25]
        n_inside = len(inside)
        for ln in (inside if inside else lines):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "samples_in_window": n_inside}


# ------------------------------------------------------------------ reference arm
def cpu_reference_step_sample(steps: int, warmup: int, threads: int) -> dict:
    """The reference's own CPU build: one sequence of the workload (B=1, T=1024)
    per step through gpt_zero_grad / gpt_forward / gpt_backward / gpt_adamw."""
    os.environ["OPENBLAS_NUM_THREADS"] = str(threads)
    os.environ.setdefault("OMP_NUM_THREADS", str(threads))
    from cngpt_b200 import abi
    from oracle import oracle
    lib = oracle.reference()
    m = abi.GPT()
    assert lib.gpt_init(C.byref(m), abi.GPTConfig(L_, H_, C_, V_, BLOCK, 0.0)) == 0
    C.CDLL(None).srand(1)
    lib.gpt_init_weights(C.byref(m))
    ids = lcg_tokens(T_ + 1, V_, 12345)
    tok, tgt = ids[:-1].copy(), ids[1:].copy()
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        lib.gpt_zero_grad(C.byref(m))
        loss = lib.gpt_forward(C.byref(m), tok.ctypes.data, tgt.ctypes.data, 1, T_)
        lib.gpt_backward(C.byref(m), tok.ctypes.data, tgt.ctypes.data, 1, T_)
        lib.gpt_adamw(C.byref(m), lr_schedule(i), 0.9, 0.95, 1e-8, 0.1, 1.0)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    lib.gpt_free(C.byref(m))
    t = float(np.mean(times))
    return {"value": T_ / t, "unit": "tokens/s", "cores": threads, "kind": "reference",
            "sample": f"per-token rate of a B=1 sample: {steps} timed step(s) after {warmup} warm-up, each one "
                      f"sequence (B=1, T=1024, 1024 tokens) of the B=8 workload through the reference's "
                      f"gpt_zero_grad/gpt_forward/gpt_backward/gpt_adamw, OpenBLAS threads={threads}, "
                      f"last loss {loss:.4f} (a full B=8 step is 8 such sequences; CPU tokens/s do not grow "
                      f"with B)",
            "s_per_step": t, "host": host_cpu()}


def host_cpu() -> dict:
    """lscpu's socket / core / thread counts and model name of this host."""
    info = {"threads": os.cpu_count()}
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
    except (OSError, subprocess.SubprocessError):
        return info
    kv = {}
    for ln in out.splitlines():
        if ":" in ln:
            k, v = ln.split(":", 1)
            kv[k.strip()] = v.strip()
    try:
        cores = int(kv.get("Core(s) per socket", "0")) * int(kv.get("Socket(s)", "0"))
        info["physical_cores"] = cores or None
    except ValueError:
        pass
    info["model"] = kv.get("Model name")
    return info


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    cb = cpu_reference_step_sample(args.steps, args.warmup, threads)
    world = args.gpus
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cb["s_per_step"] * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic (reference LCG token ids)",
            "config": bench_config(world),
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample", "host")},
            "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm
def step_gemm_shapes() -> list:
    """The GEMMs of one GPT-2 small training step (B=8, T=1024) in model
    order, as (M, N, K, a_mn, b_mn, lda, ldb, epilogue, ldd): per layer the
    forward qkv / c_proj / fc / proj and the backward dX / dW pairs, then the
    tied LM head forward, dX and dW."""
    from cngpt_b200 import abi
    BT, Vp = B_ * T_, (V_ + 3) & ~3
    shapes = []
    for _ in range(L_):
        shapes += [(BT, 3 * C_, C_, 0, 0, C_, C_, abi.EPI_STORE, 3 * C_),
                   (BT, C_, C_, 0, 0, C_, C_, abi.EPI_RESID, C_),
                   (BT, 4 * C_, C_, 0, 0, C_, C_, abi.EPI_GELU, 4 * C_),
                   (BT, C_, 4 * C_, 0, 0, 4 * C_, 4 * C_, abi.EPI_RESID, C_),
                   (BT, 4 * C_, C_, 0, 1, C_, 4 * C_, abi.EPI_GELU_BWD, 4 * C_),
                   (C_, 4 * C_, BT, 1, 1, C_, 4 * C_, abi.EPI_ACCUM, 4 * C_),
                   (BT, C_, 4 * C_, 0, 1, 4 * C_, C_, abi.EPI_STORE, C_),
                   (4 * C_, C_, BT, 1, 1, 4 * C_, C_, abi.EPI_ACCUM, C_),
                   (BT, C_, C_, 0, 1, C_, C_, abi.EPI_STORE, C_),
                   (C_, C_, BT, 1, 1, C_, C_, abi.EPI_ACCUM, C_),
                   (BT, C_, 3 * C_, 0, 1, 3 * C_, C_, abi.EPI_STORE, C_),
                   (3 * C_, C_, BT, 1, 1, 3 * C_, C_, abi.EPI_ACCUM, C_)]
    shapes += [(BT, V_, C_, 0, 0, C_, C_, abi.EPI_STORE, V_),
               (BT, C_, V_, 0, 1, Vp, C_, abi.EPI_STORE, C_),
               (V_, C_, BT, 1, 1, Vp, C_, abi.EPI_ACCUM, C_)]
    return shapes


def gemm_replay(lib, torch, dev, prec: int, iters: int) -> dict:
    """Time the tcgen05 GEMM alone on one training step's GEMM shapes (same
    operand majorness and epilogues as the model), CUDA events on the stream
    the kernels run on (the legacy default stream)."""
    from cngpt_b200 import abi
    BT, Vp = B_ * T_, (V_ + 3) & ~3
    f = lambda *s: torch.randn(*s, device=dev) * 0.02  # noqa: E731
    X = f(BT, 4 * C_)
    W = f(V_, C_)
    Y = torch.empty(BT, Vp, device=dev)
    DL = f(BT, Vp)
    Dw = torch.zeros(V_, C_, device=dev)
    bias = torch.zeros(4 * C_, device=dev)
    G = f(BT, 4 * C_)
    shapes = step_gemm_shapes()
    flops = sum(2.0 * M * N * K for (M, N, K, *_r) in shapes)
    lib.cngpt_cuda_set_precision(prec)

    def run_all():
        for (M, N, K, amn, bmn, lda, ldb, epi, ldd) in shapes:
            a = DL if lda == Vp else X
            # the operand that spans the vocabulary is the [V, C] weight
            b = W if ((not bmn and N == V_) or (bmn and K == V_)) else X
            st = lib.cngpt_cuda_gemm(a.data_ptr(), lda, amn, b.data_ptr(), ldb, bmn, M, N, K, epi, 1.0,
                                     (Dw if epi == abi.EPI_ACCUM and M == V_ else Y).data_ptr(), ldd,
                                     bias.data_ptr() if epi in (abi.EPI_RESID, abi.EPI_GELU) else None,
                                     G.data_ptr(), ldd, G.data_ptr(), ldd, G.data_ptr(), ldd)
            if st:
                raise RuntimeError(lib.cngpt_cuda_last_message().decode())
    run_all()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        run_all()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    n = len(shapes)
    return {"flops_per_step": flops, "ms_per_step": ms, "launches": n,
            "tflops": flops / (ms * 1e-3) / 1e12, "flops_per_launch": flops / n, "ms_per_launch": ms / n}


def fc_gemm_roofline(lib, torch, dev, reps: int = 20) -> dict:
    """The dominant GEMM launch alone: the MLP fc projection of GPT-2 small
    (8192 x 3072 x 768, bias + GELU epilogue writing both outputs), the shape
    profiles/gemm_tc_fc_gelu_8192x3072x768.md captures. CUDA events on the
    stream the kernel runs on (the legacy default stream)."""
    from cngpt_b200 import abi
    M, N, K = B_ * T_, 4 * C_, C_
    A = torch.randn(M, K, device=dev) * 0.02
    W = torch.randn(N, K, device=dev) * 0.02
    bias = torch.zeros(N, device=dev)
    D, D2 = torch.empty(M, N, device=dev), torch.empty(M, N, device=dev)
    lib.cngpt_cuda_set_precision(abi.PREC_TF32)

    def one():
        st = lib.cngpt_cuda_gemm(A.data_ptr(), K, 0, W.data_ptr(), K, 0, M, N, K, abi.EPI_GELU, 1.0,
                                 D.data_ptr(), N, bias.data_ptr(), D2.data_ptr(), N, None, 0, None, 0)
        if st:
            raise RuntimeError(lib.cngpt_cuda_last_message().decode())
    for _ in range(3):
        one()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        one()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = 2.0 * M * N * K
    return {"ms_per_launch": ms, "flops_per_launch": flops, "tflops": flops / (ms * 1e-3) / 1e12,
            "algorithmic_bytes": 4.0 * (M * K + N * K + 2 * M * N)}


def decode_bytes(n_params: int, L: int, C: int, B: int, ctx0: int, steps: int) -> float:
    """HBM bytes one greedy decode step must read, averaged over the window:
    every weight once (fp32) plus the K and V cache of every layer up to the
    current position."""
    ctx = ctx0 + steps / 2.0
    return 4.0 * n_params + 2.0 * 4.0 * L * C * B * ctx


def inference_bench(lib, torch, dev, world: int, rank: int, hbm_peak: float, barrier, max_over_ranks) -> dict:
    """BASELINE configs[2] (GPT-2 small: prefill 128 + 256 greedy steps at
    B = 1 and 32, one GPU) and configs[4] (GPT-2 XL: prefill 8 x 1024, then
    128 greedy steps at B = 1 and 8, tensor parallel over all ranks).

    Times are wall-clock around the blocking API calls (prompt upload, the
    device work and the token read-back included), max over ranks; decode
    rate = (t(n_new) - t(1)) / (n_new - 1) per step."""
    from cngpt_b200 import abi
    out = {}

    def timed(fn, reps=2):
        fn()  # warm-up (graph capture, workspace allocation)
        best = float("inf")
        for _ in range(reps):
            barrier()
            t0 = time.perf_counter()
            fn()
            best = min(best, time.perf_counter() - t0)
        return max_over_ranks(best)

    if world == 1:
        m = abi.GPT()
        lib.gpt_init(C.byref(m), abi.GPTConfig(L_, H_, C_, V_, BLOCK, 0.0))
        C.CDLL(None).srand(1)
        lib.gpt_init_weights(C.byref(m))
        lib.cngpt_cuda_set_precision(abi.PREC_TF32)
        small = {}
        for B in (1, 32):
            T, n = 128, 256
            prompt = lcg_tokens(B * T, V_, 7)
            toks = np.zeros(B * n, np.int32)
            fc = abi.FastCtx()
            lib.fast_init(C.byref(fc))

            def gen(k):
                return lambda: abi.check(lib, lib.cngpt_cuda_generate(
                    C.byref(m), C.byref(fc), prompt.ctypes.data, B, T, k, toks.ctypes.data), "generate")
            t1, tn = timed(gen(1)), timed(gen(n))
            per = (tn - t1) / (n - 1)
            gbs = decode_bytes(m.n_params, L_, C_, B, T, n) / per / 1e9
            small[f"B{B}"] = {"decode_tokens_per_s": B / per, "ms_per_step": per * 1e3,
                              "prefill_tokens_per_s": B * T / t1, "hbm_gbs": gbs,
                              "hbm_frac": gbs / hbm_peak}
            lib.fast_free(C.byref(fc))
        lib.gpt_free(C.byref(m))
        out["gpt2_small"] = {"config": "BASELINE configs[2]: prefill 128 + 256 greedy steps, tf32", **small}
    # GPT-2 XL, tensor parallel over every rank
    L, H, Cx = 48, 25, 1600
    m = abi.GPT()
    lib.gpt_init(C.byref(m), abi.GPTConfig(L, H, Cx, V_, BLOCK, 0.0))
    g = torch.Generator(device=dev).manual_seed(1234)  # same weights on every rank
    w = torch.randn(m.n_params, generator=g, device=dev) * 0.02
    abi.check(lib, lib.cngpt_cuda_copy(C.cast(m.param_buf, C.c_void_p), C.c_void_p(w.data_ptr()), m.n_params * 4), "copy")
    del w
    uid = (C.c_ubyte * 128)()
    if world > 1:
        import torch.distributed as dist
        if rank == 0:
            abi.check(lib, lib.cngpt_cuda_dp_unique_id(uid), "tp id")
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0)
        uid = (C.c_ubyte * 128).from_buffer_copy(obj[0])
    st = lib.cngpt_cuda_tp_init(C.byref(m), uid, world, rank)
    # every rank must have its tensor-parallel state before any rank issues a
    # collective with it: agree on the outcome first
    worst = max_over_ranks(float(st != 0))
    if worst:
        msg = lib.cngpt_cuda_last_message().decode() if st else "another rank failed tp_init"
        if st == 0:
            lib.cngpt_cuda_tp_free(C.byref(m))
        lib.gpt_free(C.byref(m))
        out["gpt2_xl"] = {"error": f"tp_init failed: {msg}"}
        return out
    lib.cngpt_cuda_set_precision(abi.PREC_TF32)
    xl = {"config": "BASELINE configs[4]: prefill 8 x 1024; decode from a 896-token prompt for 128 "
                    "greedy steps (the cache ends at block_size 1024), tf32", "tp": world}
    Bp, Tp = 8, 1024
    ptok = lcg_tokens(Bp * Tp, V_, 11)
    tpf = timed(lambda: abi.check(lib, lib.cngpt_cuda_tp_forward_last(C.byref(m), ptok.ctypes.data, Bp, Tp, None),
                                  "tp forward"))
    flops = 2.0 * m.n_params * Bp * Tp
    xl["prefill_tokens_per_s"] = Bp * Tp / tpf
    xl["prefill_tflops"] = flops / tpf / 1e12
    for B in (1, 8):
        T, n = 896, 128
        prompt = lcg_tokens(B * T, V_, 13)
        toks = np.zeros(B * n, np.int32)

        def gen(k):
            return lambda: abi.check(lib, lib.cngpt_cuda_tp_generate(C.byref(m), prompt.ctypes.data, B, T, k,
                                                                     toks.ctypes.data), "tp generate")
        t1, tn = timed(gen(1), 1), timed(gen(n), 1)
        per = (tn - t1) / (n - 1)
        # batch 1 decodes replicated on every rank (the default decode mode):
        # each GPU streams all the weights and the whole cache; above batch 1
        # the weights and the heads are split across the ranks
        replicated = world > 1 and B == 1
        shards = 1 if replicated else world
        gbs = decode_bytes(m.n_params, L, Cx, B, T, n) / shards / per / 1e9
        xl[f"decode_B{B}"] = {"tokens_per_s": B / per, "ms_per_step": per * 1e3,
                              "mode": "replicated" if replicated else ("split" if world > 1 else "one GPU"),
                              "hbm_gbs_per_gpu": gbs, "hbm_frac_per_gpu": gbs / hbm_peak}
    lib.cngpt_cuda_tp_free(C.byref(m))
    lib.gpt_free(C.byref(m))
    out["gpt2_xl"] = xl
    return out



def train_configs_bench(lib, torch, dev, world: int, rank: int, barrier, max_over_ranks, tf32_peak: float) -> dict:
    """The other two training configs of BASELINE.json, data parallel over the
    job's GPUs like the headline: configs[0] tiny (6L/384/6H, V=65, B=64,
    T=256, lr 1e-3, betas 0.9/0.99) with the reference's rand() init, and
    configs[3] GPT-2 medium (24L/1024/16H, B=16, T=1024 per GPU) with
    device-random N(0, 0.02) weights (the host init of 355 M parameters would
    dominate the run; step cost does not depend on the values). TF32, CUDA
    events around the timed steps, max over ranks."""
    from cngpt_b200 import abi
    out = {}
    for name, (L, H, Cm, V, blk, B, T, b2, lr, steps) in {
            "tiny": (6, 6, 384, 65, 256, 64, 256, 0.99, 1e-3, 20),
            "gpt2_medium": (24, 16, 1024, 50257, 1024, 16, 1024, 0.95, 3e-4, 5)}.items():
        m = abi.GPT()
        abi.check(lib, 0 if lib.gpt_init(C.byref(m), abi.GPTConfig(L, H, Cm, V, blk, 0.0)) == 0 else 3, "gpt_init")
        if name == "tiny":
            C.CDLL(None).srand(1)
            lib.gpt_init_weights(C.byref(m))
        else:
            g = torch.Generator(device=dev).manual_seed(99)
            w = torch.randn(m.n_params, generator=g, device=dev) * 0.02
            abi.check(lib, lib.cngpt_cuda_copy(C.cast(m.param_buf, C.c_void_p), C.c_void_p(w.data_ptr()),
                                               m.n_params * 4), "weights")
            del w
        if world > 1:
            import torch.distributed as dist
            uid = (C.c_ubyte * 128)()
            if rank == 0:
                abi.check(lib, lib.cngpt_cuda_dp_unique_id(uid), "dp id")
            obj = [bytes(uid)]
            dist.broadcast_object_list(obj, src=0)
            uid = (C.c_ubyte * 128).from_buffer_copy(obj[0])
            abi.check(lib, lib.cngpt_cuda_dp_init(C.byref(m), uid, world, rank), "dp init")
        ids = lcg_tokens(B * T + 1, V, 12345 + rank)
        tok = torch.from_numpy(ids[:-1].copy()).to(dev)
        tgt = torch.from_numpy(ids[1:].copy()).to(dev)

        def step():
            st = lib.cngpt_cuda_train_step(C.byref(m), tok.data_ptr(), tgt.data_ptr(), B, T, lr, 0.9, b2, 1e-8,
                                           0.1, 1.0, None)
            if st:
                raise RuntimeError(lib.cngpt_cuda_last_message().decode())
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(e0.elapsed_time(e1)) / steps
        loss = C.c_float()
        abi.check(lib, lib.cngpt_cuda_last_loss(C.byref(m), C.byref(loss)), "loss")
        fl = step_flops_cfg(L, Cm, V, B, T)
        out[name] = {"config": f"BASELINE configs[{0 if name == 'tiny' else 3}]: {L}L/{Cm}C/{H}H V={V}, "
                               f"B={B} T={T} per GPU, dp{world}",
                     "tokens_per_s": B * T * world / (ms * 1e-3), "ms_per_step": ms, "steps": steps,
                     "step_tflops_per_gpu": fl / (ms * 1e-3) / 1e12,
                     "step_frac_of_tf32_peak": fl / (ms * 1e-3) / 1e12 / tf32_peak, "loss": float(loss.value)}
        if world > 1:
            lib.cngpt_cuda_dp_free(C.byref(m))
        lib.gpt_free(C.byref(m))
    return out


def loader_e2e(lib, torch, m, rank: int, K: int, barrier, max_over_ranks, step_no) -> float:
    """ms per training step fed by the device batch loader from a host uint16
    token array (as the reference's DataLoader mmaps it), loss read back every
    step: host copy into the pinned buffer, H2D and widening inside the timed
    region, overlapped with the previous step."""
    from cngpt_b200 import abi
    data = lcg_tokens(4 * B_ * T_ + 1, V_, 777 + rank).astype(np.uint16)
    h = C.c_void_p()
    abi.check(lib, lib.cngpt_cuda_loader_create(C.byref(h), data.ctypes.data, data.size, B_, T_), "loader")
    loss = C.c_float()

    def step():
        i, t = C.c_void_p(), C.c_void_p()
        abi.check(lib, lib.cngpt_cuda_loader_next(h, C.byref(i), C.byref(t)), "loader next")
        st = lib.cngpt_cuda_train_step(C.byref(m), i, t, B_, T_, lr_schedule(step_no[0]), 0.9, 0.95, 1e-8, 0.1,
                                       1.0, C.addressof(loss))
        step_no[0] += 1
        if st:
            raise RuntimeError(lib.cngpt_cuda_last_message().decode())
    step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(K):
        step()
    e1.record()
    torch.cuda.synchronize()
    barrier()
    lib.cngpt_cuda_loader_free(h)
    return max_over_ranks(e0.elapsed_time(e1)) / K


def step_flops_cfg(L: int, Cm: int, V: int, B: int, T: int) -> float:
    """Algorithmic FLOP of one training step (3 x forward: linears, causal
    attention over T(T+1)/2 pairs, LM head)."""
    BT = B * T
    lin = 2.0 * BT * L * (3 * Cm * Cm + Cm * Cm + 8 * Cm * Cm)
    attn = 4.0 * B * L * Cm * (T * (T + 1) / 2)
    head = 2.0 * BT * V * Cm
    return 3.0 * (lin + attn + head)


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist
    from cngpt_b200 import abi

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    lib = abi.load()
    m = abi.GPT()
    abi.check(lib, 0 if lib.gpt_init(C.byref(m), abi.GPTConfig(L_, H_, C_, V_, BLOCK, 0.0)) == 0 else 3,
              "gpt_init")
    C.CDLL(None).srand(1)   # "seed 0": the C library's default stream (src/cngpt.c:112)
    lib.gpt_init_weights(C.byref(m))
    if world > 1:
        uid = (C.c_ubyte * 128)()
        if rank == 0:
            abi.check(lib, lib.cngpt_cuda_dp_unique_id(uid), "dp id")
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0)
        uid = (C.c_ubyte * 128).from_buffer_copy(obj[0])
        abi.check(lib, lib.cngpt_cuda_dp_init(C.byref(m), uid, world, rank), "dp init")

    ids = lcg_tokens(B_ * T_ + 1, V_, 12345 + rank)
    tok_h = torch.from_numpy(ids[:-1].copy()).pin_memory()
    tgt_h = torch.from_numpy(ids[1:].copy()).pin_memory()
    tok_d, tgt_d = tok_h.to(dev), tgt_h.to(dev)
    step_no = [0]

    def train_step(tok_ptr, tgt_ptr, loss_ptr):
        st = lib.cngpt_cuda_train_step(C.byref(m), tok_ptr, tgt_ptr, B_, T_, lr_schedule(step_no[0]),
                                       0.9, 0.95, 1e-8, 0.1, 1.0, loss_ptr)
        step_no[0] += 1
        if st:
            raise RuntimeError(lib.cngpt_cuda_last_message().decode())

    def timed(prec: int, host_io: bool, K: int, W: int, clocks=None):
        lib.cngpt_cuda_set_precision(prec)
        loss = C.c_float()
        args_ = ((tok_h.data_ptr(), tgt_h.data_ptr(), C.addressof(loss)) if host_io
                 else (tok_d.data_ptr(), tgt_d.data_ptr(), None))
        ctx = clocks if clocks is not None else _Null()
        with ctx:  # the sampler starts before the warm-up: nvidia-smi takes a while to report
            for _ in range(W):
                train_step(*args_)
            torch.cuda.synchronize()
            barrier()
            torch.cuda.synchronize()
            l0 = lib.cngpt_cuda_launch_count()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t_start = time.monotonic()
            e0.record()
            for _ in range(K):
                train_step(*args_)
            e1.record()
            torch.cuda.synchronize()
            if clocks is not None:
                clocks.mark(t_start, time.monotonic())
        barrier()
        launches = lib.cngpt_cuda_launch_count() - l0
        ms = max_over_ranks(e0.elapsed_time(e1)) / K
        last = C.c_float()
        abi.check(lib, lib.cngpt_cuda_last_loss(C.byref(m), C.byref(last)), "loss")
        abi.check(lib, lib.cngpt_cuda_check(), "device check")
        return ms, launches // K, float(last.value)

    clocks = ClockSampler(local)
    ms, launches, loss = timed(abi.PREC_TF32, False, args.steps, args.warmup, clocks)
    if not math.isfinite(loss):
        raise RuntimeError(f"non-finite loss {loss}")
    tokens = B_ * T_ * world
    value = tokens / (ms * 1e-3)
    ms_e2e, _, _ = timed(abi.PREC_TF32, True, max(3, args.steps // 2), 1)
    ms_loader = loader_e2e(lib, torch, m, rank, max(3, args.steps // 2), barrier, max_over_ranks, step_no)
    ms_3x, _, loss_3x = timed(abi.PREC_3XTF32, False, max(3, args.steps // 2), 1)
    fl = step_flops(B_, T_)
    peaks = {}
    pk = ROOT / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    tf32_peak = peaks.get("bf16_tflops", 1590.0) / 2.0
    peak_src = ("of measured (bf16 cuBLAS burst / 2: the tf32 tensor rate is half the bf16 rate)"
                if "bf16_tflops" in peaks else "of fallback (1.59 PF bf16 / 2)")
    replay = gemm_replay(lib, torch, dev, abi.PREC_TF32, 3)
    fc = fc_gemm_roofline(lib, torch, dev)
    traffic = None
    prof = ROOT / "profiles" / "gemm_tc_traffic.json"
    if prof.exists():
        traffic = json.loads(prof.read_text()).get("dram_bytes_per_launch")
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "tf32", "data": "synthetic (reference LCG token ids, random-init "
        "weights from the reference's rand() init)",
        "config": bench_config(world),
        "e2e": {"value": tokens / (ms_e2e * 1e-3), "unit": "tokens/s",
                "h2d_bytes_per_step": 3 * B_ * T_ * 4, "d2h_bytes_per_step": 4,
                "api": "cngpt_cuda_train_step with pinned host token buffers and the loss read back"},
        "e2e_loader": {"value": tokens / (ms_loader * 1e-3), "unit": "tokens/s",
                       "h2d_bytes_per_step": (B_ * T_ + 1) * 2, "d2h_bytes_per_step": 4,
                       "api": "cngpt_cuda_loader_next (uint16 host token array through a pinned buffer, uploaded "
                              "one batch ahead) + cngpt_cuda_train_step with the loss read back"},
        "gpu_launches": launches,
        "roofline": {"bound": "tensor", "achieved": fc["tflops"], "peak": tf32_peak,
                     "unit": "TFLOP/s", "frac": fc["tflops"] / tf32_peak, "traffic": traffic,
                     "kernel": "gemm_tc2_kernel<256,K,K,0,GELU> (CTA pair, tf32, 16 epilogue warps): GPT-2 small fc GEMM "
                               "8192x3072x768, bias+GELU",
                     "peak_source": peak_src, "flops_per_launch": fc["flops_per_launch"],
                     "ms_per_launch": fc["ms_per_launch"], "algorithmic_bytes": fc["algorithmic_bytes"]},
        "gemm_step_replay": {"tflops": replay["tflops"], "frac": replay["tflops"] / tf32_peak,
                             "launches": replay["launches"], "ms_per_step": replay["ms_per_step"],
                             "note": "all 147 GEMM shapes of one training step, same operand "
                                     "layouts and epilogues, timed alone"},
        "step_tflops": fl["total"] / (ms * 1e-3) / 1e12,
        "step_frac_of_tf32_peak": fl["total"] / (ms * 1e-3) / 1e12 / tf32_peak,
        "loss_after_steps": loss,
        "modes": {"3xtf32": {"value": tokens / (ms_3x * 1e-3), "ms_per_step": ms_3x, "loss": loss_3x}},
        "clocks": clocks.summary(),
    }
    if not args.no_inference:
        line["inference"] = inference_bench(lib, torch, dev, world, rank, peaks.get("hbm_gbs", 6650.0),
                                            barrier, max_over_ranks)
    if not args.no_other_configs:
        lib.cngpt_cuda_set_precision(abi.PREC_TF32)
        line["other_train_configs"] = train_configs_bench(lib, torch, dev, world, rank, barrier, max_over_ranks,
                                                          tf32_peak)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cb = cpu_reference_step_sample(3, 1, os.cpu_count() or 1)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample", "host")}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        lib.cngpt_cuda_dp_free(C.byref(m))
        dist.destroy_process_group()
    lib.gpt_free(C.byref(m))


class _Null:
    def __enter__(self):
        return self

    def __exit__(self, *a):
        return False


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-inference", action="store_true", help="skip the decode / prefill figures")
    ap.add_argument("--no-other-configs", action="store_true", help="skip the tiny and medium training figures")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
