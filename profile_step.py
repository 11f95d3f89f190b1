"""Run a few GPT-2 training steps (or one GEMM shape) through libcngpt_cuda,
for profilers (ncu) and quick timing.

    python profile_step.py [--B 8] [--T 1024] [--layers 12] [--steps 1]
                                      [--warmup 3] [--prec tf32|3xtf32|fp32]
    python profile_step.py --gemm M N K [--a-mn] [--b-mn] [--reps 3]
    python profile_step.py --decode xl|small [--B 1] [--T 128] [--new 8]
    python profile_step.py --attention [--B 8] [--T 1024] [--heads 12] [--reps 10]
    python profile_step.py --gemm-step [--reps 10] [--prec tf32]
    python profile_step.py --tp-reduce [--B 1] [--reps 3]

Token ids live on the device before the first step; nothing else runs.
"""
from __future__ import annotations

import argparse
import ctypes as C
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from cngpt_b200 import abi  # noqa: E402

PREC = {"tf32": abi.PREC_TF32, "3xtf32": abi.PREC_3XTF32, "fp32": abi.PREC_FP32}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--T", type=int, default=1024)
    ap.add_argument("--layers", type=int, default=12)
    ap.add_argument("--steps", type=int, default=1)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--prec", choices=list(PREC), default="tf32")
    ap.add_argument("--gemm", type=int, nargs=3, metavar=("M", "N", "K"))
    ap.add_argument("--a-mn", action="store_true")
    ap.add_argument("--b-mn", action="store_true")
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--epi", choices=["store", "gelu", "resid", "accum", "gelu_bwd"], default="store")
    ap.add_argument("--decode", choices=["xl", "small"], help="greedy KV-cache decode of GPT-2 XL / small "
                    "(device-random weights): prefill B x T, then --new tokens")
    ap.add_argument("--new", type=int, default=8)
    ap.add_argument("--attention", action="store_true", help="time one layer's causal attention forward and "
                    "backward (head size 64) through the C ABI")
    ap.add_argument("--heads", type=int, default=12)
    ap.add_argument("--gemm-step", action="store_true", help="time each distinct GEMM shape of one GPT-2 small "
                    "training step (B=8, T=1024) alone and print its share of the step's GEMM time")
    ap.add_argument("--tp-reduce", action="store_true", help="the tensor-parallel decode exchange's reduce "
                    "kernel on one GPU (self-test hook, flag published): --B rows of n_embd 1600, --reps launches")
    a = ap.parse_args()
    import torch
    torch.cuda.set_device(0)
    lib = abi.load()
    lib.cngpt_cuda_set_precision(PREC[a.prec])
    if a.tp_reduce:
        rows, Cx = min(a.B, 8), 1600
        part = torch.randn(rows, Cx, device="cuda")
        x = torch.empty(rows, Cx, device="cuda")
        stats = torch.empty(rows, 2, device="cuda")
        for _ in range(a.reps):
            abi.check(lib, lib.cngpt_cuda_selftest_tp_reduce(x.data_ptr(), part.data_ptr(), rows, Cx, 1,
                                                            stats.data_ptr()), "tp reduce")
        print(f"tp_reduce_kernel: {a.reps} launches of {rows} x {Cx}")
        return
    if a.gemm:
        M, N, K = a.gemm
        A = torch.randn((K, M) if a.a_mn else (M, K), device="cuda")
        B = torch.randn((K, N) if a.b_mn else (N, K), device="cuda")
        D = torch.zeros(M, N, device="cuda")
        D2 = torch.empty(M, N, device="cuda") if a.epi in ("gelu", "resid") else D
        R = torch.randn(M, N, device="cuda") if a.epi in ("resid", "gelu_bwd") else D
        bias = torch.zeros(N, device="cuda")
        mode = {"store": abi.EPI_STORE, "gelu": abi.EPI_GELU, "resid": abi.EPI_RESID,
                "accum": abi.EPI_ACCUM, "gelu_bwd": abi.EPI_GELU_BWD}[a.epi]
        def one():
            abi.check(lib, lib.cngpt_cuda_gemm(A.data_ptr(), A.shape[1], int(a.a_mn), B.data_ptr(), B.shape[1],
                                               int(a.b_mn), M, N, K, mode, 1.0, D.data_ptr(), N,
                                               bias.data_ptr(), D2.data_ptr(), N, R.data_ptr(), N,
                                               R.data_ptr(), N), "gemm")
        one()
        abi.check(lib, lib.cngpt_cuda_check(), "sync")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(max(a.reps - 1, 1)):
            one()
        e1.record()
        abi.check(lib, lib.cngpt_cuda_check(), "sync")
        us = e0.elapsed_time(e1) * 1e3 / max(a.reps - 1, 1)
        print(f"gemm {M}x{N}x{K} a_mn={int(a.a_mn)} b_mn={int(a.b_mn)} epi={a.epi}: {us:.1f} us "
              f"({2.0 * M * N * K / us / 1e6:.1f} TFLOP/s, CUDA events, back to back)")
        return
    if a.gemm_step:
        import bench  # the step's GEMM shapes (repository root is on sys.path)
        shapes = bench.step_gemm_shapes()
        BT, V, Cm = bench.B_ * bench.T_, bench.V_, bench.C_
        Vp = (V + 3) & ~3
        g = torch.Generator(device="cuda").manual_seed(0)
        f = lambda *sh: torch.randn(*sh, device="cuda", generator=g) * 0.02  # noqa: E731
        X, W, DL, G = f(BT, 4 * Cm), f(V, Cm), f(BT, Vp), f(BT, 4 * Cm)
        Y = torch.empty(BT, Vp, device="cuda")
        Dw = torch.zeros(V, Cm, device="cuda")
        bias = torch.zeros(4 * Cm, device="cuda")
        counts: dict = {}
        for sh in shapes:
            counts[sh] = counts.get(sh, 0) + 1
        names = {abi.EPI_STORE: "store", abi.EPI_ACCUM: "accum", abi.EPI_GELU: "gelu", abi.EPI_RESID: "resid",
                 abi.EPI_GELU_BWD: "gelu_bwd"}
        n = max(a.reps, 10)
        rows = []
        for sh, cnt in counts.items():
            M, N, K, amn, bmn, lda, ldb, epi, ldd = sh
            A_ = DL if lda == Vp else X
            B_ = W if ((not bmn and N == V) or (bmn and K == V)) else X
            D_ = Dw if epi == abi.EPI_ACCUM and M == V else Y

            def one():
                abi.check(lib, lib.cngpt_cuda_gemm(A_.data_ptr(), lda, amn, B_.data_ptr(), ldb, bmn, M, N, K, epi,
                                                   1.0, D_.data_ptr(), ldd,
                                                   bias.data_ptr() if epi in (abi.EPI_RESID, abi.EPI_GELU) else None,
                                                   G.data_ptr(), ldd, G.data_ptr(), ldd, G.data_ptr(), ldd), "gemm")
            for _ in range(2):
                one()
            abi.check(lib, lib.cngpt_cuda_check(), "sync")
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(n):
                one()
            e1.record()
            abi.check(lib, lib.cngpt_cuda_check(), "sync")
            rows.append((sh, cnt, e0.elapsed_time(e1) * 1e3 / n))
        total = sum(us * cnt for _, cnt, us in rows)
        flops = sum(2.0 * M * N * K * cnt for (M, N, K, *_r), cnt, _us in rows)
        print(f"{'M':>6} {'N':>6} {'K':>6} mn  epilogue  count      us  TFLOP/s  share")
        for (M, N, K, amn, bmn, _la, _lb, epi, _ld), cnt, us in sorted(rows, key=lambda r: -r[1] * r[2]):
            print(f"{M:>6} {N:>6} {K:>6} {amn}{bmn}  {names[epi]:<8} {cnt:>5} {us:>8.1f} {2.0 * M * N * K / us / 1e6:>8.1f}"
                  f"  {100.0 * us * cnt / total:5.1f}%")
        print(f"{len(shapes)} GEMMs, {total / 1e3:.2f} ms per step timed shape by shape, {flops / total / 1e6:.1f} "
              f"TFLOP/s (prec={a.prec}; CUDA events, back to back, each shape alone)")
        return
    if a.attention:
        B, T, H = a.B, a.T, a.heads
        Cm = 64 * H
        g = torch.Generator(device="cuda").manual_seed(1)
        qkv = torch.randn(B, T, 3 * Cm, device="cuda", generator=g)
        dout = torch.randn(B, T, Cm, device="cuda", generator=g)
        out = torch.empty(B, T, Cm, device="cuda")
        lse = torch.empty(B * H * T, device="cuda")
        dqkv = torch.empty(B, T, 3 * Cm, device="cuda")

        def fwd():
            abi.check(lib, lib.cngpt_cuda_attention_fwd(qkv.data_ptr(), out.data_ptr(), lse.data_ptr(), B, T, Cm,
                                                        H), "attention fwd")

        def bwd():
            abi.check(lib, lib.cngpt_cuda_attention_bwd(qkv.data_ptr(), out.data_ptr(), dout.data_ptr(),
                                                        lse.data_ptr(), dqkv.data_ptr(), B, T, Cm, H),
                      "attention bwd")

        def time_us(f):
            for _ in range(3):
                f()
            abi.check(lib, lib.cngpt_cuda_check(), "sync")
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            n = max(a.reps, 10)
            e0.record()
            for _ in range(n):
                f()
            e1.record()
            abi.check(lib, lib.cngpt_cuda_check(), "sync")
            return e0.elapsed_time(e1) * 1e3 / n

        tf, tb = time_us(fwd), time_us(bwd)
        flop = 4.0 * B * H * (T * (T + 1) / 2) * 64  # causal Q K^T and P V
        print(f"attention B={B} T={T} H={H} hs=64 prec={a.prec}: forward {tf:.1f} us ({flop / tf / 1e6:.0f} "
              f"TFLOP/s), backward {tb:.1f} us ({2.5 * flop / tb / 1e6:.0f} TFLOP/s incl. the rowsum(dO*O) pass; "
              f"CUDA events, back to back, inputs L2-resident)")
        return
    if a.decode:
        L, H, Cm = (48, 25, 1600) if a.decode == "xl" else (12, 12, 768)
        m = abi.GPT()
        assert lib.gpt_init(C.byref(m), abi.GPTConfig(L, H, Cm, 50257, 1024, 0.0)) == 0
        w = torch.randn(m.n_params, device="cuda", generator=torch.Generator("cuda").manual_seed(0)) * 0.02
        abi.check(lib, lib.cngpt_cuda_copy(C.cast(m.param_buf, C.c_void_p), C.c_void_p(w.data_ptr()),
                                           m.n_params * 4), "weights")
        del w
        prompt = np.arange(a.B * a.T, dtype=np.int32) % 50257
        out = np.zeros(a.B * a.new, np.int32)
        fc = abi.FastCtx()
        lib.fast_init(C.byref(fc))

        def gen(n):
            best = float("inf")
            for _ in range(a.reps):
                t0 = time.perf_counter()
                abi.check(lib, lib.cngpt_cuda_generate(C.byref(m), C.byref(fc), prompt.ctypes.data, a.B, a.T, n,
                                                       out.ctypes.data), "generate")
                best = min(best, time.perf_counter() - t0)
            return best
        dt = gen(a.new)
        print(f"decode {a.decode} B={a.B} T={a.T} new={a.new}: {dt * 1e3:.2f} ms per generate call")
        if a.new > 1:
            t1 = gen(1)
            per = (dt - t1) / (a.new - 1)
            byts = 4.0 * m.n_params + 8.0 * L * Cm * a.B * (a.T + a.new / 2.0)
            print(f"  {per * 1e3:.3f} ms per decode step, {byts / per / 1e9:.0f} GB/s of weights + K/V "
                  f"(wall clock, prompt upload and token read-back included)")
        lib.fast_free(C.byref(fc))
        lib.gpt_free(C.byref(m))
        return
    m = abi.GPT()
    assert lib.gpt_init(C.byref(m), abi.GPTConfig(a.layers, 12, 768, 50257, 1024, 0.0)) == 0
    C.CDLL(None).srand(1)
    lib.gpt_init_weights(C.byref(m))
    rng = np.random.default_rng(0)
    ids = torch.from_numpy(rng.integers(0, 50257, a.B * a.T + 1).astype(np.int32)).cuda()
    tok, tgt = ids[:-1].contiguous(), ids[1:].contiguous()
    loss = C.c_float()
    for i in range(a.warmup + a.steps):
        if i == a.warmup:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
        abi.check(lib, lib.cngpt_cuda_train_step(C.byref(m), tok.data_ptr(), tgt.data_ptr(), a.B, a.T, 1e-4,
                                                 0.9, 0.95, 1e-8, 0.1, 1.0, None), "step")
    abi.check(lib, lib.cngpt_cuda_check(), "sync")
    dt = (time.perf_counter() - t0) / max(a.steps, 1)
    abi.check(lib, lib.cngpt_cuda_last_loss(C.byref(m), C.byref(loss)), "loss")
    print(f"{a.steps} step(s) B={a.B} T={a.T} L={a.layers} prec={a.prec}: {dt * 1e3:.2f} ms/step "
          f"(host wall), loss {loss.value:.4f}")
    lib.gpt_free(C.byref(m))


if __name__ == "__main__":
    main()
