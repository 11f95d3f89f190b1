"""Generate the golden fixtures in tests/golden/ from the reference itself.

    make -C oracle ref && python tests/golden/make_golden.py

Runs the reference's own CPU build (oracle/_ref/libcngpt_ref.so: its ops.c,
model.c and fast.c compiled against OpenBLAS) on seeded weights (glibc rand()
stream, as src/cngpt.c:112 seeds it) and the reference bench's LCG tokens
(src/cngpt.c:338-342), and stores small .npz files: loss, logits, gradient
samples, post-AdamW parameter samples and fast-path last-position logits.
The fixtures pin the C restatement (oracle/cngpt_oracle.c) where the
reference tree is absent, and are compared with the CUDA path by the GPU tests.
"""
from __future__ import annotations

import ctypes as C
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from cngpt_b200 import abi  # noqa: E402  (struct layouts only)
from oracle import oracle  # noqa: E402

OUT = Path(__file__).resolve().parent

# name: (n_layer, n_head, n_embd, vocab, block, B, T, seed)
CASES = {
    "grad": (2, 4, 32, 64, 8, 2, 6, 1234),     # tests/check_grad.c:38-44
    "fast": (3, 4, 32, 70, 16, 3, 16, 42),     # tests/check_fast.c:29-33
    "hs64": (2, 2, 128, 96, 128, 2, 100, 7),
    "tiny": (2, 6, 384, 65, 256, 2, 256, None),  # BASELINE tiny widths, 2 of 6 layers
}
SAMPLE = 997  # every SAMPLE-th gradient / parameter element is stored


def tokens(B, T, V):
    # one LCG stream of B*T+1 ids; targets are the next id (src/dataloader.c:62-82)
    s = oracle.lcg_tokens(B * T + 1, V)
    return s[:-1].copy(), s[1:].copy()


def run_case(name, L, H, Cm, V, block, B, T, seed):
    lib = oracle.reference()
    m = abi.GPT()
    assert lib.gpt_init(C.byref(m), abi.GPTConfig(L, H, Cm, V, block, 0.0)) == 0
    oracle.libc_rand_stream(seed)
    lib.gpt_init_weights(C.byref(m))
    n = m.n_params
    par = lambda: np.ctypeslib.as_array(m.param_buf, shape=(n,)).copy()  # noqa: E731
    grd = lambda: np.ctypeslib.as_array(m.grad_buf, shape=(n,)).copy()  # noqa: E731
    tok, tgt = tokens(B, T, V)
    p0 = par()
    lib.gpt_zero_grad(C.byref(m))
    loss = lib.gpt_forward(C.byref(m), tok.ctypes.data, tgt.ctypes.data, B, T)
    logits = np.ctypeslib.as_array(m.acts.logits, shape=(B * T * V,)).copy()
    lib.gpt_backward(C.byref(m), tok.ctypes.data, tgt.ctypes.data, B, T)
    g = grd()
    lib.gpt_adamw(C.byref(m), 1e-3, 0.9, 0.99, 1e-8, 0.1, 1.0)
    p1 = par()
    fc = abi.FastCtx()
    lib.fast_init(C.byref(fc))
    fl = lib.gpt_forward_fast(C.byref(m), C.byref(fc), tok.ctypes.data, B, T)
    fast = np.ctypeslib.as_array(fl, shape=(B * V,)).copy()
    lib.fast_free(C.byref(fc))
    lib.gpt_free(C.byref(m))
    idx = np.arange(0, n, SAMPLE)
    np.savez_compressed(
        OUT / f"{name}.npz", cfg=np.array([L, H, Cm, V, block, B, T, -1 if seed is None else seed]),
        tokens=tok, targets=tgt, loss=np.float32(loss), logits=logits.reshape(B, T, V),
        idx=idx, p0_sample=p0[idx], grad_sample=g[idx], grad_norm=np.float64(np.linalg.norm(g.astype(np.float64))),
        p1_sample=p1[idx], fast_logits=fast.reshape(B, V))
    print(f"{name}: loss {loss:.6f} params {n} |g| {np.linalg.norm(g):.6f}")


if __name__ == "__main__":
    for k, v in CASES.items():
        run_case(k, *v)
