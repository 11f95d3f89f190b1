"""Every tile width of the CTA-pair GEMM (256, 192 and 128 output columns per
pair tile) against a float64 product, in TF32 mode: the width is normally
picked by a time model, so each width is forced in a child process through
CNGPT_CUDA_PAIR_BN (read once per process). Shapes: the GPT-2 small N = 768
products at reduced M, a ragged N that leaves a partial last tile, all four
operand orientations, every epilogue mode, and a K split.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]

WORKER = r'''
import sys
import numpy as np
sys.path.insert(0, sys.argv[1])
import torch
from cngpt_b200 import abi
from tests.test_gemm_gpu import run_gemm, nwerr
lib = abi.load()
lib.cngpt_cuda_set_precision(abi.PREC_TF32)
dev = torch.device("cuda:0")
worst = 0.0
cases = []
for M, N, K in [(512, 768, 768), (600, 768, 300), (1024, 1000, 96), (384, 2304, 192)]:
    for a_mn, b_mn in [(False, False), (False, True), (True, True), (True, False)]:
        cases.append((M, N, K, a_mn, b_mn, abi.EPI_STORE))
for mode in [abi.EPI_ACCUM, abi.EPI_GELU, abi.EPI_RESID, abi.EPI_GELU_BWD]:
    cases.append((512, 768, 256, False, False, mode))
    cases.append((512, 768, 256, False, True, mode))
cases.append((512, 768, 8192, True, True, abi.EPI_ACCUM))  # long K: split into K ranges
for M, N, K, a_mn, b_mn, mode in cases:
    r = run_gemm(lib, dev, M, N, K, a_mn, b_mn, mode=mode, bias=mode != abi.EPI_GELU_BWD, seed=M + N + K)
    ref = r["ref"]
    if mode == abi.EPI_GELU:
        errs = [nwerr(r["D"], ref),
                nwerr(r["D2"], 0.5 * ref * (1 + np.tanh(0.7978845608028654 * (ref + 0.044715 * ref ** 3))))]
    elif mode == abi.EPI_RESID:
        errs = [nwerr(r["D"], ref), nwerr(r["D2"], r["R"] + ref)]
    elif mode == abi.EPI_GELU_BWD:
        x = r["G"]
        th = np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3))
        gp = 0.5 * (1 + th) + 0.5 * x * (1 - th * th) * 0.7978845608028654 * (1 + 3 * 0.044715 * x * x)
        errs = [nwerr(r["D"], ref * gp)]
    else:
        errs = [nwerr(r["D"], ref)]
    e = max(errs)
    worst = max(worst, e)
    print(f"M={M} N={N} K={K} a_mn={a_mn} b_mn={b_mn} mode={mode}: normwise {e:.3e}")
    assert e < 2e-3, (M, N, K, a_mn, b_mn, mode, e)
print(f"worst {worst:.3e}")
'''


@pytest.mark.parametrize("bn", [256, 192, 128])
def test_pair_tile_width(cuda, bn):
    env = dict(os.environ, CNGPT_CUDA_PAIR_BN=str(bn))
    r = subprocess.run([sys.executable, "-c", WORKER, str(ROOT)], capture_output=True, text=True, env=env,
                       timeout=600, cwd=str(ROOT))
    print(r.stdout[-3000:])
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    assert "worst" in r.stdout
