"""Data-parallel training on 2 GPUs (one process per GPU, NCCL): the averaged
gradients equal the mean of the two slices' gradients computed on one GPU
(normwise 1e-6: the sum order across ranks may differ by an ulp), and the two
ranks hold bit-identical parameters after the replicated AdamW step.
Needs two GPUs; on a one-GPU box it is skipped."""
import ctypes as C
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

from cngpt_b200 import abi
from oracle import oracle
from tests.models import CudaModel, nwerr

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dp2_matches_single_gpu_average(lib, cuda):
    from tests.dp_worker import B, CFG, T
    with tempfile.TemporaryDirectory() as d:
        env = dict(os.environ, NCCL_NVLS_ENABLE="0")
        cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
               str(ROOT / "tests" / "dp_worker.py"), d]
        r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=400)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
        r0, r1 = np.load(os.path.join(d, "rank0.npz")), np.load(os.path.join(d, "rank1.npz"))
    assert np.array_equal(r0["params"], r1["params"]), "ranks diverged after AdamW"
    assert np.array_equal(r0["grads"], r1["grads"])
    m = CudaModel(lib, *CFG, 7)
    ids = oracle.lcg_tokens(2 * B * T + 1, CFG[3], seed=31)
    n = B * T
    acc = np.zeros(m.n, np.float64)
    for rank in range(2):
        m.zero_grad()
        m.forward(ids[rank * n:(rank + 1) * n].copy(), ids[rank * n + 1:(rank + 1) * n + 1].copy(), B, T)
        m.backward(ids[rank * n:(rank + 1) * n].copy(), ids[rank * n + 1:(rank + 1) * n + 1].copy(), B, T)
        acc += m.grads()
    avg = (acc / 2).astype(np.float32)
    e = nwerr(r0["grads"], avg)
    print(f"\ndp2 averaged gradient vs single-GPU mean: normwise {e:.2e}")
    assert e < 1e-6
    m.free()
