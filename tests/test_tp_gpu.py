"""Tensor-parallel inference parity (cngpt_cuda_tp_*): the split forward's
gathered final-position logits against the reference's gpt_forward_fast
(src/fast.c:227-333) on identical seeded weights, normwise 1e-5 (3xTF32),
and the split greedy decode against the one-GPU cngpt_cuda_generate.

Cases: 5 heads at n_embd 320 (uneven 3/2 head split, ragged vocabulary 1001),
3 heads of size 32 (CUDA-core attention path), two layers of GPT-2 XL's
shape (25 heads: 13/12 over two ranks), and a decode batch of 10 (above the
8 rows the peer-memory exchange takes, so its partial sums go through
ncclAllReduce). world = 1 runs on any GPU; worlds 2, 4 and 8 need that many
GPUs and are skipped on a smaller box. At world > 1 the decode exchanges of
batches up to 8 run through the GEMV's peer-memory push and tp_reduce_kernel."""
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
from tests.models import CudaModel, RefModel, nwerr
from tests.tp_worker import CASES

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def ref_last_logits(cfg, B, T):
    ref = RefModel(*cfg)
    tok = oracle.lcg_tokens(B * T, cfg[3], seed=100 + B * T)
    fc = abi.FastCtx()
    ref.lib.fast_init(C.byref(fc))
    p = ref.lib.gpt_forward_fast(C.byref(ref.m), C.byref(fc), tok.ctypes.data, B, T)
    out = np.ctypeslib.as_array(p, shape=(B * cfg[3],)).copy().reshape(B, -1)
    ref.lib.fast_free(C.byref(fc))
    ref.free()
    return out


def one_gpu_generate(lib, cfg, B, T, n):
    dev = CudaModel(lib, *cfg)
    prompt = oracle.lcg_tokens(B * T, cfg[3], seed=7)
    out = np.zeros(B * n, np.int32)
    fc = abi.FastCtx()
    lib.fast_init(C.byref(fc))
    abi.check(lib, lib.cngpt_cuda_generate(C.byref(dev.m), C.byref(fc), prompt.ctypes.data, B, T, n,
                                           out.ctypes.data), "generate")
    lib.fast_free(C.byref(fc))
    dev.free()
    return out.reshape(B, n)


def check_case(lib, name, logits, tokens):
    cfg, (fb, ft), (gb, gt, gn) = CASES[name]
    e = nwerr(logits, ref_last_logits(cfg, fb, ft))
    print(f"\n[{name}] tp logits vs reference normwise {e:.2e}")
    assert e < 1e-5
    want = one_gpu_generate(lib, cfg, gb, gt, gn)
    assert np.array_equal(tokens, want), (tokens, want)


@pytest.mark.parametrize("name", list(CASES))
def test_tp1_matches_reference(lib, cuda, name):
    cfg, (fb, ft), (gb, gt, gn) = CASES[name]
    lib.cngpt_cuda_set_precision(abi.PREC_3XTF32)
    m = CudaModel(lib, *cfg)
    uid = (C.c_ubyte * 128)()
    abi.check(lib, lib.cngpt_cuda_tp_init(C.byref(m.m), uid, 1, 0), "tp_init")
    tok = oracle.lcg_tokens(fb * ft, cfg[3], seed=100 + fb * ft)
    logits = np.zeros(fb * cfg[3], np.float32)
    abi.check(lib, lib.cngpt_cuda_tp_forward_last(C.byref(m.m), tok.ctypes.data, fb, ft, logits.ctypes.data),
              "forward_last")
    prompt = oracle.lcg_tokens(gb * gt, cfg[3], seed=7)
    out = np.zeros(gb * gn, np.int32)
    abi.check(lib, lib.cngpt_cuda_tp_generate(C.byref(m.m), prompt.ctypes.data, gb, gt, gn, out.ctypes.data),
              "tp_generate")
    m.free()  # gpt_free releases the tensor-parallel state too
    check_case(lib, name, logits.reshape(fb, -1), out.reshape(gb, gn))


def test_tp_decode_mode_rejects_unknown(lib, cuda):
    m = CudaModel(lib, 1, 2, 128, 50, 16, 3)
    uid = (C.c_ubyte * 128)()
    abi.check(lib, lib.cngpt_cuda_tp_init(C.byref(m.m), uid, 1, 0), "tp_init")
    assert lib.cngpt_cuda_tp_set_decode_mode(C.byref(m.m), 3) == abi.ERR_ARG
    lib.cngpt_cuda_clear_status()
    m.free()


def test_tp_requires_init(lib, cuda):
    m = CudaModel(lib, 1, 2, 64, 50, 16, 3)
    out = np.zeros(4, np.int32)
    assert lib.cngpt_cuda_tp_generate(C.byref(m.m), out.ctypes.data, 1, 2, 2, out.ctypes.data) == abi.ERR_STATE
    lib.cngpt_cuda_clear_status()
    m.free()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_multi_gpu_matches_reference(lib, cuda, world):
    """world ranks, one per GPU (skipped with fewer GPUs); the cases whose
    head count is at least world"""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    names = [n for n in CASES if CASES[n][0][1] >= world]
    with tempfile.TemporaryDirectory() as d:
        env = dict(os.environ, NCCL_NVLS_ENABLE="0")
        cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={29530 + world}",
               str(ROOT / "tests" / "tp_worker.py"), d, *names]
        r = subprocess.run(cmd, capture_output=True, text=True, env=env, timeout=700)
        assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
        res = [np.load(os.path.join(d, f"rank{k}.npz")) for k in range(world)]
    for name in names:
        for k in ("_logits", "_tokens", "_split"):
            for rk in range(1, world):
                assert np.array_equal(res[0][name + k], res[rk][name + k]), (name, k, rk)
        check_case(lib, name, res[0][name + "_logits"], res[0][name + "_tokens"])
        # the split decode (exchanges over NVLink) gives the same greedy tokens
        assert np.array_equal(res[0][name + "_split"], res[0][name + "_tokens"]), name
    print(f"\ntp world {world}: cases {names} match the reference and the one-GPU decode on every rank")
