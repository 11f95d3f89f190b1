"""Training checkpoints (cngpt_cuda_save_checkpoint / load_checkpoint): a
model restored from a checkpoint continues training bit-for-bit like the
model that wrote it (deterministic kernels, same optimizer moments and step),
and the file stays readable by gpt_load as a plain model file - by this
library and by the reference's own gpt_load (src/model.c:179-231)."""
import ctypes as C
import os
import tempfile

import numpy as np
import pytest

from cngpt_b200 import abi
from oracle import oracle
from tests.models import CudaModel, RefModel

pytestmark = pytest.mark.gpu

CFG = (2, 2, 128, 96, 64)
B, T = 2, 32


def steps(lib, m, ids, n):
    losses = []
    for i in range(n):
        tok = ids[i * B * T:(i + 1) * B * T].copy()
        tgt = ids[i * B * T + 1:(i + 1) * B * T + 1].copy()
        loss = C.c_float()
        abi.check(lib, lib.cngpt_cuda_train_step(C.byref(m), tok.ctypes.data, tgt.ctypes.data, B, T, 1e-3, 0.9,
                                                 0.95, 1e-8, 0.1, 1.0, C.byref(loss)), "train_step")
        losses.append(loss.value)
    return losses


def test_resume_is_bit_identical(lib, cuda):
    ids = oracle.lcg_tokens(8 * B * T + 1, CFG[3], seed=9)
    a = CudaModel(lib, *CFG, 21)
    steps(lib, a.m, ids, 3)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "ck.bin").encode()
        abi.check(lib, lib.cngpt_cuda_save_checkpoint(C.byref(a.m), path), "save")
        saved = a.params()
        cont_a = steps(lib, a.m, ids[3 * B * T:], 3)
        b = abi.GPT()  # empty: configuration from the file
        abi.check(lib, lib.cngpt_cuda_load_checkpoint(C.byref(b), path), "load")
        assert b.step == 3
        cont_b = steps(lib, b, ids[3 * B * T:], 3)
        pb = np.empty(b.n_params, np.float32)
        abi.check(lib, lib.cngpt_cuda_params_to_host(C.byref(b), pb.ctypes.data), "params")
        assert cont_a == cont_b, (cont_a, cont_b)
        assert np.array_equal(pb, a.params())
        # still a model file for gpt_load: parameters only
        c = abi.GPT()
        assert lib.gpt_load(C.byref(c), path) == 0
        pc = np.empty(c.n_params, np.float32)
        abi.check(lib, lib.cngpt_cuda_params_to_host(C.byref(c), pc.ctypes.data), "params")
        assert np.array_equal(pc, saved)
        ref = RefModel(*CFG, 21)
        assert ref.lib.gpt_load(C.byref(ref.m), path) == 0
        assert np.array_equal(ref.params(), saved)
        ref.free()
        lib.gpt_free(C.byref(b))
        lib.gpt_free(C.byref(c))
    a.free()


def test_plain_model_file_loads_with_fresh_optimizer(lib, cuda):
    a = CudaModel(lib, *CFG, 5)
    ids = oracle.lcg_tokens(2 * B * T + 1, CFG[3], seed=3)
    steps(lib, a.m, ids, 2)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "model.bin").encode()
        assert lib.gpt_save(C.byref(a.m), path) == 0
        b = abi.GPT()
        abi.check(lib, lib.cngpt_cuda_load_checkpoint(C.byref(b), path), "load")
        assert b.step == 0
        mb = np.empty(b.n_params, np.float32)
        abi.check(lib, lib.cngpt_cuda_copy(mb.ctypes.data, C.cast(b.m_buf, C.c_void_p), mb.nbytes), "m")
        assert not mb.any()
        lib.gpt_free(C.byref(b))
        wrong = CudaModel(lib, 1, 2, 64, 50, 16, 3)
        assert lib.cngpt_cuda_load_checkpoint(C.byref(wrong.m), path) == abi.ERR_ARG
        lib.cngpt_cuda_clear_status()
        wrong.free()
    a.free()


def test_truncated_trailer_leaves_model_unchanged(lib, cuda):
    """A checkpoint cut off inside the optimizer moments is rejected and the
    model keeps its parameters, moments and step count."""
    a = CudaModel(lib, *CFG, 5)
    ids = oracle.lcg_tokens(2 * B * T + 1, CFG[3], seed=3)
    steps(lib, a.m, ids, 2)
    b = CudaModel(lib, *CFG, 9)
    steps(lib, b.m, ids, 1)
    p0 = b.params()
    m0 = np.empty(b.n, np.float32)
    abi.check(lib, lib.cngpt_cuda_copy(m0.ctypes.data, C.cast(b.m.m_buf, C.c_void_p), m0.nbytes), "m")
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "ckpt.bin")
        abi.check(lib, lib.cngpt_cuda_save_checkpoint(C.byref(a.m), path.encode()), "save")
        full = open(path, "rb").read()
        with open(path, "wb") as f:
            f.write(full[:len(full) - 4 * (a.n // 2)])  # stop inside the second moments
        assert lib.cngpt_cuda_load_checkpoint(C.byref(b.m), path.encode()) == abi.ERR_ARG
        assert b"truncated" in lib.cngpt_cuda_last_message()
        lib.cngpt_cuda_clear_status()
    assert b.m.step == 1
    assert np.array_equal(b.params(), p0)
    m1 = np.empty(b.n, np.float32)
    abi.check(lib, lib.cngpt_cuda_copy(m1.ctypes.data, C.cast(b.m.m_buf, C.c_void_p), m1.nbytes), "m")
    assert np.array_equal(m1, m0)
    a.free()
    b.free()
