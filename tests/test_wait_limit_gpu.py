"""Bounded device waits that run out, on one GPU.

The tensor-parallel decode exchange waits on flags that the peers raise over
NVLink (tp_reduce_kernel). Here the flag belongs to a receive buffer of world 1
that nothing ever publishes, so the wait must give up after the wait limit,
record its site (DEV_ERR_TP_FLAG = 201), leave x untouched, and leave the
context usable: the next call, with the flag raised, must complete and give
the exact sum and LayerNorm statistics.
"""
import ctypes as C
import time

import numpy as np
import pytest
import torch

from cngpt_b200 import abi

pytestmark = pytest.mark.gpu


@pytest.fixture
def short_wait(lib):
    abi.check(lib, lib.cngpt_cuda_set_wait_limit_ns(20_000_000), "set wait limit")  # 20 ms
    yield
    abi.check(lib, lib.cngpt_cuda_set_wait_limit_ns(0), "restore wait limit")


def test_unpublished_flag_times_out_and_next_call_works(lib, cuda, short_wait):
    rows, Cc = 3, 1600
    g = torch.Generator().manual_seed(5)
    part = torch.randn(rows, Cc, generator=g).to(cuda)
    x0 = torch.full((rows, Cc), 7.0, device=cuda)
    x = x0.clone()
    stats = torch.full((rows, 2), -1.0, device=cuda)
    lib.cngpt_cuda_clear_status()
    t0 = time.perf_counter()
    st = lib.cngpt_cuda_selftest_tp_reduce(x.data_ptr(), part.data_ptr(), rows, Cc, 0, stats.data_ptr())
    dt = time.perf_counter() - t0
    assert st == abi.ERR_DEVICE_WAIT, lib.cngpt_cuda_last_message()
    assert b"site 201" in lib.cngpt_cuda_last_message()
    assert dt < 1.5, f"the 20 ms limit took {dt:.2f} s to end the wait"
    torch.cuda.synchronize()
    assert torch.equal(x, x0), "x must be left unchanged when the exchange gives up"
    assert torch.all(stats == -1.0)
    # the error word was read and cleared: nothing is pending
    lib.cngpt_cuda_clear_status()
    assert lib.cngpt_cuda_check() == abi.OK
    # the same context runs the exchange once the flag is raised
    st = lib.cngpt_cuda_selftest_tp_reduce(x.data_ptr(), part.data_ptr(), rows, Cc, 1, stats.data_ptr())
    abi.check(lib, st, "published exchange")
    torch.cuda.synchronize()
    assert torch.equal(x, part)
    p = part.double().cpu().numpy()
    mean = p.mean(axis=1)
    rstd = 1.0 / np.sqrt(((p - mean[:, None]) ** 2).mean(axis=1) + 1e-5)
    s = stats.double().cpu().numpy()
    assert np.allclose(s[:, 0], mean, rtol=0, atol=1e-6)
    assert np.allclose(s[:, 1], rstd, rtol=1e-5)


def test_wait_limit_restores_default(lib, cuda):
    """0 restores the 2 s default; a published exchange is unaffected by the limit."""
    abi.check(lib, lib.cngpt_cuda_set_wait_limit_ns(0), "default")
    part = torch.ones(1, 64, device=cuda)
    x = torch.zeros(1, 64, device=cuda)
    stats = torch.zeros(1, 2, device=cuda)
    abi.check(lib, lib.cngpt_cuda_selftest_tp_reduce(x.data_ptr(), part.data_ptr(), 1, 64, 1, stats.data_ptr()),
              "exchange")
    torch.cuda.synchronize()
    assert torch.equal(x, part)


def test_selftest_rejects_bad_arguments(lib, cuda):
    x = torch.zeros(16, device=cuda)
    host = np.zeros(16, np.float32)
    for args in [(x.data_ptr(), x.data_ptr(), 9, 4, 1, x.data_ptr()),      # rows > 8
                 (x.data_ptr(), x.data_ptr(), 1, 4096, 1, x.data_ptr()),   # C > 2048
                 (host.ctypes.data, x.data_ptr(), 1, 4, 1, x.data_ptr())]:  # host pointer
        lib.cngpt_cuda_clear_status()
        assert lib.cngpt_cuda_selftest_tp_reduce(*args) == abi.ERR_ARG
    lib.cngpt_cuda_clear_status()
