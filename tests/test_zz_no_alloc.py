"""cngpt_cuda_layernorm_bwd_noalloc: the LayerNorm backward for callers that
cannot let the library allocate device memory (cudaMalloc synchronises the
whole device and fails once the caller has reserved the GPU's memory for its
own pool). Its scratch is a fixed array inside the library instead.

Checked through the C ABI against the allocating entry point (layernorm_bwd of
cngpt/ops.h on the same device buffers) on two calls in a row, with the test
suite's ops tolerance (normwise 1e-5), plus the size limit. This file sorts
last so a run that stops at the first failure has run everything else first.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from cngpt_b200 import abi

pytestmark = pytest.mark.gpu
VP, I = C.c_void_p, C.c_int


def bind(lib):
    fn = lib.cngpt_cuda_layernorm_bwd_noalloc
    fn.restype = I
    fn.argtypes = [VP, VP, VP, VP, VP, VP, VP, VP, I, I]
    return fn


def nwerr(a, b):
    a, b = a.double(), b.double()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def run_pair(lib, noalloc, dev, T, Cc, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, Cc, generator=g).to(dev)
    w = torch.randn(Cc, generator=g).to(dev)
    b = torch.randn(Cc, generator=g).to(dev)
    dout = torch.randn(T, Cc, generator=g).to(dev)
    out = torch.empty(T, Cc, device=dev)
    mean = torch.empty(T, device=dev)
    rstd = torch.empty(T, device=dev)
    lib.layernorm_fwd(x.data_ptr(), w.data_ptr(), b.data_ptr(), out.data_ptr(), mean.data_ptr(),
                      rstd.data_ptr(), T, Cc)
    # the backward accumulates: both entry points start from the same values
    dx0 = torch.randn(T, Cc, generator=g).to(dev)
    dw0 = torch.randn(Cc, generator=g).to(dev)
    db0 = torch.randn(Cc, generator=g).to(dev)
    ref = [dx0.clone(), dw0.clone(), db0.clone()]
    new = [dx0.clone(), dw0.clone(), db0.clone()]
    lib.layernorm_bwd(dout.data_ptr(), x.data_ptr(), w.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
                      ref[0].data_ptr(), ref[1].data_ptr(), ref[2].data_ptr(), T, Cc)
    st = noalloc(dout.data_ptr(), x.data_ptr(), w.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
                 new[0].data_ptr(), new[1].data_ptr(), new[2].data_ptr(), T, Cc)
    abi.check(lib, st, "layernorm_bwd_noalloc")
    abi.check(lib, lib.cngpt_cuda_check(), "sync")
    torch.cuda.synchronize()
    return ref, new


def test_noalloc_matches_allocating_entry_point_twice(lib, cuda):
    noalloc = bind(lib)
    # two calls in a row; the second reuses the array the first left behind,
    # with a different shape
    for T, Cc, seed in [(4096, 768, 1), (1000, 1600, 2)]:
        ref, new = run_pair(lib, noalloc, cuda, T, Cc, seed)
        for r, n in zip(ref, new):
            assert nwerr(n, r) < 1e-5


def test_noalloc_rejects_oversized_shapes(lib, cuda):
    noalloc = bind(lib)
    dev = torch.zeros(16, device=cuda)
    p = dev.data_ptr()
    st = noalloc(p, p, p, p, p, p, p, p, 65536, 4096)  # needs 2M floats of scratch
    assert st == abi.ERR_ARG
    assert b"static array" in lib.cngpt_cuda_last_message()
    lib.cngpt_cuda_clear_status()
    host = np.zeros(16, np.float32)
    st = noalloc(host.ctypes.data, p, p, p, p, p, p, p, 4, 4)
    assert st == abi.ERR_ARG
    lib.cngpt_cuda_clear_status()
