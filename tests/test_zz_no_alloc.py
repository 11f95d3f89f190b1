"""cngpt_cuda_layernorm_bwd_noalloc: the LayerNorm backward for callers that
cannot let the library allocate device memory (cudaMalloc synchronises the
whole device and fails once the caller has reserved the GPU's memory for its
own pool). Its scratch is a fixed array inside the library instead.

Checked through the C ABI on two calls in a row against the allocating entry
point (layernorm_bwd of cngpt/ops.h on the same device buffers) and against
the oracle's restatement of the reference (orc_layernorm_bwd,
src/ops.c:250-338), with the ops tolerance (normwise 1e-5); that a call at a
new, larger shape leaves the device's free memory unchanged; and the size
limit. This file sorts last so a run that stops at the first failure has run
everything else first.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from cngpt_b200 import abi
from oracle import oracle

pytestmark = pytest.mark.gpu
VP, I = C.c_void_p, C.c_int


def bind(lib):
    fn = lib.cngpt_cuda_layernorm_bwd_noalloc
    fn.restype = I
    fn.argtypes = [VP, VP, VP, VP, VP, VP, VP, VP, I, I]
    return fn


def nwerr(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(float(np.max(np.abs(b))), 1e-30))


def inputs(T, Cc, seed):
    g = np.random.default_rng(seed)
    f = lambda *s: g.standard_normal(s).astype(np.float32)  # noqa: E731
    return dict(x=f(T, Cc), w=f(Cc), b=f(Cc), dout=f(T, Cc), dx0=f(T, Cc), dw0=f(Cc), db0=f(Cc))


def run_three(lib, noalloc, dev, T, Cc, seed):
    """(allocating entry point, no-allocation entry point, oracle) on the same
    inputs; the backward accumulates, so all three start from the same dx, dw, db."""
    h = inputs(T, Cc, seed)
    d = {k: torch.from_numpy(v).to(dev) for k, v in h.items()}
    out = torch.empty(T, Cc, device=dev)
    mean = torch.empty(T, device=dev)
    rstd = torch.empty(T, device=dev)
    lib.layernorm_fwd(d["x"].data_ptr(), d["w"].data_ptr(), d["b"].data_ptr(), out.data_ptr(), mean.data_ptr(),
                      rstd.data_ptr(), T, Cc)
    ref = [d["dx0"].clone(), d["dw0"].clone(), d["db0"].clone()]
    new = [d["dx0"].clone(), d["dw0"].clone(), d["db0"].clone()]
    torch.cuda.synchronize()
    lib.layernorm_bwd(d["dout"].data_ptr(), d["x"].data_ptr(), d["w"].data_ptr(), mean.data_ptr(), rstd.data_ptr(),
                      ref[0].data_ptr(), ref[1].data_ptr(), ref[2].data_ptr(), T, Cc)
    st = noalloc(d["dout"].data_ptr(), d["x"].data_ptr(), d["w"].data_ptr(), mean.data_ptr(), rstd.data_ptr(),
                 new[0].data_ptr(), new[1].data_ptr(), new[2].data_ptr(), T, Cc)
    abi.check(lib, st, "layernorm_bwd_noalloc")
    abi.check(lib, lib.cngpt_cuda_check(), "sync")
    torch.cuda.synchronize()
    # the oracle gets the device's own mean / rstd, so only the backward differs
    mh, rh = mean.cpu().numpy(), rstd.cpu().numpy()
    orc = [h["dx0"].copy(), h["dw0"].copy(), h["db0"].copy()]
    P = oracle.ptr
    oracle.restatement().orc_layernorm_bwd(P(h["dout"]), P(h["x"]), P(h["w"]), P(mh), P(rh), P(orc[0]), P(orc[1]),
                                           P(orc[2]), T, Cc)
    return [t.cpu().numpy() for t in ref], [t.cpu().numpy() for t in new], orc


def test_noalloc_matches_allocating_entry_point_and_oracle_twice(lib, cuda):
    noalloc = bind(lib)
    # two calls in a row; the second reuses the array the first left behind,
    # with a different shape
    for T, Cc, seed in [(4096, 768, 1), (1000, 1600, 2)]:
        ref, new, orc = run_three(lib, noalloc, cuda, T, Cc, seed)
        for name, r, n, o in zip(("dx", "dw", "db"), ref, new, orc):
            assert nwerr(n, r) < 1e-5, (T, Cc, name, nwerr(n, r))
            assert nwerr(n, o) < 1e-5, (T, Cc, name, nwerr(n, o))


def test_noalloc_leaves_free_memory_unchanged(lib, cuda):
    """After one small call (which looks up the array's address), a call at a
    larger shape than any before - one that would make the allocating entry
    point grow its scratch - changes nothing in the device's free memory."""
    noalloc = bind(lib)
    T0, T1, Cc = 64, 12288, 1024
    buf = {T: [torch.randn(T, Cc, device=cuda) for _ in range(3)] + [torch.randn(Cc, device=cuda) for _ in range(3)]
           + [torch.rand(T, device=cuda), torch.rand(T, device=cuda) + 0.5] for T in (T0, T1)}

    def call(T):
        x, dout, dx, w, dw, db, mean, rstd = buf[T]
        return noalloc(dout.data_ptr(), x.data_ptr(), w.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
                       dx.data_ptr(), dw.data_ptr(), db.data_ptr(), T, Cc)
    abi.check(lib, call(T0), "small call")
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    abi.check(lib, call(T1), "large call")
    abi.check(lib, lib.cngpt_cuda_check(), "sync")
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"


def test_noalloc_rejects_oversized_shapes(lib, cuda):
    noalloc = bind(lib)
    dev = torch.zeros(16, device=cuda)
    p = dev.data_ptr()
    # ceil(65536 / 128) * 2 * 4096 = 4,194,304 floats of scratch; the array holds 524,288
    st = noalloc(p, p, p, p, p, p, p, p, 65536, 4096)
    assert st == abi.ERR_ARG
    assert b"static array" in lib.cngpt_cuda_last_message()
    lib.cngpt_cuda_clear_status()
    host = np.zeros(16, np.float32)
    st = noalloc(host.ctypes.data, p, p, p, p, p, p, p, 4, 4)
    assert st == abi.ERR_ARG
    lib.cngpt_cuda_clear_status()
