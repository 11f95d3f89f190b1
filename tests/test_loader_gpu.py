"""cngpt_cuda_loader_*: the device batch sequence equals the reference's own
DataLoader (src/dataloader.c:19-82) over the same uint16 token file, across
several rewinds and a reset; and training from the loader's device batches is
bit-identical to training from the reference loader's host arrays.
"""
import ctypes as C

import numpy as np
import pytest

from cngpt_b200 import abi
from oracle import oracle
from tests.models import CudaModel

pytestmark = pytest.mark.gpu


class Loader:
    def __init__(self, lib, data: np.ndarray, B: int, T: int):
        self.lib, self.data, self.B, self.T = lib, data, B, T  # data stays referenced
        self.h = C.c_void_p()
        abi.check(lib, lib.cngpt_cuda_loader_create(C.byref(self.h), data.ctypes.data, data.size, B, T), "create")

    def next(self):
        i, t = C.c_void_p(), C.c_void_p()
        abi.check(self.lib, self.lib.cngpt_cuda_loader_next(self.h, C.byref(i), C.byref(t)), "next")
        return i.value, t.value

    def fetch(self, p):
        out = np.empty(self.B * self.T, np.int32)
        abi.check(self.lib, self.lib.cngpt_cuda_copy(out.ctypes.data, p, out.nbytes), "d2h")
        return out

    def free(self):
        self.lib.cngpt_cuda_loader_free(self.h)


@pytest.mark.parametrize("B,T,N", [(4, 64, 4 * 64 * 5 + 17), (2, 33, 2 * 33 + 1), (8, 1024, 8 * 1024 * 3 + 100)])
def test_loader_matches_reference_dataloader(lib, cuda, tmp_path, B, T, N):
    data = np.random.default_rng(N).integers(0, 50257, N, dtype=np.uint16)
    path = tmp_path / "tokens.bin"
    data.tofile(path)
    n = 3 * (N // (B * T)) + 3
    ref = oracle.reference_batches(str(path), B, T, n)
    mm = np.fromfile(path, dtype=np.uint16)
    dl = Loader(lib, mm, B, T)
    assert lib.cngpt_cuda_loader_num_batches(dl.h) == N // (B * T)
    for k, (ri, rt) in enumerate(ref):
        pi, pt = dl.next()
        assert np.array_equal(dl.fetch(pi), ri), k
        assert np.array_equal(dl.fetch(pt), rt), k
    # reset: the sequence starts again from the first batch
    abi.check(lib, lib.cngpt_cuda_loader_reset(dl.h), "reset")
    for k in range(2):
        pi, pt = dl.next()
        assert np.array_equal(dl.fetch(pi), ref[k][0])
        assert np.array_equal(dl.fetch(pt), ref[k][1])
    dl.free()


def test_training_from_loader_equals_host_batches(lib, cuda, tmp_path):
    """Three train steps fed by the loader (no synchronisation between steps:
    the next batch uploads while the step runs) against the same steps fed
    with the reference loader's host arrays."""
    cfg = (2, 2, 128, 96, 64)
    B, T = 4, 64
    data = np.random.default_rng(1).integers(0, cfg[3], B * T * 3 + 1, dtype=np.uint16)
    path = tmp_path / "tokens.bin"
    data.tofile(path)
    ref = oracle.reference_batches(str(path), B, T, 5)
    a, b = CudaModel(lib, *cfg, 3), CudaModel(lib, *cfg, 3)
    dl = Loader(lib, data, B, T)
    opt = (1e-3, 0.9, 0.95, 1e-8, 0.1, 1.0)
    for k in range(5):
        pi, pt = dl.next()
        abi.check(lib, lib.cngpt_cuda_train_step(C.byref(a.m), pi, pt, B, T, *opt, None), "loader step")
        ti, tt = ref[k]
        abi.check(lib, lib.cngpt_cuda_train_step(C.byref(b.m), ti.ctypes.data, tt.ctypes.data, B, T, *opt, None),
                  "host step")
    la, lb = C.c_float(), C.c_float()
    abi.check(lib, lib.cngpt_cuda_last_loss(C.byref(a.m), C.byref(la)), "loss")
    abi.check(lib, lib.cngpt_cuda_last_loss(C.byref(b.m), C.byref(lb)), "loss")
    assert la.value == lb.value
    assert np.array_equal(a.params(), b.params())
    dl.free()
    a.free()
    b.free()


def test_loader_rejects_short_data(lib, cuda):
    data = np.zeros(64, np.uint16)
    h = C.c_void_p()
    assert lib.cngpt_cuda_loader_create(C.byref(h), data.ctypes.data, data.size, 8, 8) == abi.ERR_ARG
    assert not h.value
    lib.cngpt_cuda_clear_status()
