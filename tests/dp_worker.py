"""One rank of the data-parallel parity tests (tests/test_dp_gpu.py),
launched by torchrun. Each rank runs forward + backward of its own slice of
the global batch through libcngpt_cuda, averages the gradient arena over NCCL
(cngpt_cuda_dp_allreduce_grads) and takes one AdamW step; then, on a fresh
model, cngpt_cuda_train_step with its per-layer buckets overlapped with the
backward (lr 0, then three real steps). It saves gradients, parameters and
losses for the parent test to compare."""
import ctypes as C
import os
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from cngpt_b200 import abi  # noqa: E402
from oracle import oracle  # noqa: E402

CFG = (2, 2, 128, 96, 128)
B, T = 2, 64


def main(out_dir: str):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    lib = abi.load()
    m = abi.GPT()
    assert lib.gpt_init(C.byref(m), abi.GPTConfig(*CFG, 0.0)) == 0
    oracle.libc_rand_stream(7)
    lib.gpt_init_weights(C.byref(m))
    uid = (C.c_ubyte * 128)()
    if rank == 0:
        abi.check(lib, lib.cngpt_cuda_dp_unique_id(uid), "uid")
    obj = [bytes(uid)]
    dist.broadcast_object_list(obj, src=0)
    uid = (C.c_ubyte * 128).from_buffer_copy(obj[0])
    abi.check(lib, lib.cngpt_cuda_dp_init(C.byref(m), uid, world, rank), "dp_init")
    ids = oracle.lcg_tokens(world * B * T + 1, CFG[3], seed=31)
    n = B * T
    tok, tgt = ids[rank * n:(rank + 1) * n].copy(), ids[rank * n + 1:(rank + 1) * n + 1].copy()
    lib.gpt_zero_grad(C.byref(m))
    loss = lib.gpt_forward(C.byref(m), tok.ctypes.data, tgt.ctypes.data, B, T)
    lib.gpt_backward(C.byref(m), tok.ctypes.data, tgt.ctypes.data, B, T)
    abi.check(lib, lib.cngpt_cuda_dp_allreduce_grads(C.byref(m)), "allreduce")
    g = np.empty(m.n_params, np.float32)
    abi.check(lib, lib.cngpt_cuda_grads_to_host(C.byref(m), g.ctypes.data), "grads")
    lib.gpt_adamw(C.byref(m), 1e-3, 0.9, 0.95, 1e-8, 0.1, 1.0)
    p = np.empty(m.n_params, np.float32)
    abi.check(lib, lib.cngpt_cuda_params_to_host(C.byref(m), p.ctypes.data), "params")
    abi.check(lib, lib.cngpt_cuda_dp_free(C.byref(m)), "dp_free")
    lib.gpt_free(C.byref(m))
    # the training step's bucketed average (overlapped with the backward): with
    # lr = 0 and no clipping the arena keeps the averaged gradients
    m = abi.GPT()
    assert lib.gpt_init(C.byref(m), abi.GPTConfig(*CFG, 0.0)) == 0
    oracle.libc_rand_stream(7)
    lib.gpt_init_weights(C.byref(m))
    uid = (C.c_ubyte * 128)()  # a communicator id serves one ncclCommInitRank round only
    if rank == 0:
        abi.check(lib, lib.cngpt_cuda_dp_unique_id(uid), "uid")
    obj = [bytes(uid)]
    dist.broadcast_object_list(obj, src=0)
    uid = (C.c_ubyte * 128).from_buffer_copy(obj[0])
    abi.check(lib, lib.cngpt_cuda_dp_init(C.byref(m), uid, world, rank), "dp_init")
    ts_loss = C.c_float()
    abi.check(lib, lib.cngpt_cuda_train_step(C.byref(m), tok.ctypes.data, tgt.ctypes.data, B, T, 0.0, 0.9, 0.95,
                                             1e-8, 0.0, 0.0, C.byref(ts_loss)), "train_step lr 0")
    ts_loss0 = ts_loss.value
    ts_g = np.empty(m.n_params, np.float32)
    abi.check(lib, lib.cngpt_cuda_grads_to_host(C.byref(m), ts_g.ctypes.data), "grads")
    # then real steps: every rank must hold the same parameters
    for _ in range(3):
        abi.check(lib, lib.cngpt_cuda_train_step(C.byref(m), tok.ctypes.data, tgt.ctypes.data, B, T, 1e-3, 0.9, 0.95,
                                                 1e-8, 0.1, 1.0, C.byref(ts_loss)), "train_step")
    ts_p = np.empty(m.n_params, np.float32)
    abi.check(lib, lib.cngpt_cuda_params_to_host(C.byref(m), ts_p.ctypes.data), "params")
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), grads=g, params=p, loss=np.float32(loss), ts_grads=ts_g,
             ts_params=ts_p, ts_loss=np.float32(ts_loss.value), ts_loss0=np.float32(ts_loss0))
    abi.check(lib, lib.cngpt_cuda_dp_free(C.byref(m)), "dp_free")
    lib.gpt_free(C.byref(m))
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
