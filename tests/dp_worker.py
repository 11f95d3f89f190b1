"""One rank of the 2-GPU data-parallel parity test (tests/test_dp_gpu.py),
launched by torchrun. Each rank runs forward + backward of its own slice of
the global batch through libcngpt_cuda, averages the gradient arena over NCCL
(cngpt_cuda_dp_allreduce_grads), takes one AdamW step, and saves its
gradients and parameters for the parent test to compare."""
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
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), grads=g, params=p, loss=np.float32(loss))
    abi.check(lib, lib.cngpt_cuda_dp_free(C.byref(m)), "dp_free")
    lib.gpt_free(C.byref(m))
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
