"""One rank of the tensor-parallel parity tests (tests/test_tp_gpu.py),
launched by torchrun, one process per GPU. Every rank builds the same model
from the same rand() seed, splits it with cngpt_cuda_tp_init, and saves the
gathered final-position logits and the greedy tokens it produced."""
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

# name -> (n_layer, n_head, n_embd, vocab, block, seed), (B, T) forward, (B, T, n_new) decode
CASES = {
    "tp5": ((2, 5, 320, 1001, 64, 11), (3, 40), (2, 12, 20)),
    "tp3": ((3, 3, 96, 77, 32, 5), (2, 17), (3, 5, 9)),
    "xl2": ((2, 25, 1600, 50257, 1024, 3), (2, 48), (2, 16, 8)),
    # batch above the peer-exchange row limit: the decode exchanges go through NCCL
    "tp5w": ((2, 5, 320, 1001, 64, 11), (3, 40), (10, 6, 5)),
    # batch 1: replicated decode by default, the split decode when asked
    "tp5b1": ((2, 5, 320, 1001, 64, 11), (3, 40), (1, 12, 20)),
}


def run(lib, name, world, rank, uid):
    cfg, (fb, ft), (gb, gt, gn) = CASES[name]
    m = abi.GPT()
    assert lib.gpt_init(C.byref(m), abi.GPTConfig(*cfg[:5], 0.0)) == 0
    oracle.libc_rand_stream(cfg[5])
    lib.gpt_init_weights(C.byref(m))
    abi.check(lib, lib.cngpt_cuda_tp_init(C.byref(m), uid, world, rank), "tp_init")
    tok = oracle.lcg_tokens(fb * ft, cfg[3], seed=100 + fb * ft)
    logits = np.zeros(fb * cfg[3], np.float32)
    abi.check(lib, lib.cngpt_cuda_tp_forward_last(C.byref(m), tok.ctypes.data, fb, ft, logits.ctypes.data),
              "tp_forward_last")
    prompt = oracle.lcg_tokens(gb * gt, cfg[3], seed=7)
    out = np.zeros(gb * gn, np.int32)
    abi.check(lib, lib.cngpt_cuda_tp_generate(C.byref(m), prompt.ctypes.data, gb, gt, gn, out.ctypes.data),
              "tp_generate")
    # the split decode, whatever the batch
    split = np.zeros(gb * gn, np.int32)
    abi.check(lib, lib.cngpt_cuda_tp_set_decode_mode(C.byref(m), 1), "decode mode")
    abi.check(lib, lib.cngpt_cuda_tp_generate(C.byref(m), prompt.ctypes.data, gb, gt, gn, split.ctypes.data),
              "tp_generate split")
    abi.check(lib, lib.cngpt_cuda_tp_free(C.byref(m)), "tp_free")
    lib.gpt_free(C.byref(m))
    return logits.reshape(fb, -1), out.reshape(gb, gn), split.reshape(gb, gn)


def main(out_dir: str, names: list[str]):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo", timeout=timedelta(seconds=120))
    lib = abi.load()
    lib.cngpt_cuda_set_precision(abi.PREC_3XTF32)
    res = {}
    for name in names:
        uid = (C.c_ubyte * 128)()
        if rank == 0:
            abi.check(lib, lib.cngpt_cuda_dp_unique_id(uid), "uid")
        obj = [bytes(uid)]
        dist.broadcast_object_list(obj, src=0)
        uid = (C.c_ubyte * 128).from_buffer_copy(obj[0])
        res[name + "_logits"], res[name + "_tokens"], res[name + "_split"] = run(lib, name, world, rank, uid)
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **res)
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2:])
