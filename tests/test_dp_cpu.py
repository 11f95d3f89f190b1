"""Data-parallel training semantics, on CPU (gloo, world size 2).

The GPU path (csrc/dist.cu) averages the gradient arena across ranks after
each rank's backward on its own B x T slice, then clips and steps. Here two
gloo ranks run the same plan with the oracle's restatement
(oracle/cngpt_oracle.c) and check it against one process on the global batch:
the averaged per-rank gradients equal the gradient of the mean loss over the
concatenated batch, and the replicated AdamW keeps the ranks bit-identical.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle

CFG = (2, 4, 32, 64, 16)  # n_layer, n_head, n_embd, vocab, block
B_RANK, T = 2, 8


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def batch(world: int):
    ids = oracle.lcg_tokens(world * B_RANK * T + 1, CFG[3], seed=99)
    return ids[:-1].copy(), ids[1:].copy()


def worker(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    c = oracle.cfg(*CFG)
    p = oracle.init_weights(c, 1234)
    tok, tgt = batch(world)
    n = B_RANK * T
    sl = slice(rank * n, (rank + 1) * n)
    loss, g = oracle.forward_backward(c, p, tok[sl].copy(), tgt[sl].copy(), B_RANK, T)
    gt = torch.from_numpy(g)
    dist.all_reduce(gt, op=dist.ReduceOp.SUM)
    g = (gt / world).numpy().astype(np.float32)
    g_avg = g.copy()  # AdamW clips g in place
    m, v = np.zeros_like(p), np.zeros_like(p)
    oracle.adamw(c, p, g, m, v, 0, 1e-3, 0.9, 0.95, 1e-8, 0.1, 1.0)
    lt = torch.tensor([loss], dtype=torch.float64)
    dist.all_reduce(lt, op=dist.ReduceOp.SUM)
    out[rank] = (g_avg, p, float(lt.item()) / world)
    dist.destroy_process_group()


def test_dp_average_equals_global_batch_gradient():
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(worker, args=(world, free_port(), out), nprocs=world, join=True)
    c = oracle.cfg(*CFG)
    p = oracle.init_weights(c, 1234)
    tok, tgt = batch(world)
    loss, g = oracle.forward_backward(c, p, tok, tgt, world * B_RANK, T)
    g0, p0, l0 = out[0]
    g1, p1, _ = out[1]
    assert np.array_equal(g0, g1) and np.array_equal(p0, p1), "ranks diverged"
    assert abs(l0 - loss) / loss < 1e-6
    assert float(np.max(np.abs(g0 - g)) / np.max(np.abs(g))) < 1e-5
    m, v = np.zeros_like(p), np.zeros_like(p)
    oracle.adamw(c, p, g, m, v, 0, 1e-3, 0.9, 0.95, 1e-8, 0.1, 1.0)
    big = np.abs(g) > 1e-3 * np.abs(g).max()
    assert np.max(np.abs(p0 - p)[big]) < 1e-6
