"""Inference path parity: gpt_forward_fast (src/fast.c:227-333), the KV-cache
greedy decode (cngpt_cuda_generate) and gpt_sample (src/model.c:991-1016)
against the reference's CPU build on identical seeded weights.

Tolerances: last-position logits normwise 1e-5 (3xTF32), 2e-3 (TF32).
Greedy ids: every device token must be the reference's argmax of the
full-prefix logits (teacher-forced on the device's own prefix: one causal
reference forward over the window gives the final-position logits of every
prefix), unless that position is a near-tie - the reference's top-1 and the
device's token within 1e-4 x max|logit| of each other - which the test counts
and reports.
"""
import ctypes as C

import numpy as np
import pytest

from cngpt_b200 import abi
from oracle import oracle
from tests.models import CudaModel, RefModel, nwerr

pytestmark = pytest.mark.gpu

CONFIGS = {
    "fast": dict(L=3, H=4, C=32, V=70, block=16, seed=42),      # tests/check_fast.c:29-33
    "hs64": dict(L=2, H=2, C=128, V=96, block=128, seed=7),
    "small1": dict(L=1, H=12, C=768, V=50257, block=1024, seed=None),
}


def pair(lib, name):
    c = CONFIGS[name]
    args = (c["L"], c["H"], c["C"], c["V"], c["block"], c["seed"])
    return RefModel(*args), CudaModel(lib, *args), c


def ref_fast(ref, tok, B, T):
    fc = abi.FastCtx()
    ref.lib.fast_init(C.byref(fc))
    p = ref.lib.gpt_forward_fast(C.byref(ref.m), C.byref(fc), tok.ctypes.data, B, T)
    out = np.ctypeslib.as_array(p, shape=(B * ref.cfg.vocab_size,)).copy()
    ref.lib.fast_free(C.byref(fc))
    return out.reshape(B, -1)


def dev_fast(lib, dev, tok, B, T):
    fc = abi.FastCtx()
    lib.fast_init(C.byref(fc))
    p = lib.gpt_forward_fast(C.byref(dev.m), C.byref(fc), tok.ctypes.data, B, T)
    assert p, lib.cngpt_cuda_last_message()
    out = dev._d2h(p, B * dev.cfg.vocab_size).reshape(B, -1)
    lib.fast_free(C.byref(fc))
    return out


@pytest.mark.parametrize("prec,tol", [(abi.PREC_3XTF32, 1e-5), (abi.PREC_TF32, 2e-3)], ids=["3xtf32", "tf32"])
@pytest.mark.parametrize("name,shapes", [("fast", [(1, 1), (1, 9), (2, 6), (3, 16), (1, 16)]),
                                         ("hs64", [(1, 1), (2, 100), (3, 128)]),
                                         ("small1", [(2, 100)])])
def test_forward_fast_matches_reference(lib, cuda, prec, tol, name, shapes):
    lib.cngpt_cuda_set_precision(prec)
    try:
        ref, dev, c = pair(lib, name)
        for B, T in shapes:
            tok = oracle.lcg_tokens(B * T, c["V"], seed=100 + B * T)
            r = ref_fast(ref, tok, B, T)
            d = dev_fast(lib, dev, tok, B, T)
            assert nwerr(d, r) < tol, (B, T, nwerr(d, r))
            # same rows from the device's own straightforward forward
            dev.forward(tok, None, B, T)
            full = dev.logits(B, T)[:, T - 1, :]
            assert nwerr(d, full) < tol
        ref.free()
        dev.free()
    finally:
        lib.cngpt_cuda_set_precision(abi.PREC_3XTF32)


@pytest.mark.parametrize("name,B,T,n_new", [("hs64", 2, 20, 40), ("small1", 1, 16, 12), ("fast", 3, 5, 11)])
def test_generate_greedy_matches_full_prefix_argmax(lib, cuda, name, B, T, n_new):
    ref, dev, c = pair(lib, name)
    prompt = oracle.lcg_tokens(B * T, c["V"], seed=7)
    out = np.zeros(B * n_new, np.int32)
    fc = abi.FastCtx()
    lib.fast_init(C.byref(fc))
    abi.check(lib, lib.cngpt_cuda_generate(C.byref(dev.m), C.byref(fc), prompt.ctypes.data, B, T, n_new,
                                           out.ctypes.data), "generate")
    lib.fast_free(C.byref(fc))
    out = out.reshape(B, n_new)
    # step i's token is the argmax of the final-position logits of the prefix
    # [0, T + i): one causal forward of the reference over the whole window
    # (the device's own prefix) gives every such row at once (row T - 1 + i)
    S = T + n_new - 1
    seq = np.concatenate([prompt.reshape(B, T), out[:, :-1]], axis=1).astype(np.int32).ravel()
    ref.forward(seq, None, B, S)
    lgs = ref.logits(B, S)[:, T - 1:, :]
    ties = 0
    for b in range(B):
        for i in range(n_new):
            lg = lgs[b, i]
            top = int(np.argmax(lg))
            got = int(out[b, i])
            if got != top:
                margin = lg[top] - lg[got]
                assert margin <= 1e-4 * np.max(np.abs(lg)), (b, i, top, got, margin)
                ties += 1
    print(f"\n[{name}] {B}x{n_new} greedy tokens, {ties} near-tie(s)")
    assert ties <= max(1, (B * n_new) // 20)
    ref.free()
    dev.free()


def test_generate_rejects_too_long(lib, cuda):
    dev = CudaModel(lib, 1, 2, 64, 50, 16, 3)
    prompt = np.zeros(10, np.int32)
    out = np.zeros(10, np.int32)
    fc = abi.FastCtx()
    lib.fast_init(C.byref(fc))
    st = lib.cngpt_cuda_generate(C.byref(dev.m), C.byref(fc), prompt.ctypes.data, 1, 10, 8, out.ctypes.data)
    assert st == abi.ERR_ARG
    lib.cngpt_cuda_clear_status()
    lib.fast_free(C.byref(fc))
    dev.free()


def test_sample_matches_reference_stream(lib, cuda):
    """gpt_sample: same rand() stream, same top-k sampling steps -> same tokens"""
    c = dict(L=2, H=4, C=32, V=64, block=16, seed=1234)
    args = (c["L"], c["H"], c["C"], c["V"], c["block"], c["seed"])
    ref, dev = RefModel(*args), CudaModel(lib, *args)
    prompt = np.array([1, 2, 3], np.int32)
    n = 20  # crosses block_size: exercises the context crop (src/model.c:1003-1007)
    for temp, k in [(1.0, 0), (0.8, 5), (1.0, 1)]:
        out_r = np.zeros(3 + n, np.int32)
        out_d = np.zeros(3 + n, np.int32)
        oracle.libc_rand_stream(5)
        ref.lib.gpt_sample(C.byref(ref.m), prompt.ctypes.data, 3, out_r.ctypes.data, n, temp, k)
        oracle.libc_rand_stream(5)
        lib.gpt_sample(C.byref(dev.m), prompt.ctypes.data, 3, out_d.ctypes.data, n, temp, k)
        assert np.array_equal(out_r, out_d), (temp, k, out_r, out_d)
    ref.free()
    dev.free()


@pytest.mark.parametrize("temp,k", [(1.0, 0), (0.8, 10), (1.0, 1)])
def test_sample_kv_cache_matches_reference_stream(lib, cuda, temp, k):
    """gpt_sample on a head-size-64 model: 80 new tokens, all within
    block_size, so every step after the prompt runs through the KV cache;
    same rand() stream, same tokens as the reference's full-prefix loop."""
    ref, dev, c = pair(lib, "hs64")
    prompt = oracle.lcg_tokens(20, c["V"], seed=4)
    n = 80
    out_r = np.zeros(20 + n, np.int32)
    out_d = np.zeros(20 + n, np.int32)
    oracle.libc_rand_stream(11)
    ref.lib.gpt_sample(C.byref(ref.m), prompt.ctypes.data, 20, out_r.ctypes.data, n, temp, k)
    oracle.libc_rand_stream(11)
    launches = lib.cngpt_cuda_launch_count()
    lib.gpt_sample(C.byref(dev.m), prompt.ctypes.data, 20, out_d.ctypes.data, n, temp, k)
    launches = lib.cngpt_cuda_launch_count() - launches
    assert np.array_equal(out_r, out_d), (temp, k, np.nonzero(out_r != out_d))
    # a full-prefix recompute launches at least 7 kernels per layer per token;
    # the cached decode step launches 5 per layer plus 3 (embedding, LM head,
    # token bookkeeping)
    assert launches <= n * (5 * c["L"] + 3) + 100, launches
    ref.free()
    dev.free()


@pytest.mark.parametrize("name,B", [("hs64", 1), ("hs64", 3), ("small1", 8)])
def test_decode_step_kernel(lib, cuda, name, B):
    """With the single-launch decode step enabled, sequences up to 8 with head
    size 64 decode each token in one cooperative launch (all layers, the LM
    head and the greedy pick), and a 16-token greedy window gives the same
    tokens as the kernel-chain decode."""
    ref, dev, c = pair(lib, name)
    ref.free()
    prompt = oracle.lcg_tokens(B * 8, c["V"], seed=2)
    fc = abi.FastCtx()
    lib.fast_init(C.byref(fc))
    toks = {}
    try:
        for on in (1, 0):
            lib.cngpt_cuda_set_decode_step_kernel(on)
            counts = []
            for n in (1, 2, 16):
                out = np.zeros(B * n, np.int32)
                l0 = lib.cngpt_cuda_launch_count()
                abi.check(lib, lib.cngpt_cuda_generate(C.byref(dev.m), C.byref(fc), prompt.ctypes.data, B, 8, n,
                                                       out.ctypes.data), "generate")
                counts.append(lib.cngpt_cuda_launch_count() - l0)
            toks[on] = out.copy()
            if on:
                assert counts[1] - counts[0] == 1, counts  # n = 2 adds one eager decode step
            else:
                assert counts[1] - counts[0] > 1, counts  # the kernel chain
    finally:
        lib.cngpt_cuda_set_decode_step_kernel(0)
    lib.fast_free(C.byref(fc))
    dev.free()
    assert np.array_equal(toks[1], toks[0])
