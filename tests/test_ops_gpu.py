"""cngpt/ops.h entry points of libcngpt_cuda against the oracle.

Each function is called twice: with plain host arrays (the library stages
them through the device, as the reference's tests/check_ops.c needs) and
with device pointers. Known answers are the ones tests/check_ops.c:69-248
pins; random cases are compared with the C restatement.
Tolerance: normwise 1e-5 (3xTF32 default precision; CUDA-core kernels for
the non-GEMM ops compute in fp32 like the reference).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from cngpt_b200 import abi
from oracle import oracle
from tests.models import nwerr

pytestmark = pytest.mark.gpu
P = oracle.ptr
f32 = np.float32


def rnd(*shape, seed=0):
    return np.random.default_rng(seed).standard_normal(shape).astype(f32)


def test_check_ops_known_answers_host_pointers(lib, cuda):
    X = np.array([1, 0, 0, 1], f32); W = np.array([2, 3, 4, 5], f32); b = np.array([1, -1], f32)
    Y = np.zeros(4, f32)
    lib.linear_fwd(P(X), P(W), P(b), P(Y), 2, 2, 2)
    assert np.allclose(Y, [3, 3, 4, 4], atol=1e-5)
    dX = np.zeros(4, f32)
    lib.linear_bwd_dx(P(X), P(W), P(dX), 2, 2, 2)
    assert np.allclose(dX, [2, 3, 4, 5], atol=1e-5)
    x = np.array([1, 2, 3, 4], f32); w = np.ones(4, f32); bb = np.zeros(4, f32)
    out, mean, rstd = np.zeros(4, f32), np.zeros(1, f32), np.zeros(1, f32)
    lib.layernorm_fwd(P(x), P(w), P(bb), P(out), P(mean), P(rstd), 1, 4)
    assert abs(mean[0] - 2.5) < 1e-4
    assert np.allclose(out, [-1.3416, -0.4472, 0.4472, 1.3416], atol=1e-3)
    g = np.array([0, 1, -1, 2], f32); go = np.zeros(4, f32)
    lib.gelu_fwd(P(g), P(go), 4)
    assert np.allclose(go, [0, 0.8413, -0.1587, 1.9545], atol=1e-3)
    s = np.array([1, 2, 3, 100, 100, 100], f32)
    lib.softmax_inplace(P(s), 2, 3)
    assert np.allclose(s[:3], [0.0900, 0.2447, 0.6652], atol=1e-3)
    assert np.allclose(s[3:], 1 / 3, atol=1e-5)
    lg = np.array([10, 0, 0, 10], f32); tg = np.array([0, 1], np.int32)
    pr, loss = np.zeros(4, f32), np.zeros(1, f32)
    lib.cross_entropy_fwd(P(lg), P(tg), P(pr), P(loss), 1, 2, 2)
    assert loss[0] < 0.01 and pr[0] > 0.99 and pr[3] > 0.99
    assert lib.cngpt_cuda_last_status() == abi.OK


@pytest.mark.parametrize("device_ptrs", [False, True], ids=["host", "device"])
def test_ops_match_restatement(lib, cuda, device_ptrs):
    o = oracle.restatement()
    keep = []

    def arg(a):
        if not device_ptrs:
            return P(a)
        t = torch.from_numpy(a).to(cuda)
        keep.append((t, a))
        return t.data_ptr()

    def back():
        for t, a in keep:
            a[...] = t.cpu().numpy().reshape(a.shape)
        keep.clear()

    M, K, N = 300, 200, 136
    X, W, b, dY = rnd(M, K), rnd(N, K, seed=1), rnd(N, seed=2), rnd(M, N, seed=3)
    y_d, y_o = np.zeros((M, N), f32), np.zeros((M, N), f32)
    lib.linear_fwd(arg(X), arg(W), arg(b), arg(y_d), M, K, N); back()
    o.orc_linear_fwd(P(X), P(W), P(b), P(y_o), M, K, N)
    assert nwerr(y_d, y_o) < 1e-5
    dx_d, dx_o = np.full((M, K), 0.5, f32), np.full((M, K), 0.5, f32)
    lib.linear_bwd_dx(arg(dY), arg(W), arg(dx_d), M, K, N); back()
    o.orc_linear_bwd_dx(P(dY), P(W), P(dx_o), M, K, N)
    assert nwerr(dx_d, dx_o) < 1e-5
    dw_d, dw_o = np.full((N, K), 0.5, f32), np.full((N, K), 0.5, f32)
    db_d, db_o = np.full(N, 0.25, f32), np.full(N, 0.25, f32)
    lib.linear_bwd_dw(arg(dY), arg(X), arg(dw_d), arg(db_d), M, K, N); back()
    o.orc_linear_bwd_dw(P(dY), P(X), P(dw_o), P(db_o), M, K, N)
    assert nwerr(dw_d, dw_o) < 1e-5 and nwerr(db_d, db_o) < 1e-5
    Bh, T, hs = 3, 70, 64
    Q, Kk, V = rnd(Bh, T, hs, seed=4), rnd(Bh, T, hs, seed=5), rnd(Bh, T, hs, seed=6)
    s_d, s_o = np.zeros((Bh, T, T), f32), np.zeros((Bh, T, T), f32)
    lib.attn_scores(arg(Q), arg(Kk), arg(s_d), Bh, T, hs); back()
    o.orc_attn_scores(P(Q), P(Kk), P(s_o), Bh, T, hs)
    assert nwerr(s_d, s_o) < 1e-5
    o_d, o_o = np.zeros((Bh, T, hs), f32), np.zeros((Bh, T, hs), f32)
    lib.attn_values(arg(s_o), arg(V), arg(o_d), Bh, T, hs); back()
    o.orc_attn_values(P(s_o), P(V), P(o_o), Bh, T, hs)
    assert nwerr(o_d, o_o) < 1e-5
    Tn, Cn = 97, 160
    x, w, bb, dout = rnd(Tn, Cn, seed=7), rnd(Cn, seed=8), rnd(Cn, seed=9), rnd(Tn, Cn, seed=10)
    res = {}
    for name in ("d", "o"):
        out, mn, rs = np.zeros((Tn, Cn), f32), np.zeros(Tn, f32), np.zeros(Tn, f32)
        dx, dw, db = np.ones((Tn, Cn), f32), np.ones(Cn, f32), np.ones(Cn, f32)
        ge, gb = np.zeros(Tn * Cn, f32), np.ones(Tn * Cn, f32)
        sm = x.copy()
        cm = rnd(Tn, Tn, seed=11)
        lgt = rnd(Tn, 333, seed=12)
        tg = (np.arange(Tn) * 7 % 333).astype(np.int32)
        prb, ls = np.zeros((Tn, 333), f32), np.zeros(1, f32)
        dl = np.full((Tn, 333), 0.1, f32)
        ra = x.copy()
        if name == "d":
            lib.layernorm_fwd(arg(x), arg(w), arg(bb), arg(out), arg(mn), arg(rs), Tn, Cn); back()
            lib.layernorm_bwd(arg(dout), arg(x), arg(w), arg(mn), arg(rs), arg(dx), arg(dw), arg(db), Tn, Cn); back()
            lib.gelu_fwd(arg(x), arg(ge), Tn * Cn); back()
            lib.gelu_bwd(arg(dout), arg(x), arg(gb), Tn * Cn); back()
            lib.softmax_inplace(arg(sm), Tn, Cn); back()
            lib.causal_mask(arg(cm), Tn); back()
            lib.cross_entropy_fwd(arg(lgt), arg(tg), arg(prb), arg(ls), 1, Tn, 333); back()
            lib.cross_entropy_bwd(arg(dl), arg(prb), arg(tg), 0.5, 1, Tn, 333); back()
            lib.residual_add(arg(ra), arg(dout), Tn * Cn); back()
        else:
            o.orc_layernorm_fwd(P(x), P(w), P(bb), P(out), P(mn), P(rs), Tn, Cn)
            o.orc_layernorm_bwd(P(dout), P(x), P(w), P(mn), P(rs), P(dx), P(dw), P(db), Tn, Cn)
            o.orc_gelu_fwd(P(x), P(ge), Tn * Cn)
            o.orc_gelu_bwd(P(dout), P(x), P(gb), Tn * Cn)
            o.orc_softmax_inplace(P(sm), Tn, Cn)
            o.orc_causal_mask(P(cm), Tn)
            o.orc_cross_entropy_fwd(P(lgt), P(tg), P(prb), P(ls), 1, Tn, 333)
            o.orc_cross_entropy_bwd(P(dl), P(prb), P(tg), 0.5, 1, Tn, 333)
            o.orc_residual_add(P(ra), P(dout), Tn * Cn)
        res[name] = [out, mn, rs, dx, dw, db, ge, gb, sm, cm, prb, ls, dl, ra]
    for k, (a, c) in enumerate(zip(res["d"], res["o"])):
        assert nwerr(a, c) < 1e-5, k
    g = rnd(100003, seed=13)
    n_d = lib.global_grad_norm(arg(g), g.size); keep.clear()
    assert abs(n_d - o.orc_global_grad_norm(P(g), g.size)) / n_d < 1e-6
    gs_d, gs_o = g.copy(), g.copy()
    lib.scale_grads(arg(gs_d), g.size, 0.3); back()
    o.orc_scale_grads(P(gs_o), g.size, 0.3)
    assert np.array_equal(gs_d, gs_o)
    assert lib.cngpt_cuda_last_status() == abi.OK


def test_dropout_uses_host_rand_stream(lib, cuda):
    """dropout_fwd draws its mask from rand() exactly like src/ops.c:610-616"""
    ref = oracle.reference()
    n, p = 5000, 0.3
    x_r, x_d = rnd(n), rnd(n)
    m_r, m_d = np.zeros(n, np.uint8), np.zeros(n, np.uint8)
    oracle.libc_rand_stream(99)
    ref.dropout_fwd(P(x_r), P(m_r), n, p)
    oracle.libc_rand_stream(99)
    lib.dropout_fwd(P(x_d), P(m_d), n, p)
    assert np.array_equal(m_r, m_d)
    assert np.allclose(x_r, x_d, rtol=1e-6)
    ref.dropout_bwd(P(x_r), P(m_r), n, p)
    lib.dropout_bwd(P(x_d), P(m_d), n, p)
    assert np.allclose(x_r, x_d, rtol=1e-6)
