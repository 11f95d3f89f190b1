"""Test-side wrappers that drive the same GPT API on two libraries:
libcngpt_cuda (device arenas) and the reference's CPU build (host arenas).
Weights come from the C library's rand() stream seeded the way the reference
driver seeds it, so both models start from identical bytes."""
from __future__ import annotations

import ctypes as C

import numpy as np

from cngpt_b200 import abi
from oracle import oracle


def _np(ptr, n, dtype=np.float32):
    return np.ctypeslib.as_array(C.cast(ptr, C.POINTER(np.ctypeslib.as_ctypes_type(dtype))), shape=(n,))


class _Base:
    def __init__(self, lib, L, H, Cemb, V, block, seed, dropout=0.0, init=True):
        self.lib = lib
        self.cfg = abi.GPTConfig(L, H, Cemb, V, block, dropout)
        self.m = abi.GPT()
        assert lib.gpt_init(C.byref(self.m), self.cfg) == 0
        if init:  # otherwise the caller sets the parameters
            oracle.libc_rand_stream(seed)
            lib.gpt_init_weights(C.byref(self.m))
        self.n = self.m.n_params

    def forward(self, tok, tgt, B, T):
        return self.lib.gpt_forward(C.byref(self.m), oracle.ptr(tok), oracle.ptr(tgt), B, T)

    def backward(self, tok, tgt, B, T):
        self.lib.gpt_backward(C.byref(self.m), oracle.ptr(tok), oracle.ptr(tgt), B, T)

    def zero_grad(self):
        self.lib.gpt_zero_grad(C.byref(self.m))

    def adamw(self, lr, b1, b2, eps, wd, clip):
        self.lib.gpt_adamw(C.byref(self.m), lr, b1, b2, eps, wd, clip)

    def free(self):
        self.lib.gpt_free(C.byref(self.m))


class RefModel(_Base):
    """The reference's own CPU library (host pointers)."""

    def __init__(self, *a, **k):
        super().__init__(oracle.reference(), *a, **k)

    def params(self):
        return _np(self.m.param_buf, self.n).copy()

    def grads(self):
        return _np(self.m.grad_buf, self.n).copy()

    def logits(self, B, T):
        return _np(self.m.acts.logits, B * T * self.cfg.vocab_size).reshape(B, T, -1).copy()

    def set_params(self, p):
        _np(self.m.param_buf, self.n)[:] = p


class CudaModel(_Base):
    """libcngpt_cuda (device pointers; read back through the C ABI)."""

    def __init__(self, lib, *a, **k):
        super().__init__(lib, *a, **k)

    def _d2h(self, ptr, n, dtype=np.float32):
        out = np.empty(n, dtype=dtype)
        abi.check(self.lib, self.lib.cngpt_cuda_copy(out.ctypes.data, C.cast(ptr, C.c_void_p),
                                                     out.nbytes), "copy")
        return out

    def params(self):
        return self._d2h(self.m.param_buf, self.n)

    def grads(self):
        return self._d2h(self.m.grad_buf, self.n)

    def logits(self, B, T):
        return self._d2h(self.m.acts.logits, B * T * self.cfg.vocab_size).reshape(B, T, -1)

    def set_params(self, p):
        p = np.ascontiguousarray(p, dtype=np.float32)
        abi.check(self.lib, self.lib.cngpt_cuda_params_from_host(C.byref(self.m), p.ctypes.data), "h2d")


def nwerr(got, ref):
    """normwise relative error max|got-ref| / max|ref|"""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(got - ref)) / max(float(np.max(np.abs(ref))), 1e-30))


def param_slices(cfg):
    """(name, offset, size) of every tensor in the flat layout (src/model.c:54-83)."""
    Cm, V, T, L = cfg.n_embd, cfg.vocab_size, cfg.block_size, cfg.n_layer
    out, off = [], 0

    def add(name, n):
        nonlocal off
        out.append((name, off, n))
        off += n

    add("wte", V * Cm)
    add("wpe", T * Cm)
    for l in range(L):
        for nm, n in [("ln1_w", Cm), ("ln1_b", Cm), ("c_attn_w", 3 * Cm * Cm), ("c_attn_b", 3 * Cm),
                      ("c_proj_w", Cm * Cm), ("c_proj_b", Cm), ("ln2_w", Cm), ("ln2_b", Cm),
                      ("mlp_fc_w", 4 * Cm * Cm), ("mlp_fc_b", 4 * Cm), ("mlp_proj_w", 4 * Cm * Cm),
                      ("mlp_proj_b", Cm)]:
            add(f"L{l}.{nm}", n)
    add("ln_f_w", Cm)
    add("ln_f_b", Cm)
    return out
