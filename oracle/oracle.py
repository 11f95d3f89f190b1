"""Python access to the parity checkers (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
import this module, and only as the checker / the timed CPU reference.

- `restatement()`: oracle/_build/libcngpt_oracle.so, the C restatement of the
  reference's algorithm (oracle/cngpt_oracle.c), orc_* entry points.
- `reference()`: oracle/_ref/libcngpt_ref.so, the reference's own ops.c /
  model.c / fast.c compiled by oracle/Makefile against OpenBLAS; the same
  drop-in API as libcngpt_cuda (struct layouts from cngpt_b200.abi).
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
RESTATEMENT_SO = HERE / "_build" / "libcngpt_oracle.so"
REFERENCE_SO = HERE / "_ref" / "libcngpt_ref.so"

VP, I, F, L = C.c_void_p, C.c_int, C.c_float, C.c_long


class OrcConfig(C.Structure):
    _fields_ = [("n_layer", I), ("n_head", I), ("n_embd", I), ("vocab_size", I), ("block_size", I)]


_ORC = {
    "orc_linear_fwd": (None, [VP, VP, VP, VP, I, I, I]),
    "orc_linear_bwd_dx": (None, [VP, VP, VP, I, I, I]),
    "orc_linear_bwd_dw": (None, [VP, VP, VP, VP, I, I, I]),
    "orc_attn_scores": (None, [VP, VP, VP, I, I, I]),
    "orc_attn_values": (None, [VP, VP, VP, I, I, I]),
    "orc_layernorm_fwd": (None, [VP, VP, VP, VP, VP, VP, I, I]),
    "orc_layernorm_bwd": (None, [VP, VP, VP, VP, VP, VP, VP, VP, I, I]),
    "orc_gelu_fwd": (None, [VP, VP, I]),
    "orc_gelu_bwd": (None, [VP, VP, VP, I]),
    "orc_softmax_inplace": (None, [VP, I, I]),
    "orc_causal_mask": (None, [VP, I]),
    "orc_cross_entropy_fwd": (None, [VP, VP, VP, VP, I, I, I]),
    "orc_cross_entropy_bwd": (None, [VP, VP, VP, F, I, I, I]),
    "orc_residual_add": (None, [VP, VP, I]),
    "orc_global_grad_norm": (F, [VP, I]),
    "orc_scale_grads": (None, [VP, I, F]),
    "orc_num_params": (L, [C.POINTER(OrcConfig)]),
    "orc_init_weights": (None, [C.POINTER(OrcConfig), VP]),
    "orc_decay_mask": (None, [C.POINTER(OrcConfig), VP]),
    "orc_forward": (F, [C.POINTER(OrcConfig), VP, VP, VP, I, I, VP, VP]),
    "orc_forward_backward": (F, [C.POINTER(OrcConfig), VP, VP, VP, I, I, VP]),
    "orc_adamw": (None, [VP, VP, VP, VP, VP, L, C.POINTER(I), F, F, F, F, F, F]),
    "orc_forward_last": (None, [C.POINTER(OrcConfig), VP, VP, I, I, VP]),
}

_cache: dict[str, C.CDLL] = {}


def _make(target: str) -> None:
    subprocess.run(["make", "-s", "-C", str(HERE), target], check=True)


def restatement() -> C.CDLL:
    if "orc" not in _cache:
        if not RESTATEMENT_SO.exists():
            _make("oracle")
        lib = C.CDLL(str(RESTATEMENT_SO))
        for n, (r, a) in _ORC.items():
            f = getattr(lib, n)
            f.restype, f.argtypes = r, a
        _cache["orc"] = lib
    return _cache["orc"]


def reference_available() -> bool:
    return REFERENCE_SO.exists()


def reference() -> C.CDLL:
    """The reference's own CPU build (raises if it was never built here)."""
    if "ref" not in _cache:
        if not REFERENCE_SO.exists():
            raise RuntimeError(f"{REFERENCE_SO} missing: run `make -C oracle ref` where the "
                               "reference tree is mounted")
        from cngpt_b200.abi import DROPIN_SIGNATURES, bind
        lib = C.CDLL(str(REFERENCE_SO))
        bind(lib, DROPIN_SIGNATURES)
        _cache["ref"] = lib
    return _cache["ref"]


def ptr(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data


def cfg(n_layer, n_head, n_embd, vocab_size, block_size) -> OrcConfig:
    return OrcConfig(n_layer, n_head, n_embd, vocab_size, block_size)


# ---------------------------------------------------------------- helpers
def libc_rand_stream(seed: int | None):
    """Seed the process's C library rand() exactly as the reference driver does
    (srand(seed); seed None = never seeded, which glibc treats as srand(1))."""
    libc = C.CDLL(None)
    libc.srand(1 if seed is None else seed)


def init_weights(c: OrcConfig, seed: int | None) -> np.ndarray:
    lib = restatement()
    libc_rand_stream(seed)
    p = np.zeros(lib.orc_num_params(C.byref(c)), dtype=np.float32)
    lib.orc_init_weights(C.byref(c), ptr(p))
    return p


def lcg_tokens(n: int, vocab: int, seed: int = 12345) -> np.ndarray:
    """The reference bench's token generator (src/cngpt.c:338-342)."""
    out = np.empty(n, dtype=np.int32)
    s = seed & 0xFFFFFFFF
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = (s >> 8) % vocab
    return out


def forward(c: OrcConfig, params: np.ndarray, tok: np.ndarray, tgt: np.ndarray | None, B: int, T: int):
    lib = restatement()
    logits = np.zeros(B * T * c.vocab_size, dtype=np.float32)
    loss = lib.orc_forward(C.byref(c), ptr(params), ptr(tok), ptr(tgt), B, T, ptr(logits), None)
    return loss, logits.reshape(B, T, c.vocab_size)


def forward_backward(c: OrcConfig, params, tok, tgt, B, T):
    lib = restatement()
    grads = np.zeros_like(params)
    loss = lib.orc_forward_backward(C.byref(c), ptr(params), ptr(tok), ptr(tgt), B, T, ptr(grads))
    return loss, grads


def adamw(c: OrcConfig, params, grads, m, v, step, lr, b1, b2, eps, wd, clip):
    lib = restatement()
    decay = np.zeros(params.size, dtype=np.uint8)
    lib.orc_decay_mask(C.byref(c), ptr(decay))
    st = C.c_int(step)
    lib.orc_adamw(ptr(params), ptr(grads), ptr(m), ptr(v), ptr(decay), params.size, C.byref(st),
                  lr, b1, b2, eps, wd, clip)
    return st.value


# ---------------------------------------------------------------- data loader
class DataLoader(C.Structure):
    """src/dataloader.h:20-36, field for field"""
    _fields_ = [("batch_size", I), ("seq_len", I), ("filename", C.c_char_p), ("fd", I),
                ("data", C.POINTER(C.c_uint16)), ("n_tokens", C.c_size_t), ("pos", C.c_size_t),
                ("inputs", C.POINTER(I)), ("targets", C.POINTER(I))]


def reference_batches(path: str, B: int, T: int, n: int) -> list[tuple[np.ndarray, np.ndarray]]:
    """n batches from the reference's own DataLoader (src/dataloader.c:19-82)
    over a uint16 token file: (inputs, targets), each int32[B*T]."""
    lib = reference()
    lib.dataloader_init.restype = I
    lib.dataloader_init.argtypes = [C.POINTER(DataLoader), C.c_char_p, I, I]
    lib.dataloader_next_batch.argtypes = [C.POINTER(DataLoader)]
    lib.dataloader_free.argtypes = [C.POINTER(DataLoader)]
    dl = DataLoader()
    assert lib.dataloader_init(C.byref(dl), path.encode(), B, T) == 0
    out = []
    for _ in range(n):
        lib.dataloader_next_batch(C.byref(dl))
        out.append((np.ctypeslib.as_array(dl.inputs, shape=(B * T,)).copy(),
                    np.ctypeslib.as_array(dl.targets, shape=(B * T,)).copy()))
    lib.dataloader_free(C.byref(dl))
    return out


def restated_batches(data: np.ndarray, B: int, T: int, n: int) -> list[tuple[np.ndarray, np.ndarray]]:
    """The same batch sequence restated (src/dataloader.c:62-82): element
    (b, t) of a batch at position pos is data[(pos + b*T + t) % N], its target
    the next token; pos advances by B*T and rewinds when pos + B*T + 1 > N."""
    N, BT, pos, out = data.size, B * T, 0, []
    for _ in range(n):
        idx = (pos + np.arange(BT)) % N
        out.append((data[idx].astype(np.int32), data[(idx + 1) % N].astype(np.int32)))
        pos += BT
        if pos + BT + 1 > N:
            pos = 0
    return out
