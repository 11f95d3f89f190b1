"""ctypes view of libcngpt_cuda's C ABI (include/cngpt/*.h, include/cngpt_cuda.h).

The structs mirror the reference's src/model.h:22-137 and src/fast.h:35-45
field for field (the library keeps them byte-identical), so the same
definitions also describe the reference's own CPU library.

`load()` opens the in-tree libcngpt_cuda.so and raises if it is missing: there
is no CPU fallback behind this module.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libcngpt_cuda.so"

FP = C.POINTER(C.c_float)
FPP = C.POINTER(FP)
IP = C.POINTER(C.c_int)
UCP = C.POINTER(C.c_ubyte)
UCPP = C.POINTER(UCP)


class GPTConfig(C.Structure):
    _fields_ = [("n_layer", C.c_int), ("n_head", C.c_int), ("n_embd", C.c_int),
                ("vocab_size", C.c_int), ("block_size", C.c_int), ("dropout", C.c_float)]


_W = ["ln1_w", "ln1_b", "c_attn_w", "c_attn_b", "c_proj_w", "c_proj_b", "ln2_w", "ln2_b",
      "mlp_fc_w", "mlp_fc_b", "mlp_proj_w", "mlp_proj_b"]


class GPTWeights(C.Structure):
    _fields_ = [("wte", FP), ("wpe", FP)] + [(n, FPP) for n in _W] + [("ln_f_w", FP), ("ln_f_b", FP)]


_A = ["ln1_out", "ln1_mean", "ln1_rstd", "qkv", "attn_scores", "attn_probs", "attn_out", "attn_proj",
      "res1", "ln2_out", "ln2_mean", "ln2_rstd", "mlp_fc_out", "mlp_gelu", "mlp_proj_out", "res2"]


class GPTActivations(C.Structure):
    _fields_ = ([("emb", FP)] + [(n, FPP) for n in _A] +
                [("ln_f_out", FP), ("ln_f_mean", FP), ("ln_f_rstd", FP), ("logits", FP), ("probs", FP),
                 ("emb_mask", UCP), ("res1_mask", UCPP), ("res2_mask", UCPP)])


class GPT(C.Structure):
    _fields_ = [("cfg", GPTConfig), ("params", GPTWeights), ("grads", GPTWeights),
                ("acts", GPTActivations), ("param_buf", FP), ("grad_buf", FP), ("act_buf", FP),
                ("mask_buf", UCP), ("m_buf", FP), ("v_buf", FP), ("decay_buf", UCP),
                ("n_params", C.c_int), ("step", C.c_int)]


class FastCtx(C.Structure):
    _fields_ = [("B", C.c_int), ("T", C.c_int), ("x", FP), ("ln", FP), ("qkv", FP), ("scores", FP),
                ("aout", FP), ("hid", FP), ("mean", FP), ("rstd", FP), ("logits", FP)]


# status / modes (include/cngpt_cuda.h)
OK, ERR_CUDA, ERR_ARG, ERR_ALLOC, ERR_DEVICE_WAIT, ERR_NCCL, ERR_STATE = range(7)
PREC_TF32, PREC_3XTF32, PREC_FP32 = 0, 1, 2
EPI_STORE, EPI_ACCUM, EPI_GELU, EPI_RESID, EPI_GELU_BWD = range(5)

VP = C.c_void_p
L = C.c_long
I = C.c_int
F = C.c_float

# drop-in API shared by this library and the reference's CPU build
# (src/ops.h:19-107, src/model.h:144-194, src/fast.h:48-60)
DROPIN_SIGNATURES = {
    "linear_fwd": (None, [VP, VP, VP, VP, I, I, I]),
    "linear_bwd_dx": (None, [VP, VP, VP, I, I, I]),
    "linear_bwd_dw": (None, [VP, VP, VP, VP, I, I, I]),
    "attn_scores": (None, [VP, VP, VP, I, I, I]),
    "attn_values": (None, [VP, VP, VP, I, I, I]),
    "layernorm_fwd": (None, [VP, VP, VP, VP, VP, VP, I, I]),
    "layernorm_bwd": (None, [VP, VP, VP, VP, VP, VP, VP, VP, I, I]),
    "gelu_fwd": (None, [VP, VP, I]),
    "gelu_bwd": (None, [VP, VP, VP, I]),
    "softmax_inplace": (None, [VP, I, I]),
    "causal_mask": (None, [VP, I]),
    "cross_entropy_fwd": (None, [VP, VP, VP, VP, I, I, I]),
    "cross_entropy_bwd": (None, [VP, VP, VP, F, I, I, I]),
    "residual_add": (None, [VP, VP, I]),
    "dropout_fwd": (None, [VP, VP, I, F]),
    "dropout_bwd": (None, [VP, VP, I, F]),
    "global_grad_norm": (F, [VP, I]),
    "scale_grads": (None, [VP, I, F]),
    "gpt_init": (I, [C.POINTER(GPT), GPTConfig]),
    "gpt_init_weights": (None, [C.POINTER(GPT)]),
    "gpt_load": (I, [C.POINTER(GPT), C.c_char_p]),
    "gpt_save": (I, [C.POINTER(GPT), C.c_char_p]),
    "gpt_free": (None, [C.POINTER(GPT)]),
    "gpt_resize_acts": (I, [C.POINTER(GPT), I, I]),
    "gpt_forward": (F, [C.POINTER(GPT), VP, VP, I, I]),
    "gpt_backward": (None, [C.POINTER(GPT), VP, VP, I, I]),
    "gpt_zero_grad": (None, [C.POINTER(GPT)]),
    "gpt_adamw": (None, [C.POINTER(GPT), F, F, F, F, F, F]),
    "gpt_sample": (None, [C.POINTER(GPT), VP, I, VP, I, F, I]),
    "gpt_num_params": (I, [C.POINTER(GPTConfig)]),
    "fast_init": (None, [C.POINTER(FastCtx)]),
    "fast_free": (None, [C.POINTER(FastCtx)]),
    "fast_set_threads": (None, [I]),
    "gpt_forward_fast": (FP, [C.POINTER(GPT), C.POINTER(FastCtx), VP, I, I]),
}

# extensions (include/cngpt_cuda.h)
EXT_SIGNATURES = {
    "cngpt_cuda_last_status": (I, []),
    "cngpt_cuda_last_message": (C.c_char_p, []),
    "cngpt_cuda_clear_status": (None, []),
    "cngpt_cuda_check": (I, []),
    "cngpt_cuda_set_precision": (I, [I]),
    "cngpt_cuda_get_precision": (I, []),
    "cngpt_cuda_set_stream": (I, [VP]),
    "cngpt_cuda_get_stream": (VP, []),
    "cngpt_cuda_set_managed": (I, [I]),
    "cngpt_cuda_launch_count": (C.c_ulonglong, []),
    "cngpt_cuda_set_wait_limit_ns": (I, [C.c_ulonglong]),
    "cngpt_cuda_set_decode_step_kernel": (I, [I]),
    "cngpt_cuda_gemm": (I, [VP, L, I, VP, L, I, I, I, I, I, F, VP, L, VP, VP, L, VP, L, VP, L]),
    "cngpt_cuda_attention_fwd": (I, [VP, VP, VP, I, I, I, I]),
    "cngpt_cuda_attention_bwd": (I, [VP, VP, VP, VP, VP, I, I, I, I]),
    "cngpt_cuda_train_step": (I, [C.POINTER(GPT), VP, VP, I, I, F, F, F, F, F, F, VP]),
    "cngpt_cuda_last_loss": (I, [C.POINTER(GPT), FP]),
    "cngpt_cuda_params_to_host": (I, [C.POINTER(GPT), VP]),
    "cngpt_cuda_params_from_host": (I, [C.POINTER(GPT), VP]),
    "cngpt_cuda_grads_to_host": (I, [C.POINTER(GPT), VP]),
    "cngpt_cuda_copy": (I, [VP, VP, C.c_size_t]),
    "cngpt_cuda_generate": (I, [C.POINTER(GPT), C.POINTER(FastCtx), VP, I, I, I, VP]),
    "cngpt_cuda_dp_unique_id": (I, [VP]),
    "cngpt_cuda_dp_init": (I, [C.POINTER(GPT), VP, I, I]),
    "cngpt_cuda_dp_allreduce_grads": (I, [C.POINTER(GPT)]),
    "cngpt_cuda_dp_free": (I, [C.POINTER(GPT)]),
    "cngpt_cuda_save_checkpoint": (I, [C.POINTER(GPT), C.c_char_p]),
    "cngpt_cuda_load_checkpoint": (I, [C.POINTER(GPT), C.c_char_p]),
    "cngpt_cuda_tp_plan": (I, [I, I, I, I, I, VP]),
    "cngpt_cuda_tp_init": (I, [C.POINTER(GPT), VP, I, I]),
    "cngpt_cuda_tp_forward_last": (I, [C.POINTER(GPT), VP, I, I, VP]),
    "cngpt_cuda_tp_generate": (I, [C.POINTER(GPT), VP, I, I, I, VP]),
    "cngpt_cuda_tp_free": (I, [C.POINTER(GPT)]),
    "cngpt_cuda_tp_set_decode_mode": (I, [C.POINTER(GPT), I]),
    "cngpt_cuda_selftest_tp_reduce": (I, [VP, VP, I, I, I, VP]),
    "cngpt_cuda_loader_create": (I, [C.POINTER(VP), VP, C.c_size_t, I, I]),
    "cngpt_cuda_loader_next": (I, [VP, C.POINTER(VP), C.POINTER(VP)]),
    "cngpt_cuda_loader_reset": (I, [VP]),
    "cngpt_cuda_loader_num_batches": (C.c_size_t, [VP]),
    "cngpt_cuda_loader_free": (None, [VP]),
}


def bind(lib: C.CDLL, table: dict) -> C.CDLL:
    for name, (res, args) in table.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


_LIB = None


def load(path: str | os.PathLike | None = None) -> C.CDLL:
    """Open libcngpt_cuda.so (in-tree build). Raises if it has not been built."""
    global _LIB
    if _LIB is not None and path is None:
        return _LIB
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is missing: build it with `python -m cngpt_b200.build` "
                           "(there is no CPU fallback)")
    lib = C.CDLL(str(p))  # RTLD_LOCAL: never interposes the reference build
    bind(lib, DROPIN_SIGNATURES)
    bind(lib, EXT_SIGNATURES)
    if path is None:
        _LIB = lib
    return lib


class CudaError(RuntimeError):
    pass


def check(lib: C.CDLL, status: int, what: str = "") -> None:
    if status != OK:
        msg = lib.cngpt_cuda_last_message().decode(errors="replace")
        raise CudaError(f"{what}: status {status}: {msg}")
