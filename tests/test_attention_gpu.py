"""Fused causal attention through the C ABI (cngpt_cuda_attention_fwd/bwd)
against a float64 PyTorch restatement of the reference's per-head loop
(src/model.c:514-563 forward, 742-822 backward): S = QK^T / sqrt(hs), causal
mask, row softmax, O = PV, lse = log-sum-exp of the scaled scores.

Tolerances (normwise max|err| / max|ref|): TF32 2e-3 (the tensor cores read
tf32 operands; forward and backward on tcgen05 for head size 64), 3xTF32
2e-5, FP32 1e-5 (backward: 5x).
Shapes: GPT-2 small heads (hs 64) at T = 1024 and ragged T, head size 32
(CUDA-core path), and an odd B*T whose rows are not 16-byte aligned."""
import numpy as np
import pytest
import torch

from cngpt_b200 import abi

pytestmark = pytest.mark.gpu

TOL = {abi.PREC_TF32: 2e-3, abi.PREC_3XTF32: 2e-5, abi.PREC_FP32: 1e-5}
SHAPES = [(2, 1024, 768, 12), (1, 1000, 768, 12), (3, 77, 128, 2), (2, 130, 256, 4), (1, 300, 96, 3)]


def nwerr(a, b):
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def reference(qkv, B, T, C, H):
    hs = C // H
    x = qkv.double().view(B, T, 3, H, hs)
    q, k, v = (x[:, :, i].permute(0, 2, 1, 3) for i in range(3))  # [B, H, T, hs]
    s = q @ k.transpose(-1, -2) / np.sqrt(hs)
    mask = torch.ones(T, T, dtype=torch.bool, device=qkv.device).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    o = torch.softmax(s, dim=-1) @ v
    return o.permute(0, 2, 1, 3).reshape(B, T, C), lse.reshape(B * H * T)


@pytest.fixture(params=[abi.PREC_TF32, abi.PREC_3XTF32, abi.PREC_FP32], ids=["tf32", "3xtf32", "fp32"])
def prec(request, lib):
    lib.cngpt_cuda_set_precision(request.param)
    yield request.param
    lib.cngpt_cuda_set_precision(abi.PREC_3XTF32)


@pytest.mark.parametrize("B,T,C,H", SHAPES)
def test_attention_forward(lib, cuda, prec, B, T, C, H):
    g = torch.Generator(device=cuda).manual_seed(B * T + C)
    qkv = torch.randn(B, T, 3 * C, device=cuda, generator=g)
    out = torch.empty(B, T, C, device=cuda)
    lse = torch.empty(B * H * T, device=cuda)
    abi.check(lib, lib.cngpt_cuda_attention_fwd(qkv.data_ptr(), out.data_ptr(), lse.data_ptr(), B, T, C, H), "fwd")
    abi.check(lib, lib.cngpt_cuda_check(), "sync")
    ro, rl = reference(qkv, B, T, C, H)
    eo, el = nwerr(out.double(), ro), float((lse.double() - rl).abs().max())
    print(f"\nattention fwd prec={prec} B={B} T={T} C={C} H={H}: out {eo:.2e}, lse abs {el:.2e}")
    assert eo < TOL[prec]
    assert el < 50 * TOL[prec]


def test_attention_forward_unaligned_rows(lib, cuda):
    """qkv starting 4 bytes past a 16-byte boundary (an odd B*T arena slot):
    the TMA and cp.async kernels decline and the CUDA-core kernel runs."""
    lib.cngpt_cuda_set_precision(abi.PREC_TF32)
    try:
        B, T, C, H = 1, 200, 768, 12
        g = torch.Generator(device=cuda).manual_seed(5)
        buf = torch.randn(B * T * 3 * C + 1, device=cuda, generator=g)
        qkv = buf[1:].view(B, T, 3 * C)
        out = torch.empty(B * T * C + 1, device=cuda)[1:].view(B, T, C)
        abi.check(lib, lib.cngpt_cuda_attention_fwd(qkv.data_ptr(), out.data_ptr(), None, B, T, C, H), "fwd")
        abi.check(lib, lib.cngpt_cuda_check(), "sync")
        ro, _ = reference(qkv, B, T, C, H)
        assert nwerr(out.double(), ro) < TOL[abi.PREC_TF32]
    finally:
        lib.cngpt_cuda_set_precision(abi.PREC_3XTF32)


@pytest.mark.parametrize("B,T,C,H", [(2, 512, 768, 12), (1, 1000, 768, 12), (3, 77, 128, 2), (1, 300, 96, 3)])
def test_attention_backward(lib, cuda, prec, B, T, C, H):
    g = torch.Generator(device=cuda).manual_seed(T)
    qkv = torch.randn(B, T, 3 * C, device=cuda, generator=g)
    dout = torch.randn(B, T, C, device=cuda, generator=g)
    out = torch.empty(B, T, C, device=cuda)
    lse = torch.empty(B * H * T, device=cuda)
    dqkv = torch.empty(B, T, 3 * C, device=cuda)
    abi.check(lib, lib.cngpt_cuda_attention_fwd(qkv.data_ptr(), out.data_ptr(), lse.data_ptr(), B, T, C, H), "fwd")
    abi.check(lib, lib.cngpt_cuda_attention_bwd(qkv.data_ptr(), out.data_ptr(), dout.data_ptr(), lse.data_ptr(),
                                                dqkv.data_ptr(), B, T, C, H), "bwd")
    abi.check(lib, lib.cngpt_cuda_check(), "sync")
    x = qkv.double().requires_grad_(True)
    ro, _ = reference(x, B, T, C, H)
    ro.backward(dout.double())
    e = nwerr(dqkv.double(), x.grad)
    print(f"\nattention bwd prec={prec} B={B} T={T}: dqkv {e:.2e}")
    assert e < 5 * TOL[prec]
