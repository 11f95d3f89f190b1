"""GEMM kernel parity: cngpt_cuda_gemm (tcgen05 TF32 / 3xTF32, CUDA-core fp32)
against a float64 product of the same fp32 inputs, through the C ABI.

Tolerances (normwise: max|err| / max|ref|, per output):
  3xTF32  5e-6   (fp32-level: fp32 accumulation over K=3072 alone reaches ~1e-6)
  TF32    2e-3   (the BASELINE "plain TF32" bound)
  FP32    5e-6
The shapes cover every linear call site of the reference (src/ops.c:109-149
via src/model.c) at reduced M, the ragged vocabulary width, K not a multiple
of the 32-element k-block, and all four operand majorness combinations.
"""
import numpy as np
import pytest
import torch

from cngpt_b200 import abi

pytestmark = pytest.mark.gpu

TOL = {abi.PREC_3XTF32: 5e-6, abi.PREC_TF32: 2e-3, abi.PREC_FP32: 5e-6}


def nwerr(got, ref):
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def run_gemm(lib, dev, M, N, K, a_mn, b_mn, mode=abi.EPI_STORE, alpha=1.0, bias=False, seed=0,
             ld_pad=0):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn((K, M + ld_pad) if a_mn else (M, K + ld_pad), generator=g)
    B = torch.randn((K, N + ld_pad) if b_mn else (N, K + ld_pad), generator=g)
    A64 = (A[:, :M].T if a_mn else A[:, :K]).double()  # [M, K]
    B64 = (B[:, :N].T if b_mn else B[:, :K]).double()  # [N, K]
    ref = alpha * (A64 @ B64.T)
    b = torch.randn(N, generator=g) if bias else torch.zeros(N)
    dA, dB, db = A.to(dev), B.to(dev), b.to(dev)  # keep device copies alive across the call
    D = torch.zeros(M, N, device=dev)
    extra = {}
    if bias:
        ref = ref + b.double()
    if mode == abi.EPI_ACCUM:
        D0 = torch.randn(M, N, generator=g)
        D.copy_(D0)
        ref = ref + D0.double()
    D2 = torch.zeros(M, N, device=dev)
    R = torch.randn(M, N, generator=g)
    G = torch.randn(M, N, generator=g)
    dR, dG = R.to(dev), G.to(dev)
    st = lib.cngpt_cuda_gemm(dA.data_ptr(), A.shape[1], int(a_mn), dB.data_ptr(), B.shape[1], int(b_mn),
                             M, N, K, mode, alpha, D.data_ptr(), N,
                             db.data_ptr() if bias else None,
                             D2.data_ptr(), N, dR.data_ptr(), N, dG.data_ptr(), N)
    abi.check(lib, st, "gemm")
    abi.check(lib, lib.cngpt_cuda_check(), "gemm sync")
    out = {"D": D.cpu().double().numpy(), "D2": D2.cpu().double().numpy(), "ref": ref.numpy(),
           "R": R.double().numpy(), "G": G.double().numpy()}
    out.update(extra)
    return out


@pytest.fixture(params=[abi.PREC_3XTF32, abi.PREC_TF32, abi.PREC_FP32], ids=["3xtf32", "tf32", "fp32"])
def prec(request, lib):
    lib.cngpt_cuda_set_precision(request.param)
    yield request.param
    lib.cngpt_cuda_set_precision(abi.PREC_3XTF32)


# (M, N, K) - GPT-2 small call sites with M reduced, LM-head ragged N, odd K
SHAPES = [(256, 2304, 768), (256, 768, 3072), (384, 50257, 64), (300, 200, 100), (128, 128, 32),
          (1000, 520, 72), (64, 3072, 768)]
# few output tiles over a long K: split into K ranges, partials summed in order
SPLITK = [(256, 384, 4096), (768, 768, 8192), (130, 200, 2080)]
# decode-shaped rows (M <= 8 takes the GEMV kernel when A and B are K-major)
SKINNY = [(1, 2304, 768), (5, 768, 3072), (8, 50257, 768), (3, 3072, 768)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)],
                         ids=["NT", "NN", "TN", "TT"])
def test_gemm_store(lib, cuda, prec, M, N, K, a_mn, b_mn):
    if M * N > 384 * 50257 // 2 and (a_mn or b_mn) and prec == abi.PREC_FP32:
        pytest.skip("large fp32 CUDA-core case covered by NT")
    r = run_gemm(lib, cuda, M, N, K, a_mn, b_mn)
    e = nwerr(r["D"], r["ref"])
    print(f"gemm prec={prec} {M}x{N}x{K} a_mn={a_mn} b_mn={b_mn}: normwise {e:.3e}")
    assert e < TOL[prec], f"normwise error {e:.3e}"


@pytest.mark.parametrize("mode", [abi.EPI_STORE, abi.EPI_ACCUM, abi.EPI_GELU, abi.EPI_RESID,
                                  abi.EPI_GELU_BWD])
def test_gemm_epilogues(lib, cuda, prec, mode):
    M, N, K = 512, 768, 256
    r = run_gemm(lib, cuda, M, N, K, False, False, mode=mode, bias=mode != abi.EPI_GELU_BWD, alpha=1.0)
    ref = r["ref"]
    if mode == abi.EPI_GELU:
        assert nwerr(r["D"], ref) < TOL[prec]
        g = 0.5 * ref * (1 + np.tanh(0.7978845608028654 * (ref + 0.044715 * ref ** 3)))
        assert nwerr(r["D2"], g) < max(TOL[prec], 1e-5)
    elif mode == abi.EPI_RESID:
        assert nwerr(r["D"], ref) < TOL[prec]
        assert nwerr(r["D2"], r["R"] + ref) < TOL[prec]
    elif mode == abi.EPI_GELU_BWD:
        x = r["G"]
        th = np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3))
        gp = 0.5 * (1 + th) + 0.5 * x * (1 - th * th) * 0.7978845608028654 * (1 + 3 * 0.044715 * x * x)
        assert nwerr(r["D"], ref * gp) < max(TOL[prec], 1e-5)
    else:
        assert nwerr(r["D"], ref) < TOL[prec]


@pytest.mark.parametrize("M,N,K", SKINNY)
@pytest.mark.parametrize("mode", [abi.EPI_STORE, abi.EPI_ACCUM, abi.EPI_GELU, abi.EPI_RESID,
                                  abi.EPI_GELU_BWD])
def test_gemm_skinny_rows(lib, cuda, prec, M, N, K, mode):
    r = run_gemm(lib, cuda, M, N, K, False, False, mode=mode, bias=mode != abi.EPI_GELU_BWD, seed=M)
    ref = r["ref"]
    if mode == abi.EPI_GELU:
        g = 0.5 * ref * (1 + np.tanh(0.7978845608028654 * (ref + 0.044715 * ref ** 3)))
        assert nwerr(r["D"], ref) < TOL[prec] and nwerr(r["D2"], g) < max(TOL[prec], 1e-5)
    elif mode == abi.EPI_RESID:
        assert nwerr(r["D"], ref) < TOL[prec] and nwerr(r["D2"], r["R"] + ref) < TOL[prec]
    elif mode == abi.EPI_GELU_BWD:
        x = r["G"]
        th = np.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3))
        gp = 0.5 * (1 + th) + 0.5 * x * (1 - th * th) * 0.7978845608028654 * (1 + 3 * 0.044715 * x * x)
        assert nwerr(r["D"], ref * gp) < max(TOL[prec], 1e-5)
    else:
        assert nwerr(r["D"], ref) < TOL[prec]


@pytest.mark.parametrize("M,N,K", SPLITK)
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (True, True)], ids=["NT", "TN"])
@pytest.mark.parametrize("mode", [abi.EPI_STORE, abi.EPI_ACCUM, abi.EPI_RESID])
def test_gemm_split_k(lib, cuda, prec, M, N, K, a_mn, b_mn, mode):
    r = run_gemm(lib, cuda, M, N, K, a_mn, b_mn, mode=mode, bias=True, alpha=0.5, seed=K)
    ref = r["ref"]
    assert nwerr(r["D"], ref) < TOL[prec]
    if mode == abi.EPI_RESID:
        assert nwerr(r["D2"], r["R"] + ref) < TOL[prec]


def test_gemm_split_k_deterministic(lib, cuda, prec):
    a = run_gemm(lib, cuda, 768, 768, 8192, True, True, seed=5)["D"]
    b = run_gemm(lib, cuda, 768, 768, 8192, True, True, seed=5)["D"]
    assert np.array_equal(a, b)


def test_gemm_alpha_and_pitch(lib, cuda, prec):
    r = run_gemm(lib, cuda, 200, 136, 96, False, True, alpha=0.125, ld_pad=8)
    assert nwerr(r["D"], r["ref"]) < TOL[prec]


def test_gemm_deterministic(lib, cuda, prec):
    a = run_gemm(lib, cuda, 512, 1024, 768, True, True, seed=3)["D"]
    b = run_gemm(lib, cuda, 512, 1024, 768, True, True, seed=3)["D"]
    assert np.array_equal(a, b)


def test_gemm_rejects_bad_epilogue(lib, cuda):
    st = lib.cngpt_cuda_gemm(None, 4, 0, None, 4, 0, 4, 4, 4, 99, 1.0, None, 4, None, None, 4, None,
                             4, None, 4)
    assert st == abi.ERR_ARG
    lib.cngpt_cuda_clear_status()
