"""The C-ABI boundary, checked without a GPU.

- libcngpt_cuda.so loads and exports every function that include/*.h declares;
- the drop-in headers declare every function of the reference's ops.h,
  model.h and fast.h with the same signature;
- GPT, GPTConfig, GPTWeights, GPTActivations, FastCtx and GPTHeader are
  byte-identical to the reference's (offset of every field, compiled by gcc
  against both headers), so code compiled against either header links here;
- the ctypes mirror in cngpt_b200/abi.py matches the C layout.
"""
import ctypes as C
import os
import re
import subprocess
import tempfile
from pathlib import Path

import pytest

from cngpt_b200 import abi

ROOT = Path(__file__).resolve().parents[1]
INC = ROOT / "include"
# the reference tree: $CNGPT_REFERENCE, else `reference` beside this repository
REF_SRC = Path(os.environ.get("CNGPT_REFERENCE") or ROOT.parent / "reference") / "src"


def declared_functions(path: Path) -> set[str]:
    txt = re.sub(r"/\*.*?\*/", "", path.read_text(), flags=re.S)
    txt = re.sub(r"//[^\n]*", "", txt)
    names = set()
    for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", txt, re.M):
        name = m.group(1)
        if name not in {"if", "for", "while", "return", "sizeof"} and not name.startswith("__"):
            names.add(name)
    return names


def exported_symbols(path: Path) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(path)], capture_output=True, text=True,
                         check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


def test_library_loads_and_exports_every_declared_symbol():
    lib = abi.load()  # dlopen works without a GPU: no CUDA call happens at load
    assert lib is not None
    syms = exported_symbols(abi.LIB_PATH)
    declared = set()
    for h in sorted(INC.rglob("*.h")):
        declared |= declared_functions(h)
    assert declared, "no declarations parsed"
    missing = sorted(declared - syms)
    assert not missing, f"declared but not exported: {missing}"
    for name in list(abi.DROPIN_SIGNATURES) + list(abi.EXT_SIGNATURES):
        assert name in syms, name


@pytest.mark.skipif(not REF_SRC.exists(), reason="reference tree absent")
def test_dropin_headers_cover_reference_api():
    for h in ("ops.h", "model.h", "fast.h"):
        ref = declared_functions(REF_SRC / h)
        ours = declared_functions(INC / "cngpt" / h)
        assert ref <= ours, f"{h}: missing {sorted(ref - ours)}"


LAYOUT_C = r"""
#include <stdio.h>
#include <stddef.h>
#include "model.h"
#include "fast.h"
#define F(T, f) printf(#T "." #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("GPT %zu\nGPTConfig %zu\nGPTWeights %zu\nGPTActivations %zu\nFastCtx %zu\nGPTHeader %zu\n",
         sizeof(GPT), sizeof(GPTConfig), sizeof(GPTWeights), sizeof(GPTActivations),
         sizeof(FastCtx), sizeof(GPTHeader));
  F(GPT, cfg) F(GPT, params) F(GPT, grads) F(GPT, acts) F(GPT, param_buf) F(GPT, grad_buf)
  F(GPT, act_buf) F(GPT, mask_buf) F(GPT, m_buf) F(GPT, v_buf) F(GPT, decay_buf)
  F(GPT, n_params) F(GPT, step)
  F(GPTActivations, emb) F(GPTActivations, qkv) F(GPTActivations, attn_scores) F(GPTActivations, res2)
  F(GPTActivations, ln_f_out) F(GPTActivations, logits) F(GPTActivations, probs)
  F(GPTActivations, emb_mask) F(GPTActivations, res2_mask)
  F(GPTWeights, wte) F(GPTWeights, c_attn_w) F(GPTWeights, mlp_proj_b) F(GPTWeights, ln_f_b)
  F(FastCtx, x) F(FastCtx, scores) F(FastCtx, logits)
  return 0;
}
"""


def _layout(include_dir: Path) -> str:
    with tempfile.TemporaryDirectory() as d:
        src = Path(d) / "l.c"
        src.write_text(LAYOUT_C)
        exe = Path(d) / "l"
        subprocess.run(["/usr/bin/gcc" if Path("/usr/bin/gcc").exists() else "gcc", "-std=c11",
                        f"-I{include_dir}", str(src), "-o", str(exe)], check=True)
        return subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout


def test_struct_layout_matches_ctypes_mirror():
    lines = dict(ln.rsplit(" ", 1) for ln in _layout(INC / "cngpt").splitlines())
    assert int(lines["GPT"]) == C.sizeof(abi.GPT)
    assert int(lines["FastCtx"]) == C.sizeof(abi.FastCtx)
    assert int(lines["GPTActivations"]) == C.sizeof(abi.GPTActivations)
    assert int(lines["GPT.n_params"]) == abi.GPT.n_params.offset
    assert int(lines["GPT.param_buf"]) == abi.GPT.param_buf.offset


@pytest.mark.skipif(not REF_SRC.exists(), reason="reference tree absent")
def test_struct_layout_identical_to_reference():
    assert _layout(INC / "cngpt") == _layout(REF_SRC)


def test_num_params_formula():
    lib = abi.load()
    for cfg, n in [((12, 12, 768, 50257, 1024), 124439808), ((24, 16, 1024, 50257, 1024), 354823168),
                   ((48, 25, 1600, 50257, 1024), 1557611200), ((6, 6, 384, 65, 256), 10770816)]:
        c = abi.GPTConfig(*cfg, 0.0)
        assert lib.gpt_num_params(C.byref(c)) == n


@pytest.mark.parametrize("H,Cemb,V", [(25, 1600, 50257), (12, 768, 50257), (5, 320, 1001), (3, 96, 77)])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_tp_plan_partitions_heads_hidden_and_vocab(H, Cemb, V, world):
    """cngpt_cuda_tp_plan is host-only: the ranks' slices tile every split
    dimension exactly once, in rank order, 16-byte aligned where read in place."""
    lib = abi.load()
    plans = []
    for rank in range(world):
        p = (C.c_int * 7)()
        st = lib.cngpt_cuda_tp_plan(H, Cemb, V, world, rank, p)
        if world > H:
            assert st == abi.ERR_ARG
            lib.cngpt_cuda_clear_status()
            return
        assert st == abi.OK
        plans.append(list(p))
    h = f = v = 0
    for h0, nh, f0, nf, v0, nv, vpad in plans:
        assert (h0, f0, v0) == (h, f, v) and nh >= 1 and nf > 0 and nv > 0
        assert f0 % 4 == 0 and nf % 4 == 0 and vpad == -(-V // world)
        h, f, v = h + nh, f + nf, v + nv
    assert (h, f, v) == (H, 4 * Cemb, V)
    assert max(p[1] for p in plans) - min(p[1] for p in plans) <= 1


def test_tp_plan_rejects_bad_rank():
    lib = abi.load()
    p = (C.c_int * 7)()
    assert lib.cngpt_cuda_tp_plan(12, 768, 50257, 2, 2, p) == abi.ERR_ARG
    assert lib.cngpt_cuda_tp_plan(12, 770, 50257, 2, 0, p) == abi.ERR_ARG
    lib.cngpt_cuda_clear_status()


def test_load_checkpoint_rejects_missing_and_foreign_files():
    """The checkpoint loader checks the file before any device work: a missing
    path and a file without the model-file magic are ERR_ARG with a message."""
    lib = abi.load()
    m = abi.GPT()
    with tempfile.TemporaryDirectory() as d:
        missing = str(Path(d) / "none.bin").encode()
        assert lib.cngpt_cuda_load_checkpoint(C.byref(m), missing) == abi.ERR_ARG
        assert "cannot open" in lib.cngpt_cuda_last_message().decode()
        foreign = Path(d) / "foreign.bin"
        foreign.write_bytes(b"\x00" * 1024)
        assert lib.cngpt_cuda_load_checkpoint(C.byref(m), str(foreign).encode()) == abi.ERR_ARG
        assert "not a cngpt model file" in lib.cngpt_cuda_last_message().decode()
    assert not m.param_buf  # nothing was allocated
    lib.cngpt_cuda_clear_status()


def test_load_checkpoint_rejects_truncated_file_before_device_work():
    """A file whose header is valid but whose parameters stop short is read
    whole on the host and rejected before the model is created."""
    import struct
    lib = abi.load()
    m = abi.GPT()
    with tempfile.TemporaryDirectory() as d:
        short = Path(d) / "short.bin"
        # magic, version, n_layer, n_head, n_embd, vocab, block (src/model.h:22-30)
        short.write_bytes(struct.pack("<7i", 0x434E4750, 1, 1, 2, 8, 10, 4) + b"\x00" * 64)
        assert lib.cngpt_cuda_load_checkpoint(C.byref(m), str(short).encode()) == abi.ERR_ARG
        assert "truncated" in lib.cngpt_cuda_last_message().decode()
    assert not m.param_buf
    lib.cngpt_cuda_clear_status()


def test_argument_errors_are_reported_before_device_work():
    """Argument checks of the extension entry points run on the host: the
    status is returned and the message recorded, with no device involved."""
    lib = abi.load()
    assert lib.cngpt_cuda_set_precision(7) == abi.ERR_ARG
    assert "precision" in lib.cngpt_cuda_last_message().decode()
    # unknown epilogue mode, and a residual epilogue without its operands
    assert lib.cngpt_cuda_gemm(None, 4, 0, None, 4, 0, 4, 4, 4, 9, 1.0, None, 4, None, None, 0, None, 0, None,
                               0) == abi.ERR_ARG
    assert lib.cngpt_cuda_gemm(None, 4, 0, None, 4, 0, 4, 4, 4, abi.EPI_RESID, 1.0, None, 4, None, None, 0, None,
                               0, None, 0) == abi.ERR_ARG
    assert "missing epilogue operand" in lib.cngpt_cuda_last_message().decode()
    # C not divisible by the head count
    assert lib.cngpt_cuda_attention_fwd(None, None, None, 1, 8, 770, 12) == abi.ERR_ARG
    # a GPT the library never initialised
    m = abi.GPT()
    uid = (C.c_ubyte * 128)()
    assert lib.cngpt_cuda_dp_init(C.byref(m), uid, 2, 0) == abi.ERR_STATE
    lib.cngpt_cuda_clear_status()
