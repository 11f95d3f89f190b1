"""The reference's own unit tests (tests/check_ops.c, check_grad.c,
check_fast.c), compiled unmodified by oracle/Makefile and linked against
libcngpt_cuda instead of the reference's ops.c / model.c / fast.c.

check_grad and check_fast dereference m->param_buf, m->grad_buf and
m->acts.logits on the host, so they run with CNGPT_CUDA_MANAGED=1 (arenas in
managed memory); check_ops passes stack arrays, which the library stages.
"""
import os
import subprocess
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref"


@pytest.mark.parametrize("name,managed", [("ops", False), ("grad", True), ("fast", True)])
@pytest.mark.parametrize("prec", ["3xtf32", "fp32"])
def test_reference_unit_test_against_dropin(cuda, name, managed, prec):
    exe = REF / f"check_{name}_cuda"
    assert exe.exists(), f"{exe} missing: build() links it where the reference tree is mounted"
    env = dict(os.environ, CNGPT_CUDA_PRECISION=prec)
    if managed:
        env["CNGPT_CUDA_MANAGED"] = "1"
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=900, env=env)
    print(r.stdout[-400:])
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert " 0 failed" in r.stdout
