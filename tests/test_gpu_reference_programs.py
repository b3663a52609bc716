"""Drop-in check with the reference's own test programs.

`make -C oracle ref` compiles the reference's bench/kernel/test_w8a8.c
(the W8A8 API: mode flag, per-tensor / per-channel quantization and
dequantization, both GEMMs, fake quantization, the fp32 GEMM) and
bench/kernel/tmac_lut.c (the T-MAC tables, with the reference's arena.c as
its test infrastructure) unmodified against the reference's headers and
links them against libjimotono_b200.so instead of the reference library.
Run on the GPU, every check of those programs must pass through this
library's CUDA path.
"""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

REF_BIN = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref")


def _run(name):
    path = os.path.join(REF_BIN, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} not built (make -C oracle ref REF=<reference checkout>)")
    out = subprocess.run([path], capture_output=True, text=True, timeout=600)
    return out.returncode, out.stdout + out.stderr


def test_reference_w8a8_program_passes():
    rc, text = _run("test_w8a8")
    assert rc == 0, text[-2000:]
    assert "w8a8: OK" in text


def test_reference_tmac_program_passes():
    rc, text = _run("tmac_lut")
    assert rc == 0, text[-2000:]
    assert "tmac: OK" in text and "FAIL" not in text
