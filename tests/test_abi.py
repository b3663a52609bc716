"""CPU checks of the C ABI: the library loads, exports every symbol the
public header declares (and the ctypes table covers them), and the host-side
validation paths that never reach the GPU behave like the reference
(NULL / dimension errors -> JT_ERR_INVAL, M == 0 -> JT_OK untouched,
mode flags)."""
import ctypes as C
import os
import re
import subprocess

import numpy as np

import jimotono_b200
from jimotono_b200 import abi, lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "jimotono_b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w \*]*?\b(jt_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


def test_header_matches_ctypes_table():
    assert header_functions() == sorted(abi.PROTOTYPES)


def test_library_exports_every_declared_symbol():
    out = subprocess.run(["nm", "-D", "--defined-only", jimotono_b200.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if line.strip()}
    missing = [n for n in header_functions() if n not in exported]
    assert not missing, missing
    lib()  # prototypes resolve


def test_version_string():
    assert b"sm_100a" in lib().jt_b200_version()


def test_w8a8_flag_semantics():
    L = lib()
    e = C.c_int(-1)
    assert L.jt_w8a8_set_enabled(0) == 0
    assert L.jt_w8a8_is_enabled() == 0
    assert L.jt_w8a8_get_enabled(C.addressof(e)) == 0 and e.value == 0
    assert L.jt_w8a8_set_enabled(1) == 0 and L.jt_w8a8_is_enabled() == 1
    assert L.jt_w8a8_set_enabled(2) == 2 and L.jt_w8a8_set_enabled(-1) == 2
    assert L.jt_w8a8_get_enabled(None) == 2
    assert L.jt_w8a8_is_enabled() == 1
    assert L.jt_w8a8_set_enabled(0) == 0


def test_gemm_host_validation_without_device():
    """Paths that must return before any CUDA call (w8a8.c:955-971, :910-953)."""
    L = lib()
    A = np.ones((4, 16), np.int8)
    B = np.ones((16, 8), np.int8)
    Cm = np.full((4, 8), 5.0, np.float32)
    sB = np.full(8, 0.5, np.float32)
    a, b, c, s = A.ctypes.data, B.ctypes.data, Cm.ctypes.data, sB.ctypes.data
    # M == 0: OK, C untouched; M == 0 with N == 0: INVAL
    assert L.jt_w8a8_gemm_per_tensor(a, b, 1.0, 1.0, c, 0, 8, 16) == 0
    assert L.jt_w8a8_gemm_per_tensor(a, b, 1.0, 1.0, c, 0, 0, 16) == 2
    assert L.jt_w8a8_gemm_per_channel(a, b, 1.0, s, c, 0, 8, 16) == 0
    # NULLs, negative M, > 4096, bad scales
    assert L.jt_w8a8_gemm_per_tensor(None, b, 1.0, 1.0, c, 4, 8, 16) == 2
    assert L.jt_w8a8_gemm_per_tensor(a, b, 1.0, 1.0, c, -1, 8, 16) == 2
    assert L.jt_w8a8_gemm_per_tensor(a, b, 1.0, 1.0, c, 4097, 8, 16) == 2
    assert L.jt_w8a8_gemm_per_tensor(a, b, 0.0, 1.0, c, 4, 8, 16) == 2
    assert L.jt_w8a8_gemm_per_tensor(a, b, 1.0, float("nan"), c, 4, 8, 16) == 2
    assert L.jt_w8a8_gemm_per_channel(a, b, 1.0, None, c, 4, 8, 16) == 2
    bad = sB.copy()
    bad[3] = 0.0
    assert L.jt_w8a8_gemm_per_channel(a, b, 1.0, bad.ctypes.data, c, 4, 8, 16) == 2
    assert (Cm == 5.0).all()
    # quant / dequant argument checks
    x = np.ones(4, np.float32)
    q = np.zeros(4, np.int8)
    sc = np.zeros(1, np.float32)
    assert L.jt_w8a8_quant_per_tensor(None, 4, q.ctypes.data, sc.ctypes.data) == 2
    assert L.jt_w8a8_quant_per_tensor(x.ctypes.data, 0, q.ctypes.data, sc.ctypes.data) == 2
    assert L.jt_w8a8_dequant_per_tensor(q.ctypes.data, 0.0, 4, x.ctypes.data) == 2
    assert L.jt_w8a8_dequant_per_tensor(q.ctypes.data, float("nan"), 4, x.ctypes.data) == 2


def test_tmac_size_helpers():
    """tmac.c:168-228 on the host: sizes, k % 4 / k % 32 and overflow."""
    import ctypes as C
    from jimotono_b200 import JT_ERR_INVAL, JT_ERR_NOMEM, lib
    L = lib()
    out = C.c_size_t(0)
    assert L.jt_tmac_qlut_bytes(2, 64, C.addressof(out)) == 0 and out.value == 256
    assert L.jt_tmac_qlut_bytes(3, 4, C.addressof(out)) == 0 and out.value == 24
    assert L.jt_tmac_param_bytes(2, 64, C.addressof(out)) == 0 and out.value == 16
    assert L.jt_tmac_param_bytes(3, 4, C.addressof(out)) == JT_ERR_INVAL and out.value == 0
    assert L.jt_tmac_qlut_bytes(2, 6, C.addressof(out)) == JT_ERR_INVAL
    assert L.jt_tmac_qlut_bytes(0, 64, C.addressof(out)) == JT_ERR_INVAL
    assert L.jt_tmac_qlut_bytes(2, 64, None) == JT_ERR_INVAL
    assert L.jt_tmac_qlut_bytes(1 << 62, 64, C.addressof(out)) == JT_ERR_NOMEM
    assert L.jt_tmac_param_bytes(1 << 62, 1 << 10, C.addressof(out)) == JT_ERR_NOMEM
