"""jimotono_b200 - Python view of libjimotono_b200.so (the B200 hot path).

The library is C11 + sm_100a CUDA behind a C ABI (include/jimotono_b200.h).
This package only loads it with ctypes and declares the prototypes; there
is no Python or CPU implementation of any kernel.  If the shared library is
missing every entry point raises instead of falling back.
"""
from __future__ import annotations

import ctypes
import os

from . import abi as _abi

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libjimotono_b200.so")
_LIB = None


class ExtensionMissing(RuntimeError):
    pass


def lib() -> ctypes.CDLL:
    """Load (once) and return the native library with prototypes set."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ExtensionMissing(
                f"{LIB_PATH} not built: run `python -c 'import __graft_entry__ as g; g.build()'`")
        handle = ctypes.CDLL(LIB_PATH, mode=ctypes.RTLD_LOCAL)
        _abi.declare(handle)
        _LIB = handle
    return _LIB


JT_OK, JT_ERR_NOMEM, JT_ERR_INVAL, JT_ERR_NOSUP, JT_ERR_CUDA = 0, 1, 2, 5, 6


class JtError(RuntimeError):
    def __init__(self, rc: int, what: str):
        super().__init__(f"{what} failed with jt_err {rc}")
        self.rc = rc


def check(rc: int, what: str) -> None:
    if rc != JT_OK:
        detail = lib().jt_b200_last_error().decode(errors="replace")
        raise JtError(rc, f"{what} [{detail}]")
