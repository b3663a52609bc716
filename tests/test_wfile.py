"""On-disk form of the prepared MoE weights (jt_b200_moe_weights_write_host /
_read_host, CPU only): round trip of every array, the header checks
against the layer dims, and rejection of truncated or corrupted files."""
import ctypes as C
import os

import numpy as np

from jimotono_b200 import JT_ERR_INVAL, lib
from jimotono_b200.moe import WEIGHT_FIELDS, Dims, synth_weights

JT_ERR_IO = 3


def _arrays(w, dm):
    sizes = (C.c_size_t * 12)()
    assert lib().jt_b200_moe_weights_sizes(C.byref(dm.c()), sizes) == 0
    arrs = []
    for n, sz in zip(WEIGHT_FIELDS, sizes):
        a = np.ascontiguousarray(w[n]).view(np.uint8).reshape(-1)[:sz] if sz else np.zeros(0, np.uint8)
        assert a.size == sz, (n, a.size, sz)
        arrs.append(np.ascontiguousarray(a))
    return arrs, list(sizes)


def _ptrs(arrs):
    return (C.c_void_p * 12)(*[a.ctypes.data if a.size else None for a in arrs])


def test_round_trip_and_layout(tmp_path):
    dm = Dims(T=1, d=256, f=128, E=4, k=2, S=2, fs=256)
    arrs, sizes = _arrays(synth_weights(dm, seed=3), dm)
    path = str(tmp_path / "w.jtb2")
    assert lib().jt_b200_moe_weights_write_host(path.encode(), C.byref(dm.c()), _ptrs(arrs)) == 0
    raw = np.fromfile(path, np.uint8)
    assert bytes(raw[:8]) == b"JTB2MOE1"
    hdr = raw[:4096].view(np.uint32)
    assert hdr[2] == 1 and hdr[3] == 4096
    offs = raw[40:40 + 96].view(np.uint64)
    assert all(int(o) % 4096 == 0 for o in offs)
    for a, o in zip(arrs, offs):  # arrays stored verbatim at their offsets
        assert np.array_equal(raw[int(o):int(o) + a.size], a)
    back = [np.zeros_like(a) for a in arrs]
    assert lib().jt_b200_moe_weights_read_host(path.encode(), C.byref(dm.c()), _ptrs(back)) == 0
    for a, b in zip(arrs, back):
        assert np.array_equal(a, b)


def test_no_shared_experts(tmp_path):
    dm = Dims(T=1, d=128, f=256, E=3, k=1, S=0, fs=0)
    w = synth_weights(dm, seed=4)
    arrs, sizes = _arrays(w, dm)
    assert sizes[6:] == [0] * 6
    path = str(tmp_path / "w0.jtb2")
    assert lib().jt_b200_moe_weights_write_host(path.encode(), C.byref(dm.c()), _ptrs(arrs)) == 0
    back = [np.zeros_like(a) for a in arrs]
    assert lib().jt_b200_moe_weights_read_host(path.encode(), C.byref(dm.c()), _ptrs(back)) == 0
    assert all(np.array_equal(a, b) for a, b in zip(arrs, back))


def test_rejects_other_dims_truncation_and_corruption(tmp_path):
    dm = Dims(T=1, d=256, f=128, E=4, k=2, S=1, fs=128)
    arrs, _ = _arrays(synth_weights(dm, seed=5), dm)
    path = str(tmp_path / "w.jtb2")
    assert lib().jt_b200_moe_weights_write_host(path.encode(), C.byref(dm.c()), _ptrs(arrs)) == 0
    back = [np.zeros_like(a) for a in arrs]
    other = Dims(T=1, d=256, f=128, E=5, k=2, S=1, fs=128)
    other_arrs, _ = _arrays(synth_weights(other, seed=5), other)
    assert lib().jt_b200_moe_weights_read_host(path.encode(), C.byref(other.c()),
                                               _ptrs([np.zeros_like(a) for a in other_arrs])) == JT_ERR_INVAL
    raw = np.fromfile(path, np.uint8)
    off = int(raw[40 + 8 * 4:40 + 8 * 5].view(np.uint64)[0])  # array 4 (wd)
    bad = raw.copy()
    bad[off + 17] ^= 0x40
    bad_path = str(tmp_path / "bad.jtb2")
    bad.tofile(bad_path)
    sentinel = [np.full_like(a, 0xA5) for a in arrs]
    back = [a.copy() for a in sentinel]
    assert lib().jt_b200_moe_weights_read_host(bad_path.encode(), C.byref(dm.c()), _ptrs(back)) == JT_ERR_IO
    # rejected before any destination is written: the arrays in front of the
    # corrupted one are untouched too
    assert all(np.array_equal(a, b) for a, b in zip(back, sentinel))
    short_path = str(tmp_path / "short.jtb2")
    raw[:raw.size - 5000].tofile(short_path)
    assert lib().jt_b200_moe_weights_read_host(short_path.encode(), C.byref(dm.c()), _ptrs(back)) == JT_ERR_IO
    assert all(np.array_equal(a, b) for a, b in zip(back, sentinel))
    assert lib().jt_b200_moe_weights_read_host(str(tmp_path / "missing").encode(), C.byref(dm.c()),
                                               _ptrs(back)) == JT_ERR_IO
    assert lib().jt_b200_moe_weights_write_host(path.encode(), C.byref(dm.c()), None) == JT_ERR_INVAL
    assert os.path.getsize(path) % 4096 == 0
