"""Prepared weights saved from device buffers and loaded into fresh ones
(jt_b200_moe_weights_save / _load) come back byte for byte."""
import ctypes as C

import numpy as np
import pytest

from jimotono_b200 import lib
from jimotono_b200.moe import WEIGHT_FIELDS, Dims, MoeWeights, synth_weights

pytestmark = pytest.mark.gpu


def test_save_load_device_round_trip(tmp_path):
    from tests import _dev
    dm = Dims(T=1, d=256, f=128, E=8, k=2, S=2, fs=256)
    w = synth_weights(dm, seed=11)
    src = {n: _dev.to_dev(np.ascontiguousarray(w[n]).view(np.uint8)) for n in WEIGHT_FIELDS}
    dst = {n: _dev.zeros(src[n].shape, np.uint8) for n in WEIGHT_FIELDS}
    ws = MoeWeights(*[src[n].data_ptr() for n in WEIGHT_FIELDS])
    wd = MoeWeights(*[dst[n].data_ptr() for n in WEIGHT_FIELDS])
    path = str(tmp_path / "dev.jtb2").encode()
    assert lib().jt_b200_moe_weights_save(path, C.byref(dm.c()), C.byref(ws)) == 0
    assert lib().jt_b200_moe_weights_load(path, C.byref(dm.c()), C.byref(wd)) == 0
    sizes = (C.c_size_t * 12)()
    assert lib().jt_b200_moe_weights_sizes(C.byref(dm.c()), sizes) == 0
    for n, sz in zip(WEIGHT_FIELDS, sizes):
        a = _dev.host(src[n]).reshape(-1)[:sz]
        b = _dev.host(dst[n]).reshape(-1)[:sz]
        assert np.array_equal(a, b), n
