"""Router logits on the GPU (jt_b200_moe_router_logits) against the oracle's
restatement of the reference's gate projection (jto_router_logits:
moe_layer.c:1114-1137 with the 4-lane double dot of moe_layer.c:67-86),
bit for bit, including a row whose products cancel heavily; a non-finite
dot is reported through jt_b200_sync."""
import numpy as np
import pytest

import oracle
from jimotono_b200 import JT_ERR_INVAL, lib

pytestmark = pytest.mark.gpu


def _oracle_logits(x, wg):
    T, d = x.shape
    E = wg.shape[0]
    out = np.zeros((T, E), np.float32)
    assert oracle.oracle().jto_router_logits(x.ctypes.data, wg.ctypes.data, T, d, E, out.ctypes.data) == 0
    return out


# up to 32768 logits the chain kernel runs, above it the tiled kernel (ragged
# token and expert tiles in the last two cases)
@pytest.mark.parametrize("T,d,E", [(1, 1024, 64), (37, 2048, 100), (64, 4096, 8), (33, 2048, 257),
                                   (300, 96, 1024), (200, 2048, 300), (16384, 64, 4)])
def test_router_logits_match_oracle(T, d, E):
    from tests import _dev
    rng = np.random.default_rng(T + d + E)
    x = rng.standard_normal((T, d)).astype(np.float32)
    wg = (rng.standard_normal((E, d)) * 0.05).astype(np.float32)
    # cancellation-heavy rows: the double sum is far from every partial sum
    x[0, ::2] = 1e4
    x[0, 1::2] = -1e4
    want = _oracle_logits(x, wg)
    dx, dw = _dev.to_dev(x), _dev.to_dev(wg)
    dl = _dev.zeros((T, E), np.float32)
    assert lib().jt_b200_moe_router_logits(dx.data_ptr(), dw.data_ptr(), T, d, E, dl.data_ptr(), _dev.stream()) == 0
    assert lib().jt_b200_sync() == 0
    got = _dev.host(dl)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"mismatches {(got != want).sum()}"


@pytest.mark.parametrize("T,E", [(4, 8), (64, 1024)])
def test_router_logits_report_non_finite(T, E):
    from tests import _dev
    x = np.ones((T, 64), np.float32)
    x[1, 3] = np.inf
    wg = np.ones((E, 64), np.float32)
    dl = _dev.zeros((T, E), np.float32)
    dx, dw = _dev.to_dev(x), _dev.to_dev(wg)
    assert lib().jt_b200_moe_router_logits(dx.data_ptr(), dw.data_ptr(), T, 64, E, dl.data_ptr(), _dev.stream()) == 0
    assert lib().jt_b200_sync() != 0
    assert lib().jt_b200_sync() == 0


def test_router_logits_reject_bad_arguments():
    L = lib()
    buf = np.zeros(64, np.float32)
    p = buf.ctypes.data
    assert L.jt_b200_moe_router_logits(None, p, 1, 64, 8, p, None) == JT_ERR_INVAL
    assert L.jt_b200_moe_router_logits(p, p, 1, 48, 8, p, None) == JT_ERR_INVAL      # d % 32
    assert L.jt_b200_moe_router_logits(p, p, 0, 64, 8, p, None) == JT_ERR_INVAL      # T
    assert L.jt_b200_moe_router_logits(p + 4, p, 1, 64, 8, p, None) == JT_ERR_INVAL  # alignment
