"""Expert-parallel layer on 2 GPUs (NCCL dispatch/combine) against the
single-GPU layer on the whole batch: routing ids, drops and renormalized
weights bit-exact, layer output within the north_star tolerance 1e-3
relative (fp32 atomics in no fixed order; the tensor cores' fp32 sums of
the routed gate/up may round differently when a row sits at another
position of another tile).  Needs at least two GPUs."""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("Tl,cf", [(96, 1.5), (200, 1.0)])
def test_ep_two_ranks_match_single_gpu(tmp_path, Tl, cf):
    out = tmp_path / "ep.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(HERE, "ep_worker.py"), str(out), str(Tl), str(cf)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["ids"] and res["drop"] and res["w"], res
    assert res["err"] < 1e-3, res
    if cf == 1.0:
        assert res["drops"] > 0
