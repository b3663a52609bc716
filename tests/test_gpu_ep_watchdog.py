"""Failure detection of the expert-parallel layer on two GPUs, without a GPU
fault: a rank leaves between steps, the other rank's next forward waits
for the gathered counts under a 3 s deadline, the watchdog aborts the
communicator and the forward returns an error; the GPU keeps running work
(tests/ep_leave_worker.py).  NVLS is off, as for every multi-rank test
whose ranks may leave."""
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
def test_rank_leaving_between_steps_is_detected(tmp_path):
    out = tmp_path / "leave.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "180", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29547",
           os.path.join(HERE, "ep_leave_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["rc"] != 0, res
    assert res["failed"] == 1, res
    assert res["seconds"] < 60, res
    assert res["gemm_ok"], res
