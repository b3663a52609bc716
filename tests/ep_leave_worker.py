"""Worker of tests/test_gpu_ep_watchdog.py (torch.distributed.run, one
process per GPU, NVLS off): both ranks run one expert-parallel forward and
synchronize; then rank 1 leaves (between steps, nothing of it in flight)
and rank 0 runs the next forward with a 3 s deadline.  The forward's wait
for the gathered counts must end with an error (the watchdog aborts the
communicator), the communicator must report itself failed, and the GPU
must still run work: a W8A8 GEMM afterwards and jt_b200_sync() == 0.  Rank 0
writes the verdict to argv[1]."""
import json
import os
import sys
import time

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    import torch
    import torch.distributed as dist
    from jimotono_b200 import lib
    from jimotono_b200.moe import WEIGHT_FIELDS, Dims, EpComm, EpPlan, MoeWeights, synth_inputs, synth_weights
    out_path = sys.argv[1]
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo")
    Tl, d, f, E, k, S, fs, cf = 64, 256, 128, 16, 4, 2, 128, 1.5
    dmg = Dims(Tl * world, d, f, E, k, S, fs, cf)
    w = synth_weights(dmg, seed=21)
    x, logits, bias = synth_inputs(dmg, Tl * world, seed=22)
    El = E // world
    routed = {"wg", "wu", "sg", "su", "wd", "sd"}
    dev = {}
    for n in WEIGHT_FIELDS:
        a = np.ascontiguousarray(w[n][rank * El:(rank + 1) * El] if n in routed else w[n])
        dev[n] = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()
    wp = MoeWeights(*[dev[n].data_ptr() for n in WEIGHT_FIELDS])
    uid = [EpComm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    comm = EpComm(uid[0], world, rank)
    plan = EpPlan(Dims(Tl, d, f, E, k, S, fs, cf), comm)
    sl = slice(rank * Tl, (rank + 1) * Tl)
    dx = torch.from_numpy(np.ascontiguousarray(x[sl])).cuda()
    dl = torch.from_numpy(np.ascontiguousarray(logits[sl])).cuda()
    y = torch.zeros((Tl, d), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    plan.forward(wp, dx.data_ptr(), dl.data_ptr(), None, y.data_ptr(), False, stream)
    assert lib().jt_b200_sync() == 0
    dist.barrier()  # both ranks finished the step; nothing in flight
    if rank != 0:
        sys.stdout.flush()
        os._exit(0)  # leaves between steps without destroying anything
    L = lib()
    assert L.jt_b200_ep_comm_set_timeout(comm.handle, 3000) == 0
    t0 = time.perf_counter()
    rc = L.jt_b200_moe_ep_forward(plan.handle, __import__("ctypes").byref(wp), dx.data_ptr(), dl.data_ptr(),
                                  None, y.data_ptr(), 0, stream)
    dt = time.perf_counter() - t0
    err = L.jt_b200_last_error().decode(errors="replace")
    failed = L.jt_b200_ep_comm_failed(comm.handle)
    sync_after = L.jt_b200_sync()
    # the context still runs work
    A = torch.randint(-127, 128, (64, 256), dtype=torch.int8, device="cuda")
    Wt = torch.randint(-127, 128, (128, 256), dtype=torch.int8, device="cuda")
    sa = torch.ones(64, device="cuda")
    sw = torch.ones(128, device="cuda")
    C = torch.zeros((64, 128), device="cuda")
    g = L.jt_b200_w8a8_gemm(A.data_ptr(), 256, sa.data_ptr(), Wt.data_ptr(), 256, sw.data_ptr(), C.data_ptr(), 128,
                            64, 128, 256, stream)
    ok_gemm = g == 0 and L.jt_b200_sync() == 0
    want = (A.float() @ Wt.float().t())
    ok_gemm = ok_gemm and bool(torch.equal(C, want))
    with open(out_path, "w") as fh:
        json.dump({"rc": rc, "seconds": dt, "error": err, "failed": failed, "sync_after": sync_after,
                   "gemm_ok": ok_gemm}, fh)
    sys.stdout.flush()
    os._exit(0)


if __name__ == "__main__":
    main()
