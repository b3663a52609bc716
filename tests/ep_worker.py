"""Worker of tests/test_gpu_ep.py (launched by torch.distributed.run, one
process per GPU): runs the expert-parallel layer on this rank's token slice
and expert shard, and on rank 0 the single-GPU layer on the whole batch;
rank 0 compares them and writes the verdict to the path in argv[1]."""
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main():
    import torch
    import torch.distributed as dist
    from jimotono_b200 import lib
    from jimotono_b200.moe import (DBG_DROP, DBG_IDS, DBG_WEIGHTS, WEIGHT_FIELDS, Dims, EpComm,
                                   EpPlan, MoeWeights, Plan, synth_inputs, synth_weights)
    out_path = sys.argv[1]
    Tl, d, f, E, k, S, fs, cf = int(sys.argv[2]), 256, 128, 16, 4, 2, 128, float(sys.argv[3])
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("gloo")
    T = Tl * world
    dmg = Dims(T, d, f, E, k, S, fs, cf)
    w = synth_weights(dmg, seed=11)
    x, logits, bias = synth_inputs(dmg, T, seed=12, zipf_s=1.2)
    El = E // world
    routed = {"wg", "wu", "sg", "su", "wd", "sd"}
    dev = {}
    for n in WEIGHT_FIELDS:
        a = w[n][rank * El:(rank + 1) * El] if n in routed else w[n]
        a = np.ascontiguousarray(a)
        dev[n] = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a).cuda()
    wp = MoeWeights(*[dev[n].data_ptr() for n in WEIGHT_FIELDS])
    uid = [EpComm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    comm = EpComm(uid[0], world, rank)
    plan = EpPlan(Dims(Tl, d, f, E, k, S, fs, cf), comm)
    sl = slice(rank * Tl, (rank + 1) * Tl)
    dx = torch.from_numpy(np.ascontiguousarray(x[sl])).cuda()
    dl = torch.from_numpy(np.ascontiguousarray(logits[sl])).cuda()
    db = torch.from_numpy(bias).cuda()
    y = torch.zeros((Tl, d), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # twice: the second call must not see state of the first
        plan.forward(wp, dx.data_ptr(), dl.data_ptr(), db.data_ptr(), y.data_ptr(), False, stream)
    assert lib().jt_b200_sync() == 0
    mine = {"y": y.cpu().numpy(), "ids": plan.debug(DBG_IDS, np.int32, Tl * k),
            "drop": plan.debug(DBG_DROP, np.uint8, Tl * k), "w": plan.debug(DBG_WEIGHTS, np.float32, Tl * k)}
    allp = [None] * world
    dist.all_gather_object(allp, mine)
    if rank == 0:
        fw = {n: torch.from_numpy(np.ascontiguousarray(w[n].view(np.int16) if w[n].dtype == np.uint16 else w[n])).cuda()
              for n in WEIGHT_FIELDS}
        fwp = MoeWeights(*[fw[n].data_ptr() for n in WEIGHT_FIELDS])
        sp = Plan(dmg)
        yy = torch.zeros((T, d), device="cuda")
        # keep the device copies alive until the forward has run
        fx, flg = torch.from_numpy(x).cuda(), torch.from_numpy(logits).cuda()
        sp.forward(fwp, fx.data_ptr(), flg.data_ptr(), db.data_ptr(), T, yy.data_ptr(), False, stream)
        assert lib().jt_b200_sync() == 0
        ids1 = sp.debug(DBG_IDS, np.int32, T * k)
        drop1 = sp.debug(DBG_DROP, np.uint8, T * k)
        w1 = sp.debug(DBG_WEIGHTS, np.float32, T * k)
        y1 = yy.cpu().numpy()
        ids = np.concatenate([p["ids"] for p in allp])
        drop = np.concatenate([p["drop"] for p in allp])
        wt = np.concatenate([p["w"] for p in allp])
        ye = np.concatenate([p["y"] for p in allp])
        err = float(np.abs(ye - y1).max() / max(np.abs(y1).max(), 1e-30))
        res = {"ids": bool(np.array_equal(ids, ids1)), "drop": bool(np.array_equal(drop, drop1)),
               "w": bool(np.array_equal(wt.view(np.uint32), w1.view(np.uint32))), "err": err,
               "drops": int(drop1.sum())}
        with open(out_path, "w") as fh:
            json.dump(res, fh)
        sp.close()
    plan.close()
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
