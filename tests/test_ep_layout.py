"""Expert-parallel bookkeeping (jt_ep_layout.c) on the CPU.

* single process: for N ranks holding consecutive token slices, the pairs
  every rank keeps under the layout's rule equal the pairs the reference's
  capacity sort keeps over the whole batch (restated by the oracle's
  jto_batch_sort, which is pinned to moe_layer.c:895-978);
* two and four gloo ranks: each rank counts its own pairs, the counts are
  all-gathered over torch.distributed (gloo, 127.0.0.1), and the send and
  receive sizes the ranks compute agree pairwise.
"""
import ctypes as C
import os

import numpy as np
import pytest

import oracle
from jimotono_b200 import lib
from jimotono_b200.moe import ep_layout


def _routing(T, k, E, seed, zipf=1.2):
    rng = np.random.default_rng(seed)
    return ((rng.zipf(zipf, (T, k)) - 1) % E).astype(np.int32)


def _oracle_kept(ids, T, k, E, cap_factor):
    flat = np.ascontiguousarray(ids.reshape(-1))
    perm = np.zeros(T * k, np.int32)
    off = np.zeros(E + 1, np.int32)
    drop = np.zeros(T * k, np.uint8)
    kept = C.c_int(0)
    assert oracle.oracle().jto_batch_sort(flat.ctypes.data, T, k, E, cap_factor, perm.ctypes.data,
                                          off.ctypes.data, drop.ctypes.data, C.addressof(kept)) == 0
    return drop == 0


@pytest.mark.parametrize("N,Tl,k,E,cf", [(2, 300, 4, 16, 1.0), (4, 128, 8, 64, 1.25), (8, 64, 8, 1024, 1.5),
                                         (3, 50, 2, 9, 1.0), (1, 200, 4, 8, 1.5)])
def test_layout_reproduces_global_capacity_sort(N, Tl, k, E, cf):
    T = N * Tl
    ids = _routing(T, k, E, seed=N * 100 + E)
    want_keep = _oracle_kept(ids, T, k, E, cf)
    cap = lib().jt_b200_ep_capacity(T, k, E, cf)
    assert cap > 0
    cnt = np.stack([np.bincount(ids[r * Tl:(r + 1) * Tl].reshape(-1), minlength=E) for r in range(N)]).astype(np.int32)
    El = E // N
    keep = np.zeros(T * k, bool)
    lays = [ep_layout(cnt, r, cap) for r in range(N)]
    for r in range(N):
        lay = lays[r]
        local = ids[r * Tl:(r + 1) * Tl].reshape(-1)
        seen = np.zeros(E, np.int64)
        for q, e in enumerate(local):  # local stable order, capacity left after lower ranks
            keep[r * Tl * k + q] = lay["gbase"][e] + seen[e] < cap
            seen[e] += 1
        # what rank r sends to owner o = its kept pairs of o's experts
        for o in range(N):
            sel = keep[r * Tl * k:(r + 1) * Tl * k] & (local // El == o)
            assert lay["send"][o] == sel.sum()
    assert np.array_equal(keep, want_keep)
    for r in range(N):
        for s in range(N):
            assert lays[r]["recv"][s] == lays[s]["send"][r]
        own = lays[r]["own_off"]
        assert own[-1] == sum(lays[s]["send"][r] for s in range(N))
        g = lays[r]["gather"]
        # every owned row is written exactly once
        dst = np.concatenate([np.arange(g[s, el, 1], g[s, el, 1] + g[s, el, 2])
                              for s in range(N) for el in range(El)])
        assert np.array_equal(np.sort(dst), np.arange(own[-1]))


def _gloo_worker(rank, world, port, result):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        Tl, k, E = 96, 4, 32
        ids = _routing(world * Tl, k, E, seed=77)[rank * Tl:(rank + 1) * Tl]
        cnt = torch.from_numpy(np.bincount(ids.reshape(-1), minlength=E).astype(np.int32))
        gathered = [torch.zeros_like(cnt) for _ in range(world)]
        dist.all_gather(gathered, cnt)
        cnt_all = torch.stack(gathered).numpy()
        cap = lib().jt_b200_ep_capacity(world * Tl, k, E, 1.0)
        lay = ep_layout(cnt_all, rank, cap)
        send = torch.from_numpy(lay["send"].copy())
        sends = [torch.zeros_like(send) for _ in range(world)]
        dist.all_gather(sends, send)
        ok = all(int(sends[s][rank]) == int(lay["recv"][s]) for s in range(world))
        result[rank] = 1 if ok else 0
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_layout_gloo_ranks(world):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as sck:
        sck.bind(("127.0.0.1", 0))
        port = sck.getsockname()[1]
    ctx = mp.get_context("spawn")
    result = ctx.Array("i", [0] * world)
    procs = [ctx.Process(target=_gloo_worker, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    assert list(result) == [1] * world
