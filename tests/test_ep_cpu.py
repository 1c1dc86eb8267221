"""Expert-parallel exchange order on CPU ranks (gloo), no GPU.

Each rank routes its own tokens (seeded random top-k), builds the canonical
permutation over all experts (the oracle's counting sort), exchanges counts
and "rows" (the global slot id each row carries) with the other ranks, and
orders what it received with hf_ep_plan -- the same host code the GPU forward
uses. Checks: every local expert's segment on its owner equals the expert's
segment of the single-process permutation of all tokens (same tokens, same
order), and the return trip puts each row back at its slot's canonical
position on the source. Also: the failure path -- a rank that never joins --
ends in a timeout error on the others instead of a hang.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _routing(T, E, k, seed):
    rng = np.random.default_rng(seed)
    return np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)


def _worker(rank, world, port, E, k, T_local, errq):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60))
        from hummingflight_b200.ep import exchange_plan
        El = E // world
        T = T_local * world
        ids_all = _routing(T, E, k, 5)
        ids = ids_all[rank * T_local:(rank + 1) * T_local]
        counts, offsets, perm = O.permute(ids, E, has_shared=True)
        send_counts = counts[:E].reshape(world, El)
        # counts exchange (all_gather stands in for the all-to-all)
        allc = [torch.zeros(world * El, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(allc, torch.from_numpy(send_counts.reshape(-1).copy()))
        recv_counts = np.stack([allc[s].numpy().reshape(world, El)[rank] for s in range(world)])
        p = exchange_plan(world, El, T_local, True, send_counts, recv_counts)
        # rows carry their global slot id: (token_global * k + i)
        slots = perm[:T_local * k]
        t_glob = slots // k + rank * T_local
        gslot = (t_glob * k + slots % k).astype(np.int64)
        maxr = T * k
        payload = np.full((world, maxr), -1, np.int64)
        for d in range(world):
            seg = gslot[p["send_off"][d]:p["send_off"][d + 1]]
            payload[d, :len(seg)] = seg
        gathered = [torch.zeros(world * maxr, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(payload.reshape(-1)))
        recv = np.concatenate([gathered[s].numpy().reshape(world, maxr)[rank]
                               [:p["recv_off"][s + 1] - p["recv_off"][s]] for s in range(world)])
        assert len(recv) == p["R"]
        # local positions: expert-major segments must equal the global ones
        _, goff, gperm = O.permute(ids_all, E, has_shared=True)
        lc = p["local_counts"]
        assert lc[El] == T_local
        base = np.concatenate([[0], np.cumsum(lc)])
        for j in range(El):
            e = rank * El + j
            mine = recv[p["local_rows"][base[j]:base[j + 1]]]
            ref = gperm[goff[e]:goff[e + 1]]
            assert np.array_equal(mine, ref), (rank, j)
        shared_rows = p["local_rows"][base[El]:base[El + 1]]
        assert np.array_equal(shared_rows, p["R"] + np.arange(T_local))
        # row_pos inverts local_rows on the received rows
        pos = np.arange(p["R"])
        assert np.array_equal(p["local_rows"][p["row_pos"]], pos)
        # return trip: the device gathers outputs through row_pos back into
        # arrival order and sends each source its segment; the source places
        # it at send_off + i, which must be the slot's own canonical position
        local_out = np.empty(p["R"], np.int64)        # output row at each local position
        local_out[p["row_pos"]] = recv                # (tagged with its slot id)
        ysend = local_out[p["row_pos"]]
        back = np.full((world, maxr), -1, np.int64)
        for s in range(world):
            seg = ysend[p["recv_off"][s]:p["recv_off"][s + 1]]
            back[s, :len(seg)] = seg
        g2 = [torch.zeros(world * maxr, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(g2, torch.from_numpy(back.reshape(-1)))
        yrecv = np.concatenate([g2[d].numpy().reshape(world, maxr)[rank]
                                [:p["send_off"][d + 1] - p["send_off"][d]] for d in range(world)])
        assert np.array_equal(yrecv, gslot)
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # noqa: BLE001
        errq.put(f"rank {rank}: {type(e).__name__}: {e}")
        raise


@pytest.mark.parametrize("world,E,k,T_local", [(2, 16, 4, 7), (4, 32, 8, 5), (2, 8, 8, 3)])
def test_exchange_order_matches_single_process(world, E, k, T_local):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, E, k, T_local, errq))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not errs, errs
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def _lonely(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    if rank == 1:
        return  # never joins: the failure the others must detect
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=timedelta(seconds=3))
        q.put("joined")
    except Exception as e:  # noqa: BLE001
        q.put(type(e).__name__)


def test_missing_rank_times_out_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lonely, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    assert all(not p.is_alive() for p in procs)
    msg = q.get(timeout=5)
    assert msg != "joined"
