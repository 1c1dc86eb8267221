"""Expert-parallel helpers: the NCCL unique id and the host-side exchange plan.

The exchange itself runs inside libhf_moe.so (hf_moe_forward with
ep_world > 1). These helpers give Python callers the id to share between
ranks and the exchange order the library uses (hf_ep_plan), which the CPU
tests check against a multi-process simulation.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import call


def unique_id() -> bytes:
    """A fresh 128-byte NCCL unique id (make it on rank 0, share it)."""
    buf = ctypes.create_string_buffer(128)
    call("hf_ep_unique_id", ctypes.cast(buf, ctypes.c_void_p))
    return buf.raw


def broadcast_unique_id(dist, rank: int, device) -> bytes:
    """Rank 0 makes the id; torch.distributed broadcasts it to every rank."""
    import torch
    t = torch.zeros(128, dtype=torch.uint8, device=device)
    if rank == 0:
        t.copy_(torch.frombuffer(bytearray(unique_id()), dtype=torch.uint8))
    dist.broadcast(t, 0)
    return bytes(t.cpu().numpy().tobytes())


def exchange_plan(world: int, e_local: int, t_local: int, has_shared: bool,
                  send_counts: np.ndarray, recv_counts: np.ndarray) -> dict:
    """hf_ep_plan: offsets and the receiver-side row order of one exchange.

    send_counts / recv_counts: int32 [world, e_local] rows this rank sends to
    / receives from each rank per local expert."""
    sc = np.ascontiguousarray(send_counts, np.int32).reshape(world, e_local)
    rc = np.ascontiguousarray(recv_counts, np.int32).reshape(world, e_local)
    R = int(rc.sum())
    n_local = R + (t_local if has_shared else 0)
    out = dict(send_off=np.zeros(world + 1, np.int32), recv_off=np.zeros(world + 1, np.int32),
               local_counts=np.zeros(e_local + 1, np.int32),
               local_rows=np.zeros(max(1, n_local), np.int32), row_pos=np.zeros(max(1, R), np.int32))
    p = lambda a: a.ctypes.data  # noqa: E731
    call("hf_ep_plan", world, e_local, t_local, int(has_shared), p(sc), p(rc), p(out["send_off"]),
         p(out["recv_off"]), p(out["local_counts"]), p(out["local_rows"]), p(out["row_pos"]))
    out["local_rows"] = out["local_rows"][:n_local]
    out["row_pos"] = out["row_pos"][:R]
    out["R"] = R
    return out
