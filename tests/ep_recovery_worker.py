"""One rank of the expert-parallel recovery checks (launched by
tests/test_gpu_ep.py through torch.distributed.run, one process per GPU, NVLS
off). Two parts:

1. Transport agreement. With HF_EP_FAIL_P2P_ON_RANK=1, rank 1 reports a failed
   peer mapping at hf_moe_create; every rank must then fall back to the same
   NCCL exchange (none may stay on peer memory while another waits in NCCL),
   and the forward must still equal the single-GPU one.
2. A skipped forward. On peer memory, rank 1 skips one forward between steps
   (it stays alive, no kernel or collective of it in flight) while rank 0 runs
   it with a 1 ms wait limit: rank 0's bounded flag waits run out and its
   forward reports HF_ERR_TIMEOUT; the context stays usable. Both ranks then
   call hf_moe_ep_resync and the next forward on both is correct again
   (equal to the first forward on the same input).
"""
import json
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from hummingflight_b200.configs import LayerShape  # noqa: E402
from hummingflight_b200.ep import broadcast_unique_id  # noqa: E402
from hummingflight_b200.moe import HfError, MoELayer  # noqa: E402

SHAPE = LayerShape(256, 16, 4, 128, 192, 2.5, True)
WSEED, T_LOCAL = 51, 32


def inputs(rank, world, dev):
    T = T_LOCAL * world
    xb = O.gen_x_bf16(WSEED + 7, T, SHAPE.hidden)
    x_all = torch.from_numpy(xb.view(np.int16)).to(dev).view(torch.bfloat16)
    return x_all, x_all[rank * T_LOCAL:(rank + 1) * T_LOCAL].contiguous()


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    x_all, x = inputs(rank, world, dev)
    res = {}

    # single-GPU reference of the same batch
    one = MoELayer(SHAPE, 1, T_LOCAL * world, local, "gemm")
    one.synth_layer(0, WSEED)
    ref = one.forward(0, x_all)[rank * T_LOCAL:(rank + 1) * T_LOCAL].clone()
    one.synchronize()
    one.close()

    # 1. a rank that cannot map its peers: all ranks agree on NCCL
    os.environ["HF_EP_FAIL_P2P_ON_RANK"] = "1"
    uid = broadcast_unique_id(dist, rank, dev)
    ep = MoELayer(SHAPE, 1, T_LOCAL, local, "gemm", 0, rank, world, uid)
    del os.environ["HF_EP_FAIL_P2P_ON_RANK"]
    ep.synth_layer(0, WSEED)
    transports = [None] * world
    dist.all_gather_object(transports, ep.ep_transport())
    out = ep.forward(0, x)
    ep.synchronize()
    res["agreement"] = dict(transports=transports,
                            same=len(set(transports)) == 1 and transports[0] != "peer",
                            maxdiff=float((out - ref).abs().max()))
    ep.close()
    dist.barrier()

    # 2. peer memory; rank 1 skips a forward
    uid = broadcast_unique_id(dist, rank, dev)
    ep = MoELayer(SHAPE, 1, T_LOCAL, local, "gemm", 0, rank, world, uid)
    ep.synth_layer(0, WSEED)
    res["transport"] = ep.ep_transport()
    first = ep.forward(0, x).clone()
    ep.synchronize()
    dist.barrier()
    status = None
    if rank == 0:
        ep.set_wait_timeout(1_000_000)  # 1 ms
        ep.forward(0, x)
        try:
            ep.synchronize()
            status = 0
        except HfError as e:
            status = e.status
        ep.set_wait_timeout(0)  # back to the default limit
    dist.barrier()  # rank 1 joins here without having run that forward
    ep.ep_resync()
    again = ep.forward(0, x)
    ep.synchronize()
    res["skip"] = dict(status=status, recovered=bool(torch.equal(again, first)),
                       first_vs_single=float((first - ref).abs().max()))
    ep.close()
    dist.barrier()
    dist.destroy_process_group()
    # one write() per line: the two ranks share the parent's pipe, and a line
    # under the pipe buffer size is written whole
    sys.stdout.flush()
    sys.stdout.write(f"EPRECOVERY {rank} {json.dumps(res)}\n")
    sys.stdout.flush()
    ok = (res["agreement"]["same"] and res["agreement"]["maxdiff"] <= 1e-5 and
          res["transport"] == "peer" and res["skip"]["recovered"] and
          res["skip"]["first_vs_single"] <= 1e-5 and
          (rank != 0 or res["skip"]["status"] == 4))
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
