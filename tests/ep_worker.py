"""One rank of the expert-parallel GPU parity check (launched by
tests/test_gpu_ep.py through torch.distributed.run, one process per GPU).

Every rank builds an expert-parallel context (its E/W experts) and a
single-GPU context holding all experts, runs the same global batch (each EP
rank its own slice of tokens) and checks that its routing, per-slot expert
outputs and shared-expert outputs equal the single-GPU ones bit for bit, and
the combined output too whenever both runs use the same router kernel; on
the small shapes it also checks its tokens against the oracle.
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
from hummingflight_b200.configs import GLM, LayerShape  # noqa: E402
from hummingflight_b200.ep import broadcast_unique_id  # noqa: E402
from hummingflight_b200.moe import MoELayer  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    cases = [("small_gemm", LayerShape(256, 16, 4, 128, 192, 2.5, True), 48, "gemm", 41),
             ("small_auto", LayerShape(256, 16, 4, 128, 192, 2.5, True), 40, "auto", 42),
             ("glm_auto", GLM, 16, "auto", 0),
             # 1200 rows: prefill tiles (CTA pairs) on both sides
             ("small_prefill", LayerShape(256, 16, 4, 128, 192, 2.5, True), 600, "auto", 43),
             # slabs above the decode-exchange size: counts sized on the host
             ("glm_sized", GLM, 256, "auto", 3),
             # expert placements other than contiguous ranges
             ("small_placed", LayerShape(256, 16, 4, 128, 192, 2.5, True), 40, "gemm", 44),
             ("glm_placed", GLM, 64, "auto", 5)]
    results = {}
    for name, shape, t_local, path, wseed in cases:
        T = t_local * world
        xb = O.gen_x_bf16(wseed + 100, T, shape.hidden)
        x_all = torch.from_numpy(xb.view(np.int16)).to(dev).view(torch.bfloat16)
        x_mine = x_all[rank * t_local:(rank + 1) * t_local].contiguous()
        uid = broadcast_unique_id(dist, rank, dev)  # one id per communicator
        ep = MoELayer(shape, 1, t_local, local, path, 0, rank, world, uid)
        if name.endswith("_placed"):  # a fixed shuffle of the experts over the ranks
            ep.set_placement(0, np.random.default_rng(wseed).permutation(shape.num_experts))
        ep.synth_layer(0, wseed)
        out_ep, r_ep = ep.forward(0, x_mine, routing=True, slot_out=True)
        ep.synchronize()
        one = MoELayer(shape, 1, T, local, path)
        one.synth_layer(0, wseed)
        out_one, r_one = one.forward(0, x_all, routing=True, slot_out=True)
        one.synchronize()
        sl = slice(rank * t_local, (rank + 1) * t_local)
        k = min(shape.top_k, shape.num_experts)
        # Expert products are bit-identical. The combined output is too when
        # both runs compute the router logits the same way: up to 16 bf16
        # tokens both take the SIMT router; larger batches take the tensor-core
        # router, whose K split (and so its summation order) depends on the
        # batch size and can move a top-k weight by one ulp.
        same_router = T <= 16
        ref = out_one[sl]
        tol = 0.0 if same_router else 1e-6 * float(ref.abs().max())
        ok_out = float((out_ep - ref).abs().max()) <= tol
        ok_w = float((r_ep["topk_weights"] - r_one["topk_weights"][sl]).abs().max()) <= (
            0.0 if same_router else 1e-6)
        ok_ids = torch.equal(r_ep["topk_ids"], r_one["topk_ids"][sl])
        so_ep, so_one = r_ep["slot_out"], r_one["slot_out"]
        ok_slots = torch.equal(so_ep[:t_local * k], so_one[rank * t_local * k:(rank + 1) * t_local * k])
        ok_shared = torch.equal(so_ep[t_local * k:t_local * k + t_local],
                                so_one[T * k + rank * t_local:T * k + (rank + 1) * t_local])
        # this rank's routing outputs, in global expert ids whatever the placement
        c, off, perm = O.permute(r_ep["topk_ids"].cpu().numpy(), shape.num_experts, True)
        ok_ids = ok_ids and (np.array_equal(r_ep["counts"].cpu().numpy(), c) and
                             np.array_equal(r_ep["offsets"].cpu().numpy(), off) and
                             np.array_equal(r_ep["perm"].cpu().numpy(), perm))
        maxdiff = float((out_ep - out_one[sl]).abs().max())
        # and against the oracle (the reference's moeLayer restated) on this
        # rank's tokens: indices off near-ties, outputs on the tokens that
        # route alike within max-abs 2e-2 / rel-L2 1e-3
        ok_oracle = True
        if shape.hidden <= 256:
            d = O.Dims(shape.hidden, shape.num_experts, shape.top_k, shape.inter,
                       shape.shared_inter, shape.scale)
            xo = O.bf16_to_f32(xb[rank * t_local:(rank + 1) * t_local]).reshape(t_local, -1)
            orc = O.moe_layer_synth(d, wseed, 0, xo)
            ids = r_ep["topk_ids"].cpu().numpy()
            firm = orc["margins"] > 1e-4
            agree = np.all(ids == orc["ids"], axis=1)
            got = out_ep.cpu().numpy().astype(np.float64)[agree]
            exp = orc["out"].astype(np.float64)[agree]
            rel = np.linalg.norm(got - exp) / max(np.linalg.norm(exp), 1e-30)
            ok_oracle = (np.array_equal(ids[firm], orc["ids"][firm]) and agree.mean() >= 0.9
                         and np.abs(got - exp).max() <= 2e-2 and rel <= 1e-3)
        results[name] = dict(out=ok_out and ok_w, ids=ok_ids, slots=ok_slots, shared=ok_shared,
                             oracle=bool(ok_oracle), transport=ep.ep_transport(),
                             maxdiff=maxdiff, same_router=same_router)
        ep.close()
        one.close()
    dist.barrier()
    dist.destroy_process_group()
    # one write() per line: the two ranks share the parent's pipe, and a line
    # under the pipe buffer size is written whole
    sys.stdout.flush()
    sys.stdout.write(f"EPRESULT {rank} {json.dumps(results)}\n")
    sys.stdout.flush()
    bad = [n for n, r in results.items()
           if not (r["out"] and r["ids"] and r["slots"] and r["shared"] and r["oracle"])]
    sys.exit(1 if bad else 0)


if __name__ == "__main__":
    main()
