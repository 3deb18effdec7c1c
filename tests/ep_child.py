"""One rank of the 2-GPU expert-parallel parity test (launched by torchrun from
tests/test_gpu_ep.py): decodes the shared problem with the bank sharded over
the ranks, with the all-gather ("ag") or all-to-all ("a2a") exchange, and
writes this rank's tokens to <out>_<rank>.npy."""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.abspath(os.path.join(os.path.dirname(__file__), "..")))
from sabah_moe_accelerator_b200 import ep, ops  # noqa: E402
from test_gpu_ep import D, E, F, K, LAYERS, QT, T, problem  # noqa: E402


def main(out, exchange):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    try:
        ops.init(local)
        e0, e1 = ep.expert_range(rank, E, world)
        banks, ids, w, x0 = problem(e0, e1)
        if exchange == "ag":
            plans = ep.pack_plans([ep.plan_layer(ids[L], w[L], rank, world, E) for L in range(LAYERS)])
        else:
            plans = ep.pack_plans_a2a([ep.plan_layer_a2a(ids[L], w[L], rank, world, E) for L in range(LAYERS)])
        t0, t1 = ep.token_range(rank, T, world)
        x = torch.from_numpy(x0[t0:t1]).cuda()
        ep.decode_step(x, plans, ep.CudaOps(banks, D, F, e1 - e0, QT), ep.TorchComm(), exchange)
        torch.cuda.synchronize()
        np.save("%s_%d.npy" % (out, rank), x.cpu().numpy())
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "ag")
