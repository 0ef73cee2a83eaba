"""TEST WORKER — the multi-GPU parity check of the expert-parallel forward, one rank per GPU
(tests/test_gpu_ep_multi.py launches it under torchrun): every rank computes its token shard with
the experts sharded over the ranks; rank 0 gathers the outputs and compares them with the whole
layer on one GPU (moeb_layer_forward, same kernels). Prints one JSON line; exits non-zero on a
mismatch.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 tests/ep_parity_worker.py \
        [config] [n_tokens]
"""
from __future__ import annotations

import json
import os
import sys
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist


def main() -> int:
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from llapis_b200 import workload
    from llapis_b200.ep import EPMoE, local_experts
    from llapis_b200.layer import MoELayer
    import dataclasses

    name = sys.argv[1] if len(sys.argv) > 1 else "ep_prefill_t8192_q4k"
    rank, local, world = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    cfg = workload.CONFIGS[name]
    T = int(sys.argv[2]) if len(sys.argv) > 2 else cfg.n_tokens
    host = workload.build_layer(cfg)
    mine = local_experts(rank, host.n_expert, world)
    shard = dataclasses.replace(host, hot_ids=mine, hot_gu=host.hot_gu[mine], hot_down=host.hot_down[mine],
                                s_hot=host.s_hot[mine], cold_gu=None, cold_down=None, s_cold=None)
    x_all = torch.from_numpy(workload.make_input(cfg, n_tokens=T, stream=11)).to(dev)
    per = T // world
    out = EPMoE.from_layer(MoELayer(shard, dev))(x_all[rank * per:(rank + 1) * per].contiguous())
    gathered = [torch.empty_like(out) for _ in range(world)] if rank == 0 else None
    dist.gather(out, gathered, dst=0)
    rc = 0
    if rank == 0:
        ep = torch.cat(gathered).cpu().numpy()
        want = MoELayer(host, dev)(x_all[:per * world].contiguous()).cpu().numpy()
        rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
        err = float(np.max(np.abs(ep - want)))
        ok = err <= 1e-5 * rms
        print(json.dumps({"check": "ep_parity", "config": name, "n_tokens": per * world, "world": world,
                          "max_abs_over_rms": err / rms, "ok": ok}))
        rc = 0 if ok else 1
    dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
