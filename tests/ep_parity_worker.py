"""TEST WORKER — the multi-GPU parity check of the expert-parallel forward, one rank per GPU
(tests/test_gpu_ep_multi.py launches it under torchrun): every rank computes its token shard with
the experts sharded over the ranks; rank 0 gathers the outputs and compares them with the whole
layer on one GPU (moeb_layer_forward, same kernels). Prints one JSON line; exits non-zero on a
mismatch.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 tests/ep_parity_worker.py \
        [config] [n_tokens] [norms]

With "norms" the forward is the Gemma-4 MoE block (the norms on the source rank around the
exchange, against moeb_layer_forward_gemma4 on one GPU; tokens whose top-k is a near tie are left
out, since the single-GPU kernel factors the router's row scale out of the dot) and every step runs
the heartbeat check.
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
    from llapis_b200.ep import EPMoE, Heartbeat, local_experts
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
    use_norms = len(sys.argv) > 3 and sys.argv[3] == "norms"
    norms = workload.block_norms(cfg) if use_norms else None
    x_np = workload.make_block_input(cfg, n_tokens=T, stream=11) if use_norms else workload.make_input(cfg, n_tokens=T,
                                                                                                        stream=11)
    x_all = torch.from_numpy(x_np).to(dev)
    per = T // world
    hb = Heartbeat(dist.distributed_c10d._get_default_store(), rank, world, deadline_s=60.0) if use_norms else None
    ep_layer = EPMoE.from_layer(MoELayer(shard, dev), norms=norms, heartbeat=hb)
    out = ep_layer(x_all[rank * per:(rank + 1) * per].contiguous())
    gathered = [torch.empty_like(out) for _ in range(world)] if rank == 0 else None
    dist.gather(out, gathered, dst=0)
    rc = 0
    if rank == 0:
        ep = torch.cat(gathered).cpu().numpy()
        n = per * world
        logits = torch.empty((n, host.n_expert), dtype=torch.float32, device=dev)
        want = MoELayer(host, dev, norms=norms)(x_all[:n].contiguous(), aux={"logits": logits}).cpu().numpy()
        keep = np.arange(n)
        if use_norms:
            srt = -np.sort(-logits.cpu().numpy(), axis=-1)
            k = host.top_k
            gap = np.abs(srt[:, k - 1] - srt[:, k])
            keep = np.nonzero(gap > 1e-5 * np.maximum(1.0, np.abs(srt[:, k - 1])))[0]
        rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2)))
        err = float(np.max(np.abs(ep[keep] - want[keep])))
        ok = err <= (1e-4 if use_norms else 1e-5) * rms
        print(json.dumps({"check": "ep_parity", "config": name, "n_tokens": n, "world": world, "norms": use_norms,
                          "tokens_compared": int(keep.size), "max_abs_over_rms": err / rms, "ok": ok}))
        rc = 0 if ok else 1
    dist.destroy_process_group()
    return rc


if __name__ == "__main__":
    sys.exit(main())
