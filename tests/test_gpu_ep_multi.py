"""The expert-parallel forward on 2 GPUs against the whole layer on one (-m gpu; skipped on a box
with fewer than two GPUs). The ranks run as child processes under torchrun over NCCL
(tests/ep_parity_worker.py), with NVLS off and a bounded process-group timeout."""
import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("name,T,mode", [("ep_prefill_t8192_q4k", 2048, ""), ("ep_prefill_t8192_q4k", 600, ""),
                                         ("ep_prefill_t8192_q4k", 600, "norms")])
def test_ep_two_ranks_match_single_gpu(name, T, mode):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", MASTER_ADDR="127.0.0.1")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node", "2", "--master-addr", "127.0.0.1", "--master-port", "29531",
           os.path.join(ROOT, "tests", "ep_parity_worker.py"), name, str(T)] + ([mode] if mode else [])
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert r.returncode == 0 and lines, r.stdout[-2000:] + r.stderr[-2000:]
    res = json.loads(lines[-1])
    print(res)
    assert res["ok"] and res["world"] == 2
    if mode == "norms":
        assert res["tokens_compared"] >= 0.9 * res["n_tokens"]
