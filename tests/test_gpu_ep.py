"""The expert half on given routing (moeb_layer_forward_routed) and the expert-parallel forward at
world size 1 over NCCL, on a B200 (-m gpu). Multi-rank runs: bench.py --config
ep_prefill_t8192_q4k under torchrun; tests/test_gpu_ep_multi.py runs the 2-GPU parity check."""
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist

from conftest import assert_layer_close, host_layer
from llapis_b200 import workload
from llapis_b200.layer import MoELayer

pytestmark = pytest.mark.gpu


def test_routed_halves_sum_to_full():
    """Masking complementary halves of each token's experts to -1 gives partial sums that add up
    to the routed output over all k experts (and that equals the whole-layer forward)."""
    host = host_layer("decode_t4_mixed")
    layer = MoELayer(host)
    x = torch.from_numpy(workload.make_input(workload.CONFIGS["decode_t4_mixed"], n_tokens=200, stream=3)).cuda()
    _, ids, w = layer.route(x)
    full = layer.forward_routed(x, ids, w).clone()
    odd = (torch.arange(host.top_k, device="cuda") % 2 == 1)[None, :]
    a = layer.forward_routed(x, torch.where(odd, ids, -1).contiguous(), w).clone()
    b = layer.forward_routed(x, torch.where(~odd, ids, -1).contiguous(), w).clone()
    ref = full.cpu().numpy()
    assert_layer_close((a + b).cpu().numpy(), ref, tol=1e-5)
    # the whole-layer forward routes with the router's K split in four parts (summed in order),
    # moeb_layer_route in one: logits agree to f32 rounding, outputs to far below the parity bar
    layer_out = layer(x).cpu().numpy()
    assert_layer_close(layer_out, ref, tol=5e-5 if layer.prefill_path(200) else 5e-4)
    none = layer.forward_routed(x, torch.full_like(ids, -1), w)
    assert torch.count_nonzero(none).item() == 0


def test_routed_q8k_rows_equal_f32_rows():
    """The expert half on Q8_K rows quantised by moeb_quantize_act gives the same bits as on the f32
    rows it quantises itself (the expert-parallel exchange sends the Q8_K rows)."""
    host = host_layer("decode_t4_mixed")
    layer = MoELayer(host)
    x = torch.from_numpy(workload.make_input(workload.CONFIGS["decode_t4_mixed"], n_tokens=150, stream=4)).cuda()
    _, ids, w = layer.route(x)
    a = layer.forward_routed(x, ids, w).clone()
    xq = layer.quantize_q8k(x)
    assert xq.shape == (150, 11 * 292)
    b = layer.forward_routed_q8k(xq, ids, w).clone()
    torch.cuda.synchronize()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))
    assert layer.device_error() == 0


def test_ep_world1_matches_layer():
    from llapis_b200.ep import EPMoE
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1,
                            timeout=timedelta(seconds=120), device_id=torch.device("cuda", 0))
    try:
        host = host_layer("mini_mixed")
        layer = MoELayer(host)
        x = torch.from_numpy(workload.make_input(workload.CONFIGS["mini_mixed"], n_tokens=300, stream=8)).cuda()
        out = EPMoE.from_layer(layer)(x)
        out_f32 = EPMoE.from_layer(layer, wire="f32")(x)
        assert torch.equal(out.view(torch.int32), out_f32.view(torch.int32))   # Q8_K rows on the wire: same bits
        want = layer(x)
        assert_layer_close(out.cpu().numpy(), want.cpu().numpy(), tol=5e-5 if layer.prefill_path(300) else 5e-4)
    finally:
        dist.destroy_process_group()
