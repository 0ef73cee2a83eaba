"""The Gemma-4 feed-forward block on a B200 (-m gpu): the MoE block plus the dense MLP branch
(gemma4.cpp:376-431), the dense branch on a side stream. The block's output is the two branches'
outputs added, bit for bit, with or without the side stream; against the oracle's two branches
within the parity bar."""
import numpy as np
import pytest
import torch

from conftest import assert_layer_close, host_layer, spec_of
from llapis_b200 import workload
from llapis_b200.layer import FfnBlock, MoELayer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def block():
    cfg = workload.CONFIGS["decode_t4_mixed"]
    moe = MoELayer(host_layer("decode_t4_mixed"), norms=workload.block_norms(cfg))
    mlp = MoELayer(workload.build_dense_layer(), norms=workload.dense_block_norms())
    return FfnBlock(moe, mlp)


@pytest.mark.parametrize("T", [4, 96])
def test_ffn_block_is_the_sum_of_its_branches(block, T):
    x = torch.from_numpy(workload.make_block_input(workload.CONFIGS["decode_t4_mixed"], n_tokens=T, stream=5)).cuda()
    side = torch.cuda.Stream()
    got = block(x, side_stream=side)
    seq = block(x)
    a, b = block.moe(x), block.mlp(x)
    torch.cuda.synchronize()
    want = (a.cpu().numpy() + b.cpu().numpy()).astype(np.float32)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert np.array_equal(seq.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert block.moe.device_error() == 0


def test_ffn_block_vs_oracle(block, port):
    T = 96
    x = workload.make_block_input(workload.CONFIGS["decode_t4_mixed"], n_tokens=T, stream=6)
    got = block(torch.from_numpy(x).cuda(), side_stream=torch.cuda.Stream())
    torch.cuda.synchronize()
    moe = port.gemma4_block(spec_of(block.moe.host, x), block.moe.norms, n_threads=8, want=())["out"]
    mlp = port.gemma4_block(spec_of(block.mlp.host, x), block.mlp.norms, n_threads=8, want=())["out"]
    want = (moe + mlp).astype(np.float32)
    rel = assert_layer_close(got.cpu().numpy(), want)
    print(f"ffn block T={T} vs oracle: max-abs / rms {rel:.2e}")
