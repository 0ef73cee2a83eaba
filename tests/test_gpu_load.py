"""Layers loaded from files straight into the HBM class pools (llapis_b200.loader.load_layer:
moeb_load_file_range for the GGUF's stacked cold tensors, moeb_load_store_pages for the hot slots)
against the same layers uploaded from host arrays: outputs bit-identical on the decode and prefill
paths, with and without the block norms; run on a B200 with -m gpu."""
import time

import numpy as np
import pytest
import torch

from conftest import host_layer
from gguf_fixture import layer_files
from llapis_b200 import workload
from llapis_b200.layer import MoELayer
from test_gpu_prefill import prefill_from  # noqa: F401  (fixture)

pytestmark = pytest.mark.gpu


def same(a: torch.Tensor, b: torch.Tensor) -> bool:
    return np.array_equal(a.cpu().numpy().view(np.uint32), b.cpu().numpy().view(np.uint32))


@pytest.mark.parametrize("split", [False, True])
def test_mini_layer_from_files(tmp_path, prefill_from, split):
    from llapis_b200.loader import load_layer
    name = "mini_mixed"
    host = host_layer(name)
    norms = workload.block_norms(workload.CONFIGS[name])
    gp, sp = str(tmp_path / "m.gguf"), str(tmp_path / "m.gguf.experts.index")
    layer_files(host, norms, gp, sp, il=1, n_layers=2, split_gate_up=split)
    for use_norms in (True, False):
        loaded, nbytes = load_layer(gp, 1, sp, host.hot_ids, use_norms=use_norms)
        want = MoELayer(host, norms=norms if use_norms else None)
        assert nbytes == sum(getattr(host, n).nbytes for n in ("hot_gu", "hot_down", "cold_gu", "cold_down"))
        for thr, T in ((1 << 30, 20), (1, 200)):   # decode path, prefill path
            prefill_from(thr)
            x = torch.from_numpy(workload.make_block_input(workload.CONFIGS[name], n_tokens=T, stream=T)).cuda()
            assert same(loaded(x), want(x))
    torch.cuda.synchronize()
    assert loaded.device_error() == 0


def test_real_shape_layer_from_files(tmp_path):
    """decode_t4_mixed (128 experts: 80 IQ2_S/IQ4_NL from the GGUF, 48 Q4_K/Q5_0 slots from the
    store, 459 MB of pools): bit-identical outputs, and the load throughput beside the pinned
    host-to-device copy rate measured in the same process."""
    from llapis_b200.loader import load_layer
    name = "decode_t4_mixed"
    host = host_layer(name)
    norms = workload.block_norms(workload.CONFIGS[name])
    gp, sp = str(tmp_path / "r.gguf"), str(tmp_path / "r.gguf.experts.index")
    layer_files(host, norms, gp, sp)
    load_layer(gp, 0, sp, host.hot_ids)   # warm: file pages cached, CUDA contexts and allocator ready
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    loaded, nbytes = load_layer(gp, 0, sp, host.hot_ids)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    pin = torch.empty(256 << 20, dtype=torch.uint8).pin_memory()
    dev = torch.empty_like(pin, device="cuda")
    dev.copy_(pin)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    for _ in range(4):
        dev.copy_(pin, non_blocking=True)
    torch.cuda.synchronize()
    h2d = 4 * pin.numel() / (time.perf_counter() - t1)
    print(f"load_layer: {nbytes / 1e6:.1f} MB of pools in {1e3 * dt:.1f} ms = {nbytes / dt / 1e9:.2f} GB/s "
          f"(pinned host-to-device copy {h2d / 1e9:.1f} GB/s)")
    want = MoELayer(host, norms=norms)
    x = torch.from_numpy(workload.make_block_input(workload.CONFIGS[name], n_tokens=4, stream=11)).cuda()
    assert same(loaded(x), want(x))
    assert loaded.device_error() == 0
