"""GPU: the allocation-free layer entry (moeb_layer_forward_static) against the workspace entry.

Some callers cannot allocate device memory where they run a layer: a host whose memory manager has
reserved all of HBM into its own pools, a plug-in that must not disturb that allocator, or a
latency-critical path that cannot pay cudaMalloc's implicit synchronisation. For them the library
keeps the workspace in a static device array. This file is collected last, so a run that stops at
its first failure has run every other test before it; it also passes alone in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import host_layer
from llapis_b200 import capi, workload
from llapis_b200.layer import MoELayer

pytestmark = pytest.mark.gpu


def _forward_static(layer, x):
    out = torch.empty_like(x)
    rc = capi.lib().moeb_layer_forward_static(C.byref(layer.c), x.data_ptr(), x.shape[0], out.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream)
    capi.check(rc)
    return out


def test_static_scratch_entry_matches_workspace_entry():
    """Both entries run the same decode kernel on the same 8-token chunks (every reduction in a
    fixed order), so their outputs must be identical bit for bit."""
    host = host_layer("decode_t4_mixed")
    layer = MoELayer(host)
    cfg = workload.CONFIGS["decode_t4_mixed"]
    # two calls in a row, different inputs and token counts (the second runs as three 8-token chunks)
    for T, seed in ((4, 101), (20, 102)):
        x = torch.from_numpy(workload.make_input(cfg, n_tokens=T, stream=seed)).cuda()
        got = _forward_static(layer, x)
        want = layer(x)
        torch.cuda.synchronize()
        assert np.array_equal(got.cpu().numpy().view(np.uint32), want.cpu().numpy().view(np.uint32)), f"T={T}"
    assert layer.device_error() == 0


def test_static_scratch_entry_rejects_oversized_layer():
    """A layer whose workspace exceeds the static array is refused with MOEB_ESPACE, before any
    device work."""
    host = host_layer("mini_mixed")
    layer = MoELayer(host)
    big = capi.Layer.from_buffer_copy(layer.c)
    big.d_model = 65536          # workspace of 16 tokens x 65536 features no longer fits
    x = torch.zeros((1, 8), dtype=torch.float32, device="cuda")
    rc = capi.lib().moeb_layer_forward_static(C.byref(big), x.data_ptr(), 16, x.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == -4, capi.lib().moeb_last_error()
    assert b"static scratch" in capi.lib().moeb_last_error()
