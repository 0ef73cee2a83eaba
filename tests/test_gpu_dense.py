"""Gemma-4's dense (shared) MLP on a B200 (-m gpu), as this path's layer with one expert: d_model
2816, inner width 2112 (Q4_K gate / up, Q5_0 down), every token routed to the one expert at top-1
with weight 1.0. Against the REFERENCE's own build_ffn output (tests/golden/make_golden.py --dense):
gate_up bit for bit on every token (per-token digests), the GeGLU-quantised activations through
them, outputs within the parity bar. The decode kernel does not fit this width, so every batch size
runs the prefill kernels; a token's output does not depend on the batch it runs in."""
import hashlib
import os

import numpy as np
import pytest

from conftest import ROOT, sha
from llapis_b200 import workload
from test_gpu_parity import TOL, run_layer

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def golden_dense():
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "golden_dense.npz"), allow_pickle=False))


@pytest.fixture(scope="module")
def dense_host():
    return workload.build_dense_layer()


def digests(a, T):
    rows = a.reshape(T, -1)
    return np.array([np.frombuffer(hashlib.sha256(np.ascontiguousarray(rows[t]).tobytes()).digest()[:8], np.uint64)[0]
                     for t in range(T)], np.uint64)


def test_dense_mlp_vs_reference(golden_dense, dense_host):
    g, h = golden_dense, dense_host
    nff = h.n_ff
    assert sha(h.hot_gu[0][:nff]) == str(g["sha_gate"]) and sha(h.hot_gu[0][nff:]) == str(g["sha_up"])
    assert sha(h.hot_down[0]) == str(g["sha_down"]), "quantised weights differ from the reference quantiser"
    x = workload.make_dense_input(64)
    out, aux, layer = run_layer(h, x, aux_names=("ids", "weights", "gate_up"))
    assert layer.prefill_path(64) and layer.prefill_path(1)
    assert (aux["ids"] == 0).all() and (aux["weights"] == 1.0).all()
    dg = digests(aux["gate_up"], 64)
    bad = np.nonzero(dg != g["gate_up_digest"])[0]
    assert bad.size == 0, f"{bad.size} tokens' gate_up differ from the reference, first {bad[:8].tolist()}"
    rows = g["out_rows"]
    err = np.abs(out[rows].astype(np.float64) - g["out"]).max() / float(g["out_rms"])
    same = int((digests(out, 64) == g["out_digest"]).sum())
    print(f"dense MLP T=64: gate_up bit-equal on all tokens; outputs max-abs / rms {err:.2e}, "
          f"{same} of 64 output rows bit-equal to the reference")
    assert err <= TOL


def test_dense_mlp_batch_independent(dense_host):
    """The same tokens in batches of 1, 6 and 64 give the same output bits."""
    x = workload.make_dense_input(64)
    full, _, _ = run_layer(dense_host, x, aux_names=())
    for T in (1, 6):
        part, _, _ = run_layer(dense_host, np.ascontiguousarray(x[:T]), aux_names=())
        assert np.array_equal(part.view(np.uint32), full[:T].view(np.uint32)), T
