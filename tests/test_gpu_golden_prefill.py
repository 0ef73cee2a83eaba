"""The prefill workloads at full size against the REFERENCE's own outputs (tests/golden/make_golden.py
--prefill, from oracle/_ref): T=2048 all-Q4_K and the stack layer at T=256 (mixed Q4_K / IQ2_S,
Zipf-skewed routing) through the prefill path on a B200 (-m gpu). gate_up is compared on every
token as per-token digests of its f32 bits (the kernels reproduce the reference's float order),
routing on every token, outputs on a sample of tokens against the parity bar."""
import hashlib
import os

import numpy as np
import pytest

from conftest import ROOT, host_layer, near_tie_tokens, sha
from llapis_b200 import workload
from test_gpu_parity import TOL, run_layer
from test_gpu_prefill import prefill_from  # noqa: F401  (fixture)

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def golden_prefill():
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "golden_prefill.npz"), allow_pickle=False))


def digests(a, T):
    rows = a.reshape(T, -1)
    return np.array([np.frombuffer(hashlib.sha256(np.ascontiguousarray(rows[t]).tobytes()).digest()[:8], np.uint64)[0]
                     for t in range(T)], np.uint64)


@pytest.mark.parametrize("name", ["prefill_t2048_q4k", "stack30_t256_mixed"])
def test_prefill_layer_vs_reference(golden_prefill, prefill_from, name):
    prefill_from(1)
    host = host_layer(name)
    g = golden_prefill
    for n in ("hot_gu", "hot_down", "cold_gu", "cold_down"):
        got = sha(getattr(host, n)) if getattr(host, n) is not None else ""
        assert got == str(g[f"{name}_sha_{n}"]), f"quantised {n} differs from the reference quantiser"
    x = workload.make_input(workload.CONFIGS[name])
    T = x.shape[0]
    out, aux, layer = run_layer(host, x, aux_names=("logits", "ids", "gate_up"))
    assert layer.prefill_path(T) and layer.device_error() == 0
    ties = set(near_tie_tokens(aux["logits"], host.top_k, rel=1e-5).tolist())
    same = np.array([t for t in range(T) if t not in ties])
    assert np.array_equal(aux["ids"][same], g[f"{name}_ids"][same])
    # gate_up of every token (off near ties) is the reference's, bit for bit
    dg = digests(aux["gate_up"], T)
    bad = [int(t) for t in same if dg[t] != g[f"{name}_gate_up_digest"][t]]
    assert not bad, f"{len(bad)} tokens' gate_up differ from the reference, first {bad[:8]}"
    rows = g[f"{name}_out_rows"]
    keep = np.array([i for i, t in enumerate(rows) if t not in ties])
    err = np.abs(out[rows[keep]].astype(np.float64) - g[f"{name}_out"][keep]).max() / float(g[f"{name}_out_rms"])
    print(f"{name}: {len(same)} of {T} tokens off near ties, gate_up bit-equal on all; sampled outputs max-abs / rms {err:.2e}")
    assert err <= TOL
