"""The Gemma-4 MoE block (moeb_layer_forward_gemma4: pre-norm and router-input norm fused into the
layer's first kernels, output norm into its combine) against the reference fixtures and the oracle
port, on every path (decode fused kernel, prefill tcgen05, prefill mid-size); run on a B200 with
-m gpu."""
import numpy as np
import pytest

from conftest import assert_layer_close, host_layer, near_tie_tokens, spec_of
from llapis_b200 import workload
from test_gpu_parity import TOL, run_layer
from test_gpu_prefill import gemm, prefill_from, q80_flips  # noqa: F401  (fixtures)

pytestmark = pytest.mark.gpu

AUX = ("logits", "ids", "weights", "gate_up", "down", "counts", "perm")


def norms_of(name):
    return workload.block_norms(workload.CONFIGS[name])


def select(path, prefill_from, gemm):
    prefill_from(1 << 30 if path == "decode" else 1)
    gemm("mid" if path == "mid" else "tcgen05")


@pytest.mark.parametrize("path", ["decode", "tcgen05", "mid"])
def test_block_mini_vs_reference_fixture(golden_block, prefill_from, gemm, path):
    """16 tokens of the mini block: routing exact, logits to f32 summation order, gate_up / down /
    output to the parity bar of the reference's own graph."""
    select(path, prefill_from, gemm)
    name = "mini_mixed"
    host = host_layer(name)
    x = golden_block[f"{name}_x"]
    out, aux, layer = run_layer(host, x, aux_names=AUX, norms=norms_of(name))
    assert layer.prefill_path(x.shape[0]) == (path != "decode")
    assert layer.mid_path(x.shape[0], 1) == (path == "mid")
    ties = set(near_tie_tokens(golden_block[f"{name}_logits"], host.top_k).tolist())
    same = [t for t in range(x.shape[0]) if t not in ties]
    assert np.array_equal(aux["ids"][same], golden_block[f"{name}_ids"][same])
    np.testing.assert_allclose(aux["logits"], golden_block[f"{name}_logits"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(aux["weights"], golden_block[f"{name}_weights"], rtol=1e-5, atol=1e-7)
    if not ties:
        assert_layer_close(aux["gate_up"], golden_block[f"{name}_gate_up"], tol=1e-5)
        assert_layer_close(aux["down"], golden_block[f"{name}_down"], tol=TOL)
    assert_layer_close(out, golden_block[f"{name}_out"], tol=TOL)


def test_block_decode_t4_vs_reference_fixture(golden_block):
    """The benchmark shape (d 2816, 128 experts, top-8) through the decode kernel with the norms."""
    name = "decode_t4_mixed"
    host = host_layer(name)
    x = golden_block[f"{name}_x"]
    out, aux, layer = run_layer(host, x, aux_names=("logits", "ids"), norms=norms_of(name))
    assert not layer.prefill_path(x.shape[0])
    ties = set(near_tie_tokens(golden_block[f"{name}_logits"], host.top_k).tolist())
    same = [t for t in range(x.shape[0]) if t not in ties]
    assert np.array_equal(aux["ids"][same], golden_block[f"{name}_ids"][same])
    np.testing.assert_allclose(aux["logits"], golden_block[f"{name}_logits"], rtol=1e-5, atol=2e-6)
    assert_layer_close(out[same], golden_block[f"{name}_out"][same], tol=TOL)


def check_block_stages(port, host, norms, x, out, aux, tokens):
    """As test_gpu_prefill.check_stages, through the block: routing of the router input exact off
    near ties, gate_up of the expert input within 1e-5, the rest conditioned on our ids and gate_up
    within 5e-5, and end to end within 2e-3 x RMS excluding Q8_0-flip tokens."""
    T, k = x.shape[0], host.top_k
    tok = np.asarray(tokens)
    pr = (tok[:, None] * k + np.arange(k)[None, :]).reshape(-1)
    xs = np.ascontiguousarray(x[tok])
    want = port.gemma4_block(spec_of(host, xs), norms, want=("logits", "ids", "gate_up", "act"))
    ties = set(near_tie_tokens(want["logits"], k).tolist())
    same = [i for i in range(len(tok)) if i not in ties]
    assert np.array_equal(aux["ids"][tok][same], want["ids"][same])
    rows = np.array([i * k + j for i in same for j in range(k)], dtype=np.int64)
    assert_layer_close(aux["gate_up"][pr][rows], want["gate_up"][rows], tol=1e-5)
    spec = spec_of(host, xs)
    spec.ids_in, spec.gate_up_in = aux["ids"][tok], aux["gate_up"][pr]
    cond = port.gemma4_block(spec, norms, want=("act", "down"))
    assert_layer_close(aux["down"][pr], cond["down"], tol=5e-5)
    assert_layer_close(out[tok], cond["out"], tol=5e-5)
    flips = {same[i // k] for i in q80_flips(port, want["act"][rows], cond["act"][rows])}
    keep = [i for i in same if i not in flips]
    return assert_layer_close(out[tok][keep], want["out"][keep], tol=TOL), len(ties), len(flips)


@pytest.mark.parametrize("path", ["decode", "tcgen05", "mid"])
@pytest.mark.parametrize("name,T", [("decode_t4_mixed", 96), ("prefill_t2048_q4k", 160)])
def test_block_paths_vs_port_oracle(port, prefill_from, gemm, path, name, T):
    """Real shapes, T over several decode chunks / several prefill tiles: every path with the norms
    against the oracle's block, stage by stage (every 2nd token)."""
    select(path, prefill_from, gemm)
    host = host_layer(name)
    norms = norms_of(name)
    x = workload.make_block_input(workload.CONFIGS[name], n_tokens=T, stream=T + 5)
    out, aux, layer = run_layer(host, x, aux_names=AUX, norms=norms)
    assert layer.prefill_path(T) == (path != "decode")
    rel, nt, nf = check_block_stages(port, host, norms, x, out, aux, tokens=np.arange(0, T, 2))
    print(f"block {path} {name} T={T}: max-abs / rms = {rel:.2e}; near-tie tokens {nt}, Q8_0-flip tokens {nf}")


def test_block_norm_invariance(prefill_from):
    """With eps = 0 the block is exactly invariant to scaling a token's input by a power of two (the
    squares' sum scales by 64 exactly, the square root by 8, so every normed value is the same
    float): outputs bit-equal for x and 8x, on the decode and prefill paths."""
    name = "mini_mixed"
    host = host_layer(name)
    norms = norms_of(name)
    norms.eps = 0.0
    x = workload.make_block_input(workload.CONFIGS[name], n_tokens=70, stream=3)
    for thr in (1 << 30, 1):
        prefill_from(thr)
        a, _, _ = run_layer(host, x, aux_names=(), norms=norms)
        b, _, _ = run_layer(host, (x * np.float32(8.0)).astype(np.float32), aux_names=(), norms=norms)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_rms_norm_entry_vs_reference_fixture(golden_block):
    """moeb_rms_norm (the norms the expert-parallel block applies around its exchange) against the
    reference's rms_norm / scale / mul nodes: zero row and 1e-3 .. 1e3 magnitudes, bit for bit (the
    double sum of the squares can differ from the reference's order only across an f32 rounding
    boundary of the mean, which these rows do not meet)."""
    import torch

    from llapis_b200 import capi
    from llapis_b200.workload import NORM_EPS
    x = torch.from_numpy(golden_block["rms_x"]).cuda()
    w = torch.from_numpy(golden_block["rms_w"]).cuda()
    c = float(golden_block["rms_c"])
    s = torch.cuda.current_stream().cuda_stream
    for wt, scale, key in ((None, 1.0, "rms_plain"), (w, 1.0, "rms_weight"), (w, c, "rms_router")):
        out = torch.empty_like(x)
        capi.check(capi.lib().moeb_rms_norm(x.data_ptr(), x.shape[0], x.shape[1], None if wt is None else wt.data_ptr(),
                                            scale, NORM_EPS, out.data_ptr(), s))
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy().view(np.uint32), golden_block[key].view(np.uint32)), key
