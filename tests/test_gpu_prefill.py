"""Parity of the prefill path (tcgen05 grouped GEMMs) against the oracle, the reference fixtures and
the decode path; run on a B200 with -m gpu."""
import numpy as np
import pytest
import torch

from conftest import assert_layer_close, host_layer, near_tie_tokens, spec_of
from llapis_b200 import capi, workload
from test_gpu_parity import TOL, run_layer

pytestmark = pytest.mark.gpu


@pytest.fixture
def prefill_from():
    """Sets the prefill threshold for one test and restores it afterwards."""
    lib = capi.lib()
    prev = lib.moeb_set_prefill_min_tokens(0)
    yield lambda n: lib.moeb_set_prefill_min_tokens(n)
    lib.moeb_set_prefill_min_tokens(prev)


@pytest.fixture
def gemm():
    """Selects the prefill path's down GEMM for one test ("mid" / "mid_down": int8 MMAs on the weight
    codes; "tcgen05": the converted-operand tensor-core GEMM) and restores the thresholds
    afterwards. gate_up always runs the lane-exact tcgen05 kernel."""
    lib = capi.lib()
    prev = lib.moeb_set_mid_max_pairs(0), lib.moeb_set_mid_max_pairs_down(0)

    def select(kind):
        lib.moeb_set_mid_max_pairs(1)
        lib.moeb_set_mid_max_pairs_down(1 << 30 if kind in ("mid", "mid_down") else 1)
    yield select
    lib.moeb_set_mid_max_pairs(prev[0])
    lib.moeb_set_mid_max_pairs_down(prev[1])


@pytest.mark.parametrize("kind", ["tcgen05", "mid"])
def test_prefill_mini_vs_reference_fixture(golden, prefill_from, gemm, kind):
    prefill_from(1)
    gemm(kind)
    host = host_layer("mini_mixed")
    out, aux, layer = run_layer(host, golden["mini_x"])
    # router, top-k, dispatch, activation quantisation, gate_up (gather, min term, GEMM), down (GeGLU
    # images + GEMM on either path), combine
    assert layer.launches(golden["mini_x"].shape[0]) == 10
    assert layer.mid_path(golden["mini_x"].shape[0], 1) == (kind == "mid")
    assert np.array_equal(aux["ids"], golden["mini_ids"])
    np.testing.assert_allclose(aux["logits"], golden["mini_logits"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(aux["weights"], golden["mini_weights"], rtol=1e-5, atol=1e-7)
    flat = golden["mini_ids"].reshape(-1)
    counts = np.bincount(flat, minlength=host.n_expert)
    assert np.array_equal(aux["counts"], counts)
    assert np.array_equal(aux["offsets"], np.concatenate([[0], np.cumsum(counts)]))
    assert np.array_equal(aux["perm"], np.argsort(flat, kind="stable"))
    # gate_up is the reference's own bits (its x86 8-lane float order, reproduced on tcgen05)
    assert np.array_equal(aux["gate_up"].view(np.uint32), golden["mini_gate_up"].view(np.uint32))
    assert_layer_close(aux["down"], golden["mini_down"], tol=1e-5)
    assert_layer_close(out, golden["mini_out"], tol=1e-5)


def host_layer_mid(host, T):
    lib = capi.lib()
    return any(m > 1 and T * host.top_k < m * host.n_expert
               for m in (int(lib.moeb_set_mid_max_pairs(0)), int(lib.moeb_set_mid_max_pairs_down(0))))


def q80_flips(port, want_act, cond_act):
    """Indices of the pairs whose down input (the GeGLU output quantised to Q8_0) differs between
    the oracle's own gate_up and ours: a last-bit difference upstream that moved a value across
    a Q8_0 rounding boundary (or a fp16 GELU-table boundary)."""
    from oracle.oracle import Q8_0
    return [int(i) for i in np.nonzero(np.any(want_act != cond_act, axis=1))[0]
            if not np.array_equal(port.quantize_act(Q8_0, want_act[i]), port.quantize_act(Q8_0, cond_act[i]))]


def check_stages(port, host, x, out, aux, tokens=None, dispatch=True, exact=True):
    """Stage by stage against the oracle port (whose dots are the reference's bit for bit), on
    `tokens` (default all) of a forward of x:
      1. routing (ids, counts, stable permutation over the whole batch) exact for tokens without
         a near tie;
      2. gate_up: with `exact`, equal to the oracle's bit for bit (the lane-exact kernels reproduce
         the reference's float order); otherwise within 1e-5;
      3. GeGLU -> Q8_0 -> down -> scale -> combine, fed with OUR ids and gate_up, within 5e-5 of
         the oracle fed the same (every later stage is exact given its input up to float
         summation order);
      4. end to end within 2e-3 x RMS on every token off near ties; without `exact`, the tokens
         where a last-bit gate_up difference flipped a Q8_0 rounding of the down input are left
         out and counted.
    Returns (end-to-end max-abs / rms, near-tie tokens, flip tokens)."""
    T, k = x.shape[0], host.top_k
    if dispatch:   # the whole batch's dispatch (the decode path reports it for one-chunk calls only)
        flat = aux["ids"].reshape(-1)
        assert np.array_equal(aux["counts"], np.bincount(flat, minlength=host.n_expert))
        assert np.array_equal(aux["perm"], np.argsort(flat, kind="stable"))
    tok = np.arange(T) if tokens is None else np.asarray(tokens)
    pr = (tok[:, None] * k + np.arange(k)[None, :]).reshape(-1)
    xs = np.ascontiguousarray(x[tok])
    want = port.moe_layer(spec_of(host, xs), want=("logits", "ids", "gate_up", "act"))
    ties = set(near_tie_tokens(want["logits"], k).tolist())
    same = [i for i in range(len(tok)) if i not in ties]
    assert np.array_equal(aux["ids"][tok][same], want["ids"][same])
    rows = np.array([i * k + j for i in same for j in range(k)], dtype=np.int64)
    if exact:
        got_gu = aux["gate_up"][pr][rows]
        bad = np.argwhere(got_gu.view(np.uint32) != want["gate_up"][rows].view(np.uint32))
        assert bad.size == 0, f"{len(bad)} gate_up values differ from the reference order, first (pair, row) {bad[:4].tolist()}"
    else:
        assert_layer_close(aux["gate_up"][pr][rows], want["gate_up"][rows], tol=1e-5)
    spec = spec_of(host, xs)
    spec.ids_in, spec.gate_up_in = aux["ids"][tok], aux["gate_up"][pr]
    cond = port.moe_layer(spec, want=("act", "down"))
    assert_layer_close(aux["down"][pr], cond["down"], tol=5e-5)
    assert_layer_close(out[tok], cond["out"], tol=5e-5)
    flips = set() if exact else {same[i // k] for i in q80_flips(port, want["act"][rows], cond["act"][rows])}
    keep = [i for i in same if i not in flips]
    rel = assert_layer_close(out[tok][keep], want["out"][keep], tol=TOL)
    return rel, len(ties), len(flips)


@pytest.mark.parametrize("path", ["tcgen05", "mid", "decode"])
@pytest.mark.parametrize("name,T", [("mini_mixed", 64), ("mini_mixed", 1100), ("decode_t4_mixed", 96),
                                    ("prefill_t2048_q4k", 160), ("stack30_t256_mixed", 256), ("decode_t4_iq2xxs", 96)])
def test_layer_paths_vs_port_oracle(port, prefill_from, gemm, path, name, T):
    """Every path, stage by stage (check_stages). mini_mixed at T=1100 puts more than 128 pairs on
    most experts (several tiles per expert); decode_t4_mixed and the stack layer mix Q4_K/Q5_0 and
    IQ2_S/IQ4_NL tiles at the real shapes; decode_t4_iq2xxs has the product files' cold class
    (IQ2_XXS gate_up, IQ4_NL down). On the prefill path gate_up is always the lane-exact tcgen05
    kernel; "mid" runs the down projection on the mid-size kernel."""
    if path == "decode" and T > 160:
        pytest.skip("the decode path's share of this batch adds nothing over T=160")
    prefill_from(1 << 30 if path == "decode" else 1)
    gemm("mid_down" if path == "mid" else "tcgen05")
    host = host_layer(name)
    x = workload.make_input(workload.CONFIGS[name], n_tokens=T, stream=T + 1)
    out, aux, layer = run_layer(host, x, aux_names=("logits", "ids", "gate_up", "down", "counts", "perm"))
    assert layer.prefill_path(T) == (path != "decode")
    assert not layer.mid_path(T, 0) and layer.mid_path(T, 1) == (path == "mid")
    tokens = np.arange(0, T, 4) if T >= 256 else None
    rel, nt, nf = check_stages(port, host, x, out, aux, tokens=tokens, dispatch=path != "decode" or T <= 8,
                               exact=path != "decode")
    print(f"{path} {name} T={T}: max-abs / rms = {rel:.2e}; near-tie tokens {nt}, Q8_0-flip tokens {nf}")


@pytest.mark.parametrize("name,T", [("prefill_t2048_q4k", 160), ("stack30_t256_mixed", 256)])
def test_mid_down_after_exact_gate_up(port, prefill_from, gemm, name, T):
    """gate_up on the lane-exact tcgen05 kernel, down on the mid-size kernel: the two hand over the
    gate_up rows in the same slot-order buffer (and share the operand-image buffer in turn)."""
    prefill_from(1)
    gemm("mid_down")
    host = host_layer(name)
    x = workload.make_input(workload.CONFIGS[name], n_tokens=T, stream=T + 3)
    out, aux, layer = run_layer(host, x, aux_names=("logits", "ids", "gate_up", "down", "counts", "perm"))
    assert not layer.mid_path(T, 0) and layer.mid_path(T, 1)
    rel, nt, nf = check_stages(port, host, x, out, aux, tokens=np.arange(0, T, 4))
    print(f"mid down {name} T={T}: max-abs / rms = {rel:.2e}; near-tie tokens {nt}")


def test_prefill_full_size(port, prefill_from):
    """The prefill config at its full T=2048 (about 128 pairs per expert: full 128-pair tiles and
    experts split over two tiles): the whole batch through the prefill path, stage-by-stage
    parity on every 8th token (the oracle's share of the work stays a few seconds), and routing
    against the decode path on all tokens."""
    name = "prefill_t2048_q4k"
    host = host_layer(name)
    x = workload.make_input(workload.CONFIGS[name])
    T = x.shape[0]
    prefill_from(1)
    assert not host_layer_mid(host, T), "T=2048 (128 pairs per expert) runs the tcgen05 GEMMs by default"
    out, aux, layer = run_layer(host, x, aux_names=("logits", "ids", "gate_up", "down", "counts", "offsets",
                                                    "perm"))
    assert layer.launches(T) == 10
    counts = np.bincount(aux["ids"].reshape(-1), minlength=host.n_expert)
    assert np.array_equal(aux["offsets"], np.concatenate([[0], np.cumsum(counts)]))
    assert counts.max() > 128, "the workload should put more than one tile on some expert"
    assert np.isfinite(out).all()
    rel, nt, nf = check_stages(port, host, x, out, aux, tokens=np.arange(0, T, 8))
    print(f"prefill T={T} (every 8th token vs oracle): max-abs / rms = {rel:.2e}; near-tie {nt}, flips {nf}")
    prefill_from(1 << 30)
    _, aux_d, layer = run_layer(host, x, aux_names=("logits", "ids"))
    assert not layer.prefill_path(T)
    # f32 dots of 2816 terms in two summation orders: |difference| ~ 1e-6 of logits ~ N(0, 1)
    np.testing.assert_allclose(aux["logits"], aux_d["logits"], rtol=1e-5, atol=2e-5)
    ties = set(near_tie_tokens(aux["logits"], host.top_k, rel=1e-5).tolist())
    same = [t for t in range(T) if t not in ties]
    assert np.array_equal(aux["ids"][same], aux_d["ids"][same])


@pytest.mark.parametrize("kind", ["tcgen05", "mid"])
def test_prefill_zero_and_small_batches(prefill_from, gemm, port, kind):
    """T=1 and T=2 on the prefill path (tiles of one pair: MMA N = 16 with 15 padding columns on
    the tcgen05 path, one column block with 7 absent pairs on the mid path)."""
    prefill_from(1)
    gemm(kind)
    host = host_layer("mini_mixed")
    for T in (1, 2):
        x = workload.make_input(workload.CONFIGS["mini_mixed"], n_tokens=T, stream=500 + T)
        out, _, _ = run_layer(host, x, aux_names=())
        assert_layer_close(out, port.moe_layer(spec_of(host, x))["out"], tol=TOL)
    torch.cuda.synchronize()


@pytest.mark.parametrize("path", ["decode", "tcgen05", "mid"])
def test_per_expert_down_scales_both_classes(port, prefill_from, gemm, path):
    """Non-unit per-expert down scales in BOTH precision classes (ffn_down_exps.scale of the hot
    slots and of the cold experts), on every path: applied once to each pair's down row before the
    weighted combine, as the reference's ggml_mul by the scale does."""
    import dataclasses
    prefill_from(1 << 30 if path == "decode" else 1)
    gemm("mid" if path == "mid" else "tcgen05")
    base = host_layer("mini_mixed")
    rng = np.random.default_rng(31)
    h = dataclasses.replace(base, s_hot=rng.uniform(0.5, 2.0, base.n_slots).astype(np.float32),
                            s_cold=rng.uniform(0.5, 2.0, base.n_expert).astype(np.float32))
    x = workload.make_input(workload.CONFIGS["mini_mixed"], n_tokens=96, stream=41)
    out, aux, layer = run_layer(h, x, aux_names=("ids", "gate_up"))
    assert layer.prefill_path(96) == (path != "decode")
    want = port.moe_layer(spec_of(h, x), n_threads=8, want=("ids", "gate_up"))
    same = np.all(aux["ids"] == want["ids"], axis=1)
    assert same.mean() > 0.95
    k = h.top_k
    pairs = (np.nonzero(same)[0][:, None] * k + np.arange(k)[None, :]).reshape(-1)
    assert np.array_equal(aux["gate_up"][pairs].view(np.uint32), want["gate_up"][pairs].view(np.uint32))
    cold_routed = ~np.isin(aux["ids"], h.hot_ids)
    assert cold_routed.any() and (~cold_routed).any(), "both classes must be routed"
    rel = assert_layer_close(out[same], want["out"][same], tol=TOL)
    print(f"{path}: down scales in both classes, max-abs / rms {rel:.2e}")
