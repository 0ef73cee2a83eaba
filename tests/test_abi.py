"""The C-ABI library without a GPU: it loads, exports every symbol the public headers declare (and
capi.py binds exactly those), its moert structs have the reference's layout, and argument
validation and the host-side helpers work on a CPU-only machine."""
import ctypes as C
import json
import os
import re
import sys

import numpy as np
import pytest

from conftest import ROOT

sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
import abi_layout  # noqa: E402

HEADERS = [os.path.join(ROOT, "include", h) for h in ("moeb200.h", "moert_cuda.h", "moert_store.h")]


def declared_functions():
    names = set()
    for h in HEADERS:
        src = re.sub(r"/\*.*?\*/", "", open(h).read(), flags=re.S)
        src = re.sub(r"#define[^\n]*", "", src)
        for m in re.finditer(r"\b((?:moeb|moert)_\w+)\s*\(", src):
            # declarations only: skip the names of function-pointer typedefs, `(*name)(`
            if re.search(r"\(\s*\*\s*$", src[max(0, m.start() - 8):m.start()]):
                continue
            names.add(m.group(1))
    # inline helpers defined in the header, not exported
    return {n for n in names if n != "moert_cuda_config_defaults"}


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_capi_binds_exactly_the_declared_symbols():
    from llapis_b200 import capi
    assert set(capi.SIGNATURES) == declared_functions()


def test_moert_struct_layouts_match_reference():
    want = json.load(open(os.path.join(ROOT, "tests", "golden", "moert_abi_layout.json")))
    assert abi_layout.ours() == want


def test_python_struct_mirrors_match_c(lib):
    from llapis_b200 import capi
    # moeb_pool: 4 x i32 + 3 pointers; moeb_layer: 4 x i32, 2 pointers, 2 pools, 3 pointers
    assert C.sizeof(capi.Pool) == 16 + 3 * 8
    assert C.sizeof(capi.Layer) == 16 + 2 * 8 + 2 * C.sizeof(capi.Pool) + 3 * 8
    assert C.sizeof(capi.LayerAux) == 8 * 8
    # moeb_norms: 3 pointers, f32 eps, i32 pad
    assert C.sizeof(capi.Norms) == 3 * 8 + 8 and capi.Norms.eps.offset == 24


def test_row_sizes(lib):
    from llapis_b200 import capi
    assert capi.row_size(capi.Q4_K, 2816) == 11 * 144
    assert capi.row_size(capi.IQ2_S, 2816) == 11 * 82
    assert capi.row_size(capi.Q5_0, 704) == 22 * 22
    assert capi.row_size(capi.IQ4_NL, 704) == 22 * 18


def test_argument_validation_without_device(lib):
    from llapis_b200 import capi
    assert lib.moeb_layer_forward(None, None, 1, None, None, None, 0, None) == -1      # null layer
    L = capi.Layer()
    L.d_model, L.n_ff, L.n_expert, L.top_k = 100, 64, 32, 4                              # d % 256 != 0
    assert lib.moeb_layer_forward(C.byref(L), None, 1, None, None, None, 0, None) == -1
    assert "d_model" in lib.moeb_last_error().decode()
    assert lib.moeb_router_topk(None, 1, 32, 4, None, None, None) == -1
    assert lib.moeb_layer_workspace_size(None, 8) == 0
    prev = lib.moeb_set_prefill_min_tokens(0)
    assert prev > 0 and lib.moeb_set_prefill_min_tokens(0) == prev


def test_no_device_means_enodev(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert lib.moeb_init() == -2


def test_workspace_sizes_by_path(lib):
    """Decode workspace is one 8-token chunk for any T; the prefill workspace grows with T."""
    from llapis_b200 import capi
    L = capi.Layer()
    L.d_model, L.n_ff, L.n_expert, L.top_k = 2816, 704, 128, 8
    prev = lib.moeb_set_prefill_min_tokens(1 << 30)
    try:
        a, b = lib.moeb_layer_workspace_size(C.byref(L), 8), lib.moeb_layer_workspace_size(C.byref(L), 4096)
        assert a == b and 2_000_000 < a < 2_400_000
        lib.moeb_set_prefill_min_tokens(64)
        p = lib.moeb_layer_workspace_size(C.byref(L), 2048)
        assert p > 2048 * 8 * 2816 * 4          # the f32 down outputs of every pair
        assert lib.moeb_layer_workspace_size(C.byref(L), 32) == a   # below the threshold: decode
    finally:
        lib.moeb_set_prefill_min_tokens(prev)


def test_host_quantiser_matches_reference_quantiser(ref):
    """The library's weight quantiser (moeb_quantize_weights) is byte-identical to
    ggml_quantize_chunk of the reference build, for every type the pools use."""
    from llapis_b200 import capi
    rng = np.random.default_rng(3)
    for t, n in ((capi.Q4_K, 512), (capi.IQ2_S, 512), (capi.Q5_0, 128), (capi.IQ4_NL, 128)):
        w = (rng.standard_normal((4, n)) * 0.02).astype(np.float32)
        rs = capi.row_size(t, n)
        ours = np.zeros(4 * rs, np.uint8)
        got = capi.lib().moeb_quantize_weights(t, w.ctypes.data, ours.ctypes.data, 4, n, 1)
        assert got == 4 * rs
        assert np.array_equal(ours, ref.quantize(t, w).reshape(-1)), t


def test_host_iq2xxs_quantiser_matches_reference(ref):
    """IQ2_XXS through moeb_quantize_weights equals ggml_quantize_chunk given a uniform importance
    matrix (the reference quantises this type only with one), byte for byte: ordinary rows, a zero
    row, tiny values, a dominant value, sign patterns of odd parity and the workload's scale."""
    from llapis_b200 import capi
    rng = np.random.default_rng(17)
    n = 1024
    w = (rng.standard_normal((12, n)) * 0.02).astype(np.float32)
    w[1] = 0.0
    w[2] *= 1e-6
    w[3, 100] = 3.0
    w[4, :8] = [-1, 2, 3, 4, 5, 6, 7, 8]
    w[5] = np.abs(w[5])
    w[6] = -np.abs(w[6])
    rs = capi.row_size(capi.IQ2_XXS, n)
    assert rs == n // 256 * 66
    ours = np.zeros(12 * rs, np.uint8)
    assert capi.lib().moeb_quantize_weights(capi.IQ2_XXS, w.ctypes.data, ours.ctypes.data, 12, n, 3) == 12 * rs
    want = ref.quantize(16, w).reshape(-1)
    bad = [r for r in range(12) if not np.array_equal(ours[r * rs:(r + 1) * rs], want[r * rs:(r + 1) * rs])]
    assert not bad, f"rows {bad} differ"


def test_host_q8_0_weight_quantiser_matches_reference(ref):
    """Q8_0 weights through moeb_quantize_weights equal ggml_quantize_chunk (quantize_row_q8_0_ref:
    round half away from zero), including a zero block and exact .5 ties."""
    from llapis_b200 import capi
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((5, 128)) * 0.02).astype(np.float32)
    w[1, :32] = 0.0
    w[2, :32] = np.arange(32, dtype=np.float32) - 15.5      # amax 16.5 ... ties after scaling
    w[3, :4] = [127.0, 0.5, -0.5, 1.5]
    rs = capi.row_size(capi.Q8_0, 128)
    ours = np.zeros(5 * rs, np.uint8)
    assert capi.lib().moeb_quantize_weights(capi.Q8_0, w.ctypes.data, ours.ctypes.data, 5, 128, 1) == 5 * rs
    assert np.array_equal(ours, ref.quantize(capi.Q8_0, w).reshape(-1))


def test_layer_path_and_new_entries_validate_without_device(lib):
    """moeb_layer_path picks the prefill kernels for every batch size of a layer whose decode kernel
    does not fit (the dense MLP's 2112-wide inner dimension) and refuses bad layers; the block,
    rms_norm and Q8_K routed entries reject bad arguments before any device work."""
    from llapis_b200 import capi, workload
    dense = workload.build_dense_layer()
    L = capi.Layer()
    L.d_model, L.n_ff, L.n_expert, L.top_k = dense.d_model, dense.n_ff, dense.n_expert, dense.top_k
    dummy = C.c_void_p(256)   # never dereferenced: the path query reads only the shape and pointers' presence
    L.w_router = dummy
    L.hot = capi.Pool(capi.Q4_K, capi.Q5_0, 1, 0, dummy, dummy, None)
    L.exp_slot = L.slot_exp = L.slot_state = dummy
    assert lib.moeb_layer_path(C.byref(L), 1) == 1 and lib.moeb_layer_path(C.byref(L), 4096) == 1
    M = capi.Layer.from_buffer_copy(L)
    M.n_ff = 704
    prev = lib.moeb_set_prefill_min_tokens(0)
    assert lib.moeb_layer_path(C.byref(M), 1) == 0 and lib.moeb_layer_path(C.byref(M), max(prev, 1)) == 1
    M.n_ff = 8192                          # neither kernel family covers it
    assert lib.moeb_layer_path(C.byref(M), 1) == -1
    assert lib.moeb_layer_path(None, 1) == -1
    # the feed-forward block: shapes must agree and the dense MLP must be a one-expert layer
    B = capi.Layer.from_buffer_copy(L)
    B.d_model = 512
    ws = C.c_void_p(4096)
    assert lib.moeb_ffn_block_gemma4(C.byref(L), None, C.byref(B), None, None, 4, None, ws, 1 << 30, None, None) == -1
    assert "d_model" in lib.moeb_last_error().decode()
    assert lib.moeb_ffn_block_gemma4(C.byref(L), None, C.byref(L), None, None, 4, None, None, 0, None, None) == -1
    assert "workspace" in lib.moeb_last_error().decode()
    E = capi.Layer.from_buffer_copy(L)
    E.top_k = 2
    assert lib.moeb_ffn_block_gemma4(C.byref(L), None, C.byref(E), None, None, 4, None, ws, 1 << 30, None, None) == -1
    assert "one-expert" in lib.moeb_last_error().decode()
    assert lib.moeb_ffn_block_workspace_size(C.byref(L), C.byref(L), 64) > 64 * 2816 * 4
    # rms_norm: row width a multiple of 4, aligned pointers, eps >= 0
    assert lib.moeb_rms_norm(None, 2, 6, None, 1.0, 1e-6, None, None) == -1
    assert lib.moeb_rms_norm(C.c_void_p(17), 2, 8, None, 1.0, 1e-6, C.c_void_p(32), None) == -1
    assert lib.moeb_rms_norm(C.c_void_p(16), 2, 8, None, 1.0, -1.0, C.c_void_p(32), None) == -1
    assert lib.moeb_rms_norm(None, 0, 8, None, 1.0, 1e-6, None, None) == 0      # nothing to do
    # Q8_K routed half: null rows refused
    assert lib.moeb_layer_forward_routed_q8k(C.byref(L), None, 4, None, None, None, None, 0, None) == -1
