"""GPU parity: the sm_100a path through the C-ABI against the oracle (and the reference fixtures).

Bars: routing indices, dispatch and dequantised weights / quantised activations bit-exact; layer
outputs max-abs <= 2e-3 x output RMS (the tolerance is written at each call site)."""
import ctypes as C

import numpy as np
import pytest
import torch

from conftest import assert_layer_close, host_layer, near_tie_tokens, spec_of
from llapis_b200 import capi
from llapis_b200.layer import HostLayer, MoELayer
from oracle.oracle import IQ2_S, IQ4_NL, Q4_K, Q5_0, Q8_0, Q8_K

pytestmark = pytest.mark.gpu
TOL = 2e-3   # max-abs / RMS of the reference output


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.fixture(scope="module", autouse=True)
def _init():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    capi.check(capi.lib().moeb_init())
    yield
    torch.cuda.synchronize()
    assert capi.lib().moeb_device_error(stream()) == 0, "a kernel reported a device error"


@pytest.mark.parametrize("t,n", [(Q4_K, 512), (IQ2_S, 512), (Q5_0, 64), (IQ4_NL, 64)])
def test_dequant_bit_exact(golden, t, n):
    src, want = golden[f"deq_{t}_src"], golden[f"deq_{t}_f32"]
    out = torch.empty(want.shape, dtype=torch.float32, device="cuda")
    capi.check(capi.lib().moeb_dequantize(t, dev(src).data_ptr(), out.data_ptr(), src.shape[0], n, stream()))
    got = out.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("t,n", [(16, 512), (8, 64)])
def test_dequant_iq2xxs_q8_0_bit_exact(t, n):
    """IQ2_XXS and Q8_0 expert weights (the other types the product files use) dequantise bit for
    bit as the reference's dequantize_row_iq2_xxs / _q8_0 (rows from tests/golden/golden_types.npz)."""
    import os
    from conftest import ROOT
    g = np.load(os.path.join(ROOT, "tests", "golden", "golden_types.npz"))
    src, want = g[f"deq_{t}_src"], g[f"deq_{t}_f32"]
    out = torch.empty(want.shape, dtype=torch.float32, device="cuda")
    capi.check(capi.lib().moeb_dequantize(t, dev(src).data_ptr(), out.data_ptr(), src.shape[0], n, stream()))
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert capi.lib().moeb_row_size(t, n) == src.shape[1]


@pytest.mark.parametrize("wt,vdt", [(Q4_K, Q8_K), (Q5_0, Q8_0)])
def test_activation_quant_bit_exact(golden, wt, vdt):
    x, want = golden[f"act_{vdt}_x"], golden[f"act_{vdt}_q"]
    out = torch.zeros(want.shape, dtype=torch.uint8, device="cuda")
    capi.check(capi.lib().moeb_quantize_act(wt, dev(x).data_ptr(), out.data_ptr(), x.shape[0], x.shape[1], stream()))
    assert np.array_equal(out.cpu().numpy(), want)


def test_dequant_real_expert_matches_oracle(port):
    host = host_layer("decode_t4_mixed")
    for pool, t, n in ((host.cold_gu[100], IQ2_S, 2816), (host.cold_down[100], IQ4_NL, 704),
                       (host.hot_gu[3], Q4_K, 2816), (host.hot_down[3], Q5_0, 704)):
        rows = pool.shape[0]
        out = torch.empty((rows, n), dtype=torch.float32, device="cuda")
        capi.check(capi.lib().moeb_dequantize(t, dev(pool).data_ptr(), out.data_ptr(), rows, n, stream()))
        got = out.cpu().numpy()
        for r in (0, 1, rows // 2, rows - 1):
            assert np.array_equal(got[r].view(np.uint32), port.dequantize(t, pool[r], n).view(np.uint32))


def test_router_topk_indices_bit_exact(golden):
    """The reference's own logits through the GPU top-k: same experts, same order."""
    for name in ("mini", "decode_t1_iq2s", "decode_t4_mixed"):
        logits = golden[f"{name}_logits"]
        k = golden[f"{name}_ids"].shape[1]
        T, E = logits.shape
        ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
        w = torch.empty((T, k), dtype=torch.float32, device="cuda")
        capi.check(capi.lib().moeb_router_topk(dev(logits).data_ptr(), T, E, k, ids.data_ptr(), w.data_ptr(), stream()))
        ties = set(near_tie_tokens(logits, k).tolist())
        got = ids.cpu().numpy()
        for t in range(T):
            if t not in ties:
                assert np.array_equal(got[t], golden[f"{name}_ids"][t]), (name, t)
        np.testing.assert_allclose(w.cpu().numpy(), golden[f"{name}_weights"], rtol=2e-6, atol=1e-7)


def test_router_topk_ties_and_many_tokens(port):
    rng = np.random.default_rng(3)
    T, E, k = 37, 128, 8
    logits = rng.normal(0, 1, (T, E)).astype(np.float32)
    logits[0, [5, 9, 77, 100]] = 9.0          # exact ties: lowest index first
    logits[1, :] = 0.0                          # all equal
    ids = torch.empty((T, k), dtype=torch.int32, device="cuda")
    capi.check(capi.lib().moeb_router_topk(dev(logits).data_ptr(), T, E, k, ids.data_ptr(), None, stream()))
    got = ids.cpu().numpy()
    for t in range(T):
        assert got[t].tolist() == port.topk(logits[t], k).tolist(), t
    assert got[0, :4].tolist() == [5, 9, 77, 100]
    assert got[1].tolist() == list(range(8))


def test_dispatch_bit_exact():
    rng = np.random.default_rng(4)
    T, k, E = 16, 8, 128
    ids = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    ids[3] = ids[2]                             # repeated rows: stability matters
    cnt = torch.empty(E, dtype=torch.int32, device="cuda")
    off = torch.empty(E + 1, dtype=torch.int32, device="cuda")
    perm = torch.empty(T * k, dtype=torch.int32, device="cuda")
    capi.check(capi.lib().moeb_dispatch(dev(ids).data_ptr(), T, k, E, cnt.data_ptr(), off.data_ptr(), perm.data_ptr(),
                                        stream()))
    flat = ids.reshape(-1)
    want_cnt = np.bincount(flat, minlength=E)
    want_off = np.concatenate([[0], np.cumsum(want_cnt)])
    want_perm = np.argsort(flat, kind="stable")
    assert np.array_equal(cnt.cpu().numpy(), want_cnt)
    assert np.array_equal(off.cpu().numpy(), want_off)
    assert np.array_equal(perm.cpu().numpy(), want_perm)


def run_layer(host, x, aux_names=("logits", "ids", "weights", "counts", "offsets", "perm", "gate_up", "down"),
              norms=None):
    """One forward through the C-ABI (moeb_layer_forward, or moeb_layer_forward_gemma4 with norms)."""
    layer = MoELayer(host, norms=norms)
    T, E, k = x.shape[0], host.n_expert, host.top_k
    shapes = dict(logits=((T, E), torch.float32), ids=((T, k), torch.int32), weights=((T, k), torch.float32),
                  counts=((E,), torch.int32), offsets=((E + 1,), torch.int32), perm=((T * k,), torch.int32),
                  gate_up=((T * k, 2 * host.n_ff), torch.float32), down=((T * k, host.d_model), torch.float32))
    aux = {n: torch.empty(*shapes[n][0], dtype=shapes[n][1], device="cuda") for n in aux_names}
    out = layer(dev(x), aux=aux)
    torch.cuda.synchronize()
    # every bounded wait ended in time (a timed-out wait would leave its outputs unwritten)
    assert layer.device_error() == 0
    return out.cpu().numpy(), {n: t.cpu().numpy() for n, t in aux.items()}, layer


def test_mini_layer_vs_reference_fixture(golden, port):
    host = host_layer("mini_mixed")
    x = golden["mini_x"]
    out, aux, _ = run_layer(host, x)
    assert np.array_equal(aux["ids"], golden["mini_ids"])
    np.testing.assert_allclose(aux["logits"], golden["mini_logits"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(aux["weights"], golden["mini_weights"], rtol=1e-5, atol=1e-7)
    flat = golden["mini_ids"].reshape(-1)
    assert np.array_equal(aux["counts"], np.bincount(flat, minlength=host.n_expert))
    assert np.array_equal(aux["perm"], np.argsort(flat, kind="stable"))
    assert_layer_close(aux["gate_up"], golden["mini_gate_up"], tol=1e-5)
    assert_layer_close(aux["down"], golden["mini_down"], tol=TOL)
    assert_layer_close(out, golden["mini_out"], tol=TOL)


@pytest.mark.parametrize("name,T", [("decode_t1_iq2s", 2), ("decode_t4_mixed", 4)])
def test_real_layer_vs_reference_fixture(golden, name, T):
    host = host_layer(name)
    x = golden[f"{name}_x"]
    out, aux, _ = run_layer(host, x, aux_names=("logits", "ids", "weights"))
    ties = set(near_tie_tokens(golden[f"{name}_logits"], host.top_k).tolist())
    for t in range(T):
        if t not in ties:
            assert np.array_equal(aux["ids"][t], golden[f"{name}_ids"][t]), t
    np.testing.assert_allclose(aux["logits"], golden[f"{name}_logits"], rtol=1e-4, atol=2e-5)
    rel = assert_layer_close(out, golden[f"{name}_out"], tol=TOL)
    print(f"{name}: max-abs / rms = {rel:.2e}")


@pytest.mark.parametrize("name,T", [("decode_t1_iq2s", 1), ("decode_t4_mixed", 4), ("decode_t4_mixed", 20),
                                    ("mini_mixed", 16)])
def test_layer_vs_port_oracle(port, name, T):
    from llapis_b200 import workload
    host = host_layer(name)
    x = workload.make_input(workload.CONFIGS[name], n_tokens=T, stream=T)
    out, aux, _ = run_layer(host, x, aux_names=("logits", "ids", "gate_up"))
    want = port.moe_layer(spec_of(host, x), want=("logits", "ids", "gate_up"))
    ties = set(near_tie_tokens(want["logits"], host.top_k).tolist())
    same = [t for t in range(T) if t not in ties]
    assert np.array_equal(aux["ids"][same], want["ids"][same])
    if not ties:
        assert_layer_close(aux["gate_up"], want["gate_up"], tol=1e-5)
    assert_layer_close(out[same], want["out"][same], tol=TOL)


def test_residency_filling_slot_and_all_hot(port):
    """A FILLING slot serves its expert from the cold pool; a layer with no cold pool works."""
    import dataclasses
    from llapis_b200 import workload
    base = host_layer("mini_mixed")
    x = workload.make_input(workload.CONFIGS["mini_mixed"], n_tokens=8, stream=99)
    # slot 0 not READY -> expert hot_ids[0] must come from the cold pool, which must then hold it
    cold_gu, cold_down = base.cold_gu.copy(), base.cold_down.copy()
    e0 = int(base.hot_ids[0])
    cfg = workload.CONFIGS["mini_mixed"]
    gu, dn = workload.expert_f32(cfg, 0, e0)
    cold_gu[e0] = workload.quantize(IQ2_S, gu)
    cold_down[e0] = workload.quantize(IQ4_NL, dn)
    h = dataclasses.replace(base, cold_gu=cold_gu, cold_down=cold_down)
    layer = MoELayer(h)
    st = layer.t["slot_state"]
    st[0] = 1
    out = layer(dev(x)).cpu().numpy()
    spec = spec_of(h, x)
    spec.slot_state = st.cpu().numpy()
    want = port.moe_layer(spec)
    assert_layer_close(out, want["out"], tol=TOL)
    # every expert hot (K = E), no cold pool
    E = base.n_expert
    gus, dns = zip(*[workload.expert_f32(cfg, 0, e) for e in range(E)])
    hot = HostLayer(base.d_model, base.n_ff, E, base.top_k, base.w_router, None, np.arange(E, dtype=np.int32),
                    workload.quantize(Q4_K, np.stack(gus)), workload.quantize(Q5_0, np.stack(dns)), None, None,
                    s_hot=np.linspace(0.5, 1.5, E).astype(np.float32))
    out = MoELayer(hot)(dev(x)).cpu().numpy()
    assert_layer_close(out, port.moe_layer(spec_of(hot, x))["out"], tol=TOL)


def test_zero_tokens_and_bad_args(lib):
    host = host_layer("mini_mixed")
    layer = MoELayer(host)
    x = torch.zeros((0, host.d_model), dtype=torch.float32, device="cuda")
    assert layer(x).shape == (0, host.d_model)
    L = layer.c
    bad = capi.Layer.from_buffer_copy(L)
    bad.d_model = 100
    rc = lib.moeb_layer_forward(C.byref(bad), x.data_ptr(), 1, x.data_ptr(), None, None, 0, stream())
    assert rc == -1


class _Pool:
    """LIFO device scratch for the moert vtable (the ggml pool contract)."""

    def __init__(self):
        self.live = []
        self.alloc = C.CFUNCTYPE(C.c_void_p, C.c_void_p, C.c_uint64)(self._alloc)
        self.free = C.CFUNCTYPE(None, C.c_void_p, C.c_void_p)(self._free)

    def _alloc(self, user, n):
        t = torch.empty(int(n), dtype=torch.uint8, device="cuda")
        self.live.append(t)
        return t.data_ptr()

    def _free(self, user, p):
        assert self.live and self.live[-1].data_ptr() == p, "pool free must be LIFO"
        self.live.pop()


class _Host(C.Structure):
    _fields_ = [("user", C.c_void_p), ("pool_alloc", C.c_void_p), ("pool_free", C.c_void_p), ("mm", C.c_void_p)]


class _Args(C.Structure):
    _fields_ = [("kind", C.c_int32), ("top_k", C.c_int32), ("il", C.c_int32), ("planc_mode", C.c_int32),
                ("n_used", C.c_int32), ("n_tokens", C.c_int32), ("ids_s1", C.c_int32), ("d_in", C.c_int32),
                ("d_out", C.c_int32), ("n_expert", C.c_int32), ("k", C.c_int32), ("cold_type_tag", C.c_int32),
                ("expert_bytes", C.c_uint64), ("cur", C.c_void_p), ("ids", C.c_void_p), ("exp_slot", C.c_void_p),
                ("slot_exp", C.c_void_p), ("slot_state", C.c_void_p), ("s_hot", C.c_void_p), ("s_cold", C.c_void_p),
                ("w_cold_dev", C.c_uint64), ("s_cold_dev", C.c_uint64), ("has_w_cold", C.c_int32),
                ("dst", C.c_void_p), ("stream", C.c_void_p)]


def test_moert_ffn_moe_per_kind(port, lib):
    """The moert island ABI: kind 0 (gate_up) and kind 1 (down) on given routes, argsort-view
    row stride, hot/cold by the residency mirror, scale applied once on down."""
    host = host_layer("decode_t4_mixed")
    layer = MoELayer(host)
    T, k, E, d, nff = 3, host.top_k, host.n_expert, host.d_model, host.n_ff
    from llapis_b200 import workload
    x = workload.make_input(workload.CONFIGS["decode_t4_mixed"], n_tokens=T, stream=5)
    want = port.moe_layer(spec_of(host, x), want=("ids", "gate_up", "act", "down"))
    ids_view = np.zeros((T, E), np.int32)      # argsort_top_k view: row stride n_expert
    ids_view[:, :k] = want["ids"]
    t = layer.t
    il = 7
    capi.check(lib.moeb_bind_pools(il, 0, t["hot_gu"].data_ptr(), Q4_K, host.n_slots, t["cold_gu"].data_ptr(), IQ2_S, E))
    capi.check(lib.moeb_bind_pools(il, 1, t["hot_down"].data_ptr(), Q5_0, host.n_slots, t["cold_down"].data_ptr(),
                                   IQ4_NL, E))
    pool = _Pool()
    h = _Host(None, C.cast(pool.alloc, C.c_void_p), C.cast(pool.free, C.c_void_p), None)
    ids_d = dev(ids_view)
    for kind, cur, d_in, d_out, ref_out, ctype in ((0, x, d, 2 * nff, want["gate_up"], IQ2_S),
                                                   (1, want["act"], nff, d, want["down"], IQ4_NL)):
        cur_d = dev(cur)
        dst = torch.empty((T * k, d_out), dtype=torch.float32, device="cuda")
        a = _Args(kind, k, il, 0, k, T, E, d_in, d_out, E, host.n_slots, ctype,
                  d_out * capi.row_size(ctype, d_in), cur_d.data_ptr(), ids_d.data_ptr(),
                  t["exp_slot"].data_ptr(), t["slot_exp"].data_ptr(), t["slot_state"].data_ptr(),
                  t["s_hot"].data_ptr(), t["s_cold"].data_ptr(), 0, 0, 1, dst.data_ptr(), stream())
        lib.moert_ffn_moe(C.byref(a), C.byref(h))
        torch.cuda.synchronize()
        assert not pool.live
        assert_layer_close(dst.cpu().numpy(), ref_out, tol=1e-5 if kind == 0 else TOL)
