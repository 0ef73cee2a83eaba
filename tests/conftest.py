import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")
GOLDEN_BLOCK = os.path.join(ROOT, "tests", "golden", "golden_block.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN, allow_pickle=False))


@pytest.fixture(scope="session")
def golden_block():
    """Reference outputs of the Gemma-4 block norms (tests/golden/make_golden.py --block)."""
    return dict(np.load(GOLDEN_BLOCK, allow_pickle=False))


@pytest.fixture(scope="session")
def port():
    from oracle import Port
    return Port()


@pytest.fixture(scope="session")
def ref():
    from oracle import Ref, ref_available
    if not ref_available():
        pytest.skip("oracle/_ref not built (make -C oracle ref needs the reference sources)")
    return Ref()


@pytest.fixture(scope="session")
def lib():
    from llapis_b200 import capi
    return capi.lib()


_layers = {}


def host_layer(name):
    """Quantised host weights of layer 0 of a workload config (built once per session)."""
    from llapis_b200 import workload
    if name not in _layers:
        _layers[name] = workload.build_layer(workload.CONFIGS[name])
    return _layers[name]


def spec_of(host, x):
    """oracle.LayerSpec for a llapis_b200 HostLayer."""
    from oracle import LayerSpec
    exp_slot, slot_exp, slot_state = host.residency()
    K = host.n_slots
    return LayerSpec(host.d_model, host.n_ff, host.n_expert, host.top_k, x=x, w_router=host.w_router,
                     b_router=host.b_router, n_slots=K, exp_slot=exp_slot if K else None,
                     slot_exp=slot_exp if K else None, slot_state=slot_state if K else None,
                     hot_type_gu=host.hot_type_gu, hot_type_down=host.hot_type_down, hot_gu=host.hot_gu,
                     hot_down=host.hot_down, s_hot=host.s_hot, cold_type_gu=host.cold_type_gu,
                     cold_type_down=host.cold_type_down, cold_gu=host.cold_gu, cold_down=host.cold_down,
                     s_cold=host.s_cold)


def sha(a):
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def near_tie_tokens(logits, k, rel=1e-6):
    """Tokens whose k-th and (k+1)-th largest logits are within rel: their top-k set is not
    determined by the float values alone (the reference's argsort is unstable)."""
    s = -np.sort(-logits, axis=-1)
    gap = np.abs(s[:, k - 1] - s[:, k])
    return np.nonzero(gap <= rel * np.maximum(1.0, np.abs(s[:, k - 1])))[0]


def assert_layer_close(out, want, tol=2e-3):
    """The parity bar: max-abs <= tol x RMS of the reference output."""
    rms = float(np.sqrt(np.mean(np.square(want, dtype=np.float64))))
    err = float(np.max(np.abs(out.astype(np.float64) - want)))
    assert err <= tol * rms, f"max-abs {err:.3e} > {tol} x rms {rms:.3e}"
    return err / rms
