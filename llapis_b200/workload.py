"""Seeded synthetic MoE layers with the shapes and value distributions of the benchmark configs.

No dataset or checkpoint is involved: weights are f32 N(0, 0.02) per expert matrix, quantised with
this library's quantiser (byte-identical to the reference quantiser, ggml_quantize_chunk), router
weights f32 N(0, 0.02), activations N(0, 1) (bf16-rounded for the prefill configs, whose inputs
are bf16). Gemma-4 26B-A4B MoE shapes: d_model 2816, 128 experts, top-8, expert inner dim 704,
merged gate_up [1408 x 2816] (gate rows first), down [2816 x 704]. 704 is not a multiple of 256,
so the down projection uses the reference quantiser's fallback types: IQ2_S -> IQ4_NL,
Q4_K -> Q5_0 (third_party/llama/src/llama-quant.cpp:362-388).
"""
from __future__ import annotations

import hashlib
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np

from . import capi
from .capi import IQ2_S, IQ2_XXS, IQ4_NL, Q4_K, Q5_0
from .layer import HostLayer


@dataclass(frozen=True)
class LayerConfig:
    name: str
    n_tokens: int
    hot: tuple            # experts in the Q4_K / Q5_0 class (slot order)
    bias_s: float | None  # router bias b_e = -s * ln(1 + e) (Zipf-like skew to low ids), or None
    bf16_input: bool
    d_model: int = 2816
    n_ff: int = 704
    n_expert: int = 128
    top_k: int = 8
    seed: int = 0
    n_layers: int = 1
    cold_gu_type: int = IQ2_S   # the cold class's gate_up type (IQ2_XXS: the product files' type)


CONFIGS = {
    # BASELINE.json configs[0..4]
    "decode_t1_iq2s": LayerConfig("decode_t1_iq2s", 1, (), None, False),
    "decode_t4_mixed": LayerConfig("decode_t4_mixed", 4, tuple(range(48)), 1.1, False),
    "prefill_t2048_q4k": LayerConfig("prefill_t2048_q4k", 2048, tuple(range(128)), None, True),
    "stack30_t256_mixed": LayerConfig("stack30_t256_mixed", 256, tuple(range(64)), 1.2, True, n_layers=30),
    "ep_prefill_t8192_q4k": LayerConfig("ep_prefill_t8192_q4k", 8192, tuple(range(128)), None, True),
    # reduced shapes for tests (same structure, seconds to build)
    "mini_mixed": LayerConfig("mini_mixed", 3, tuple(range(8)), 1.1, False, d_model=512, n_ff=64, n_expert=32,
                              top_k=4, seed=11),
    # decode_t4_mixed's experts with the product files' cold class, IQ2_XXS gate_up / IQ4_NL down, and
    # no router skew, so both classes are routed
    "decode_t4_iq2xxs": LayerConfig("decode_t4_iq2xxs", 4, tuple(range(48)), None, False, cold_gu_type=IQ2_XXS),
}


def _normal(seed_words, shape, scale) -> np.ndarray:
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence(list(seed_words))))
    a = rng.standard_normal(shape, dtype=np.float32)
    a *= np.float32(scale)
    return a


def expert_f32(cfg: LayerConfig, layer: int, e: int):
    """f32 gate_up [2nff, d] and down [d, nff] of expert e (N(0, 0.02))."""
    gu = _normal((cfg.seed, layer, e, 0), (2 * cfg.n_ff, cfg.d_model), 0.02)
    dn = _normal((cfg.seed, layer, e, 1), (cfg.d_model, cfg.n_ff), 0.02)
    return gu, dn


def quantize(wtype: int, w: np.ndarray, n_threads: int = 0) -> np.ndarray:
    w = np.ascontiguousarray(w, np.float32)
    n = w.shape[-1]
    nrow = w.size // n
    out = np.empty((nrow, capi.row_size(wtype, n)), np.uint8)
    nb = capi.lib().moeb_quantize_weights(wtype, w.ctypes.data, out.ctypes.data, nrow, n, n_threads)
    if nb != out.nbytes:
        raise capi.MoebError(-1, f"quantisation of type {wtype} failed")
    return out.reshape(*w.shape[:-1], out.shape[-1])


def _cache_dir() -> str | None:
    d = os.environ.get("LLAPIS_B200_CACHE", os.path.join(os.path.expanduser("~"), ".cache", "llapis_b200"))
    try:
        os.makedirs(d, exist_ok=True)
        return d
    except OSError:
        return None


def _cached(key: str, make):
    d = _cache_dir()
    path = os.path.join(d, hashlib.sha256(key.encode()).hexdigest()[:24] + ".npy") if d else None
    if path and os.path.exists(path):
        try:
            return np.load(path)
        except (OSError, ValueError):
            pass
    a = make()
    if path:
        try:
            np.save(path + ".tmp.npy", a)
            os.replace(path + ".tmp.npy", path)
        except OSError:
            pass
    return a


def build_layer(cfg: LayerConfig, layer: int = 0, n_threads: int = 0) -> HostLayer:
    """Quantised weights of one layer of `cfg` (cold pool entries of hot experts are left zero:
    the residency mirror never routes a hot expert's pair to the cold pool)."""
    E, d, nff = cfg.n_expert, cfg.d_model, cfg.n_ff
    hot = np.array(cfg.hot, np.int32)
    is_hot = np.zeros(E, bool)
    is_hot[hot] = True

    ct = cfg.cold_gu_type

    def one(e):
        def make():
            gu, dn = expert_f32(cfg, layer, e)
            if is_hot[e]:
                a, b = quantize(Q4_K, gu, 1), quantize(Q5_0, dn, 1)
            else:
                a, b = quantize(ct, gu, 1), quantize(IQ4_NL, dn, 1)
            return np.concatenate([a.reshape(-1), b.reshape(-1)])
        tag = "" if is_hot[e] or ct == IQ2_S else f"|{ct}"
        return _cached(f"v1|{cfg.seed}|{layer}|{e}|{d}|{nff}|{int(is_hot[e])}{tag}", make)

    nt = n_threads or os.cpu_count() or 1
    capi.lib().moeb_quantize_weights(ct, np.zeros(256, np.float32).ctypes.data, np.zeros(128, np.uint8).ctypes.data, 1,
                                     256, 1)   # build the codebook search tables once
    with ThreadPoolExecutor(max_workers=nt) as ex:
        blobs = list(ex.map(one, range(E)))
    hgu, hdn = 2 * nff * capi.row_size(Q4_K, d), d * capi.row_size(Q5_0, nff)
    cgu, cdn = 2 * nff * capi.row_size(ct, d), d * capi.row_size(IQ4_NL, nff)
    K = len(hot)
    hot_gu = np.zeros((K, 2 * nff, capi.row_size(Q4_K, d)), np.uint8) if K else None
    hot_dn = np.zeros((K, d, capi.row_size(Q5_0, nff)), np.uint8) if K else None
    n_cold = int((~is_hot).sum())
    cold_gu = np.zeros((E, 2 * nff, capi.row_size(ct, d)), np.uint8) if n_cold else None
    cold_dn = np.zeros((E, d, capi.row_size(IQ4_NL, nff)), np.uint8) if n_cold else None
    slot = {int(e): s for s, e in enumerate(hot)}
    for e in range(E):
        b = blobs[e]
        if is_hot[e]:
            hot_gu[slot[e]] = b[:hgu].reshape(2 * nff, -1)
            hot_dn[slot[e]] = b[hgu:hgu + hdn].reshape(d, -1)
        else:
            cold_gu[e] = b[:cgu].reshape(2 * nff, -1)
            cold_dn[e] = b[cgu:cgu + cdn].reshape(d, -1)
    w_router = _normal((cfg.seed, layer, 1 << 20), (E, d), 0.02)
    b_router = None
    if cfg.bias_s is not None:
        b_router = (-cfg.bias_s * np.log1p(np.arange(E, dtype=np.float64))).astype(np.float32)
    return HostLayer(d_model=d, n_ff=nff, n_expert=E, top_k=cfg.top_k, w_router=w_router, b_router=b_router,
                     hot_ids=hot, hot_gu=hot_gu, hot_down=hot_dn, cold_gu=cold_gu, cold_down=cold_dn, cold_type_gu=ct,
                     s_hot=np.ones(K, np.float32) if K else None, s_cold=np.ones(E, np.float32) if n_cold else None)


def make_input(cfg: LayerConfig, n_tokens: int | None = None, stream: int = 0) -> np.ndarray:
    """Activations [T, d] N(0, 1); bf16-rounded when the config's inputs are bf16."""
    T = cfg.n_tokens if n_tokens is None else n_tokens
    x = _normal((cfg.seed, 7777, stream), (T, cfg.d_model), 1.0)
    if cfg.bf16_input:
        u = x.view(np.uint32)
        u = ((u + 0x7fff + ((u >> 16) & 1)) & 0xffff0000).astype(np.uint32)   # round to nearest even bf16
        x = u.view(np.float32)
    return x


NORM_EPS = 1e-6   # Gemma-4 f_norm_rms_eps


def block_norms(cfg: LayerConfig, layer: int = 0):
    """Seeded Gemma-4 block norm vectors for layer `layer` of cfg (f32 [d_model]), eps 1e-6:
    ffn_pre_norm_2 and ffn_post_norm_2 1 + N(0, 0.1); ffn_gate_inp_s sqrt(d) * (1 + N(0, 0.1)), so
    that the router input rms_norm(x) / sqrt(d) * ffn_gate_inp_s has unit scale and the N(0, 0.02)
    router weights give logits of the same spread as the plain layer's N(0, 1) input does."""
    from .layer import BlockNorms
    d = cfg.d_model
    v = [np.float32(1.0) + _normal((cfg.seed, layer, 1 << 21, i), (d,), 0.1) for i in range(3)]
    v[1] = (v[1] * np.sqrt(np.float32(d))).astype(np.float32)
    return BlockNorms(pre_norm=v[0], router_scale=v[1], post_norm=v[2], eps=NORM_EPS)


def make_block_input(cfg: LayerConfig, n_tokens: int | None = None, stream: int = 0) -> np.ndarray:
    """Block input (attn_out, the residual stream) [T, d]: make_input's rows times a per-token
    magnitude 2^u, u uniform in [0, 4), so the norms' row scales vary over tokens."""
    x = make_input(cfg, n_tokens, stream)
    rng = np.random.Generator(np.random.PCG64(np.random.SeedSequence([cfg.seed, 9191, stream])))
    mag = np.exp2(rng.uniform(0.0, 4.0, (x.shape[0], 1))).astype(np.float32)
    return (x * mag).astype(np.float32)


def algorithmic_bytes(host: HostLayer, ids: np.ndarray, n_tokens: int) -> int:
    """Unique routed experts' weight bytes + router + activations in and out (f32)."""
    uniq = np.unique(ids.reshape(-1))
    wb = sum(host.expert_bytes(int(e)) for e in uniq)
    return int(wb + host.w_router.nbytes + 2 * n_tokens * host.d_model * 4)


def layer_flops(host: HostLayer, n_tokens: int) -> int:
    per_pair = 2 * (2 * host.n_ff) * host.d_model + 2 * host.d_model * host.n_ff
    return int(n_tokens * host.top_k * per_pair + n_tokens * 2 * host.d_model * host.n_expert)


# ---------------------------------------------------------------- Gemma-4 dense (shared) MLP
# The dense MLP beside the MoE in every Gemma-4 MoE block (third_party/llama/src/models/gemma4.cpp:
# 376-391: build_ffn with GELU / PAR, gate and up [n_ff_dense x d], down [d x n_ff_dense]) is this
# path's layer with one expert: a hot slot holding [gate rows; up rows] and down, zero router weights
# with a bias that puts every token on expert 0 at top-1 (softmax weight exactly 1.0), scale 1.
DENSE_D, DENSE_NFF, DENSE_E, DENSE_SEED = 2816, 2112, 32, 3


def dense_mlp_f32(d: int = DENSE_D, nff: int = DENSE_NFF, seed: int = DENSE_SEED):
    """f32 gate [nff, d], up [nff, d] and down [d, nff] of the dense MLP (N(0, 0.02))."""
    return (_normal((seed, 5151, 0), (nff, d), 0.02), _normal((seed, 5151, 1), (nff, d), 0.02),
            _normal((seed, 5151, 2), (d, nff), 0.02))


def dense_as_layer(w_gate_q: np.ndarray, w_up_q: np.ndarray, w_down_q: np.ndarray, d: int, nff: int,
                   gu_type: int = Q4_K, dn_type: int = Q5_0, n_expert: int = DENSE_E) -> HostLayer:
    """A quantised dense GeGLU MLP as a one-expert MoE layer (see the block comment above)."""
    b = np.full(n_expert, -1e4, np.float32)
    b[0] = 0.0
    return HostLayer(d_model=d, n_ff=nff, n_expert=n_expert, top_k=1, w_router=np.zeros((n_expert, d), np.float32),
                     b_router=b, hot_ids=np.zeros(1, np.int32), hot_gu=np.concatenate([w_gate_q, w_up_q])[None],
                     hot_down=np.asarray(w_down_q)[None], cold_gu=None, cold_down=None, hot_type_gu=gu_type,
                     hot_type_down=dn_type, s_hot=np.ones(1, np.float32))


def build_dense_layer(d: int = DENSE_D, nff: int = DENSE_NFF, seed: int = DENSE_SEED) -> HostLayer:
    """The seeded dense MLP (Q4_K gate / up, Q5_0 down), quantised with this library's quantiser."""
    def make():
        g, u, w = dense_mlp_f32(d, nff, seed)
        return np.concatenate([quantize(Q4_K, g).reshape(-1), quantize(Q4_K, u).reshape(-1),
                               quantize(Q5_0, w).reshape(-1)])
    blob = _cached(f"dense-v1|{seed}|{d}|{nff}", make)
    ng = nff * capi.row_size(Q4_K, d)
    g = blob[:ng].reshape(nff, -1)
    u = blob[ng:2 * ng].reshape(nff, -1)
    w = blob[2 * ng:].reshape(d, -1)
    return dense_as_layer(g, u, w, d, nff)


def make_dense_input(n_tokens: int, seed: int = DENSE_SEED) -> np.ndarray:
    """Dense-MLP input rows [T, d] N(0, 1)."""
    return _normal((seed, 7777, 0), (n_tokens, DENSE_D), 1.0)


def dense_block_norms(d: int = DENSE_D, seed: int = DENSE_SEED):
    """Seeded norms of the dense branch (f32 [d], eps 1e-6): ffn_norm and ffn_post_norm_1
    1 + N(0, 0.1); router_scale ones (unused: the one-expert layer's router weights are zero)."""
    from .layer import BlockNorms
    v = [np.float32(1.0) + _normal((seed, 6161, i), (d,), 0.1) for i in range(2)]
    return BlockNorms(pre_norm=v[0], router_scale=np.ones(d, np.float32), post_norm=v[1], eps=NORM_EPS)
