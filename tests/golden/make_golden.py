"""Generates the golden fixtures under tests/golden/ from the REFERENCE itself.

    make -C oracle ref          # builds oracle/_ref from the reference sources
    python tests/golden/make_golden.py           # golden.npz
    python tests/golden/make_golden.py --block   # golden_block.npz (the Gemma-4 block norms)
    python tests/golden/make_golden.py --types   # golden_types.npz + the IQ2_XXS tables (IQ2_XXS / Q8_0 weights)
    python tests/golden/make_golden.py --prefill # golden_prefill.npz (T=2048 prefill layer, stack layer 0)
    python tests/golden/make_golden.py --dense   # golden_dense.npz (the Gemma-4 dense MLP, 2112 wide)

Everything in the fixtures comes out of the reference's own code (ggml-base + ggml-cpu of the
vendored llama.cpp, compiled into oracle/_ref): quantised bytes from ggml_quantize_chunk, dequantised
rows from the type traits' to_float, activation blocks from the CPU from_float, the fp16 GELU table
ggml_cpu_init fills, and whole-layer outputs from the O1 ggml graph (oracle/ref_runner.cpp). Large
arrays are stored as SHA-256 digests; the tests regenerate them and compare digests.

It also writes the IQ2_S / IQ4_NL format tables that the library and the restated oracle compile in
(llapis_b200/csrc/ggml_tables.inc, oracle/ggml_tables.inc), recovered by dequantising crafted
blocks through the reference dequantiser.
"""
from __future__ import annotations

import hashlib
import os
import sys
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.oracle import IQ2_S, IQ2_XXS, IQ4_NL, Q4_K, Q5_0, Q8_0, Q8_K, LayerSpec, Ref  # noqa: E402
from llapis_b200 import workload  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def canonical_nan_f16(t: np.ndarray) -> np.ndarray:
    """f16 table with every NaN replaced by 0x7e00 (NaN payload bits carry no meaning here)."""
    t = t.copy()
    t[np.isnan(t.view(np.float16))] = 0x7E00
    return t


def extract_tables(r: Ref):
    grid = np.zeros(1024, np.uint64)
    for b in range(32):
        blk = np.zeros(82, np.uint8)
        blk[0:2] = np.frombuffer(np.float16(8.0).tobytes(), np.uint8)
        for g in range(32):
            idx = b * 32 + g
            ib32, l = g // 4, g % 4
            blk[2 + l + 4 * ib32] = idx & 255
            blk[2 + 64 + ib32] |= ((idx >> 8) & 3) << (2 * l)
        y = r.dequantize(IQ2_S, blk, 256)
        for g in range(32):
            grid[b * 32 + g] = np.frombuffer(y[g * 8:(g + 1) * 8].astype(np.uint8).tobytes(), np.uint64)[0]
    blk = np.zeros(18, np.uint8)
    blk[0:2] = np.frombuffer(np.float16(1.0).tobytes(), np.uint8)
    blk[2:18] = np.arange(16, dtype=np.uint8)
    kv = r.dequantize(IQ4_NL, blk, 32)[:16].astype(np.int8)
    return grid, kv


def extract_iq2xxs_tables(r: Ref):
    """The IQ2_XXS codebook (256 rows) and its 128 sign patterns, through the reference dequantiser
    (dequantize_row_iq2_xxs, ggml-quants.c:2416): with d = 8 and a zero sub-scale a group's
    multiplier is exactly 1, so sign index 0 returns codebook rows verbatim, and codebook row 0
    (no zero magnitude) shows each sign pattern as the negative entries."""
    def block(idx, sgn):   # 32 groups: codebook indices and sign indices, sub-scale 0
        blk = np.zeros(66, np.uint8)
        blk[0:2] = np.frombuffer(np.float16(8.0).tobytes(), np.uint8)
        for ib in range(8):
            w0 = sum(int(idx[4 * ib + l]) << (8 * l) for l in range(4))
            w1 = sum(int(sgn[4 * ib + l]) << (7 * l) for l in range(4))
            blk[2 + 8 * ib:2 + 8 * ib + 8] = np.frombuffer(np.array([w0, w1], np.uint32).tobytes(), np.uint8)
        return blk
    grid = np.zeros(256, np.uint64)
    for b in range(8):
        y = r.dequantize(IQ2_XXS, block(range(32 * b, 32 * b + 32), [0] * 32), 256)
        for g in range(32):
            grid[32 * b + g] = np.frombuffer(y[8 * g:8 * g + 8].astype(np.uint8).tobytes(), np.uint64)[0]
    assert all(((int(grid[0]) >> (8 * j)) & 0xff) for j in range(8))
    signs = np.zeros(128, np.uint8)
    for b in range(4):
        y = r.dequantize(IQ2_XXS, block([0] * 32, range(32 * b, 32 * b + 32)), 256)
        for g in range(32):
            signs[32 * b + g] = sum(1 << j for j in range(8) if y[8 * g + j] < 0)
    return grid, signs


def write_tables(grid, kv, xxs_grid=None, xxs_signs=None):
    body = ("/* IQ2_S codebook: 1024 rows of 8 unsigned magnitudes in {8, 25, 43}, packed little-endian\n"
            " * into one 64-bit word per row. Format constant of ggml's block_iq2_s; the values were\n"
            " * recovered by dequantising crafted blocks through the reference dequantiser\n"
            " * (dequantize_row_iq2_s, third_party/llama/ggml/src/ggml-quants.c:2471) with d = 8 and a\n"
            " * zero sub-scale, which returns each codebook row verbatim. */\n"
            "#define MOE_IQ2S_GRID_ROWS 1024\n#define MOE_IQ2S_GRID_INIT { \\\n")
    for i in range(0, 1024, 4):
        body += "    " + ", ".join("0x%016xull" % int(v) for v in grid[i:i + 4]) + (", \\\n" if i + 4 < 1024 else " \\\n")
    body += "}\n\n/* IQ4_NL non-linear 4-bit levels (block_iq4_nl format constant), recovered the same way through\n" \
            " * dequantize_row_iq4_nl (ggml-quants.c:2653) with d = 1. */\n"
    body += "#define MOE_IQ4NL_VALUES_INIT { " + ", ".join(str(int(v)) for v in kv) + " }\n"
    if xxs_grid is not None:
        body += ("\n/* IQ2_XXS codebook (256 rows of 8 magnitudes, one 64-bit word per row) and its 128 sign\n"
                 " * patterns (bit j set: value j negative), format constants of ggml's block_iq2_xxs, recovered\n"
                 " * through dequantize_row_iq2_xxs (ggml-quants.c:2416) with d = 8 and a zero sub-scale. */\n"
                 "#define MOE_IQ2XXS_GRID_INIT { \\\n")
        for i in range(0, 256, 4):
            body += "    " + ", ".join("0x%016xull" % int(v) for v in xxs_grid[i:i + 4]) + (", \\\n" if i + 4 < 256 else " \\\n")
        body += "}\n#define MOE_IQ2XXS_SIGNS_INIT { " + ", ".join(str(int(v)) for v in xxs_signs) + " }\n"
    with open(os.path.join(ROOT, "llapis_b200", "csrc", "ggml_tables.inc"), "w") as f:
        f.write("/* Generated by tests/golden/make_golden.py — do not edit. */\n" + body)
    with open(os.path.join(ROOT, "oracle", "ggml_tables.inc"), "w") as f:
        f.write("/* TEST INFRASTRUCTURE copy of the ggml format tables, generated by tests/golden/make_golden.py. */\n"
                + body)


def ref_pools(r: Ref, cfg, n_threads=8):
    """The reference quantiser over every expert of layer 0 of cfg (same f32 source as the library)."""
    E = cfg.n_expert
    hot = set(cfg.hot)
    r.quantize(IQ2_S, np.zeros((1, 256), np.float32))   # builds the reference's IQ2_S tables once

    def one(e):
        gu, dn = workload.expert_f32(cfg, 0, e)
        if e in hot:
            return e, r.quantize(Q4_K, gu), r.quantize(Q5_0, dn)
        return e, r.quantize(IQ2_S, gu), r.quantize(IQ4_NL, dn)

    with ThreadPoolExecutor(n_threads) as ex:
        res = list(ex.map(one, range(E)))
    return res


def layer_spec(cfg, pools, x):
    hot = np.array(cfg.hot, np.int32)
    E, K = cfg.n_expert, len(hot)
    exp_slot = np.full(E, -1, np.int32)
    exp_slot[hot] = np.arange(K, dtype=np.int32)
    by_e = {e: (a, b) for e, a, b in pools}
    hot_gu = np.stack([by_e[int(e)][0] for e in hot]) if K else None
    hot_dn = np.stack([by_e[int(e)][1] for e in hot]) if K else None
    n_cold = E - K
    cold_gu = cold_dn = None
    if n_cold:
        some = next(e for e in range(E) if e not in set(cfg.hot))
        cold_gu = np.zeros((E,) + by_e[some][0].shape, np.uint8)
        cold_dn = np.zeros((E,) + by_e[some][1].shape, np.uint8)
        for e in range(E):
            if e not in set(cfg.hot):
                cold_gu[e], cold_dn[e] = by_e[e]
    w_router = workload._normal((cfg.seed, 0, 1 << 20), (E, cfg.d_model), 0.02)
    b = None if cfg.bias_s is None else (-cfg.bias_s * np.log1p(np.arange(E, dtype=np.float64))).astype(np.float32)
    return LayerSpec(cfg.d_model, cfg.n_ff, E, cfg.top_k, x=x, w_router=w_router, b_router=b, n_slots=K,
                     exp_slot=exp_slot if K else None, slot_exp=hot if K else None,
                     slot_state=np.full(K, 2, np.int32) if K else None, hot_gu=hot_gu, hot_down=hot_dn,
                     s_hot=np.ones(K, np.float32) if K else None, cold_gu=cold_gu, cold_down=cold_dn,
                     s_cold=np.ones(E, np.float32) if n_cold else None)


def pool_digests(spec: LayerSpec) -> dict:
    out = {}
    for n in ("hot_gu", "hot_down", "cold_gu", "cold_down"):
        a = getattr(spec, n)
        out[n] = sha(a) if a is not None else ""
    return out


def main():
    r = Ref()
    grid, kv = extract_tables(r)
    write_tables(grid, kv)
    rng = np.random.default_rng(20261201)
    fx = {"iq2s_grid": grid, "iq4nl_values": kv}

    # ---- primitives: dequantisation of reference-quantised rows, activation blocks, GELU table
    for t, n in ((Q4_K, 512), (IQ2_S, 512), (Q5_0, 64), (IQ4_NL, 64)):
        w = rng.normal(0, 0.02, (6, n)).astype(np.float32)
        w[1] *= 1e-3
        w[2, 3] = 0.5
        q = r.quantize(t, w)
        fx[f"deq_{t}_src"] = q
        fx[f"deq_{t}_f32"] = np.stack([r.dequantize(t, q[i], n) for i in range(len(q))])
    for vdt, n in ((Q8_K, 512), (Q8_0, 64)):
        x = rng.normal(0, 1, (5, n)).astype(np.float32)
        x[1] = 0.0
        x[2, 7] = -x[2].__abs__().max() * 2        # signed max drives the Q8_K scale
        x[3, :2] = [1e-4, -1e-4]
        fx[f"act_{vdt}_x"] = x
        fx[f"act_{vdt}_q"] = np.stack([r.quantize_act(vdt, x[i]) for i in range(len(x))])
    fx["gelu_table_sha"] = np.array(sha(canonical_nan_f16(r.gelu_table())))

    # ---- whole layer, reduced shape (mixed classes, bias, scales), every intermediate
    cfg = workload.CONFIGS["mini_mixed"]
    pools = ref_pools(r, cfg)
    x = workload.make_input(cfg)
    spec = layer_spec(cfg, pools, x)
    res = r.moe_layer(spec, n_threads=4)
    for k, v in res.items():
        fx[f"mini_{k}"] = v
    fx["mini_x"] = x
    for k, v in pool_digests(spec).items():
        fx[f"mini_sha_{k}"] = np.array(v)

    # ---- real shapes: decode T=1 all IQ2_S and decode T=4 mixed (BASELINE configs 0 and 1)
    for name, T in (("decode_t1_iq2s", 2), ("decode_t4_mixed", 4)):
        cfg = workload.CONFIGS[name]
        pools = ref_pools(r, cfg)
        x = workload.make_input(cfg, n_tokens=T)
        spec = layer_spec(cfg, pools, x)
        res = r.moe_layer(spec, n_threads=8, want=("logits", "ids", "weights"))
        for k in ("logits", "ids", "weights", "out"):
            fx[f"{name}_{k}"] = res[k]
        fx[f"{name}_x"] = x
        for k, v in pool_digests(spec).items():
            fx[f"{name}_sha_{k}"] = np.array(v)
        print(name, "done")

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **fx)
    print("wrote", os.path.join(HERE, "golden.npz"), os.path.getsize(os.path.join(HERE, "golden.npz")), "bytes")


def block_spec(cfg, x):
    """The layer of cfg for the block fixtures: pools from this library's quantiser, whose bytes
    golden.npz pins to the reference quantiser's (the mini and decode_t4_mixed pool digests)."""
    from oracle import LayerSpec
    host = workload.build_layer(cfg)
    exp_slot, slot_exp, slot_state = host.residency()
    K = host.n_slots
    return LayerSpec(host.d_model, host.n_ff, host.n_expert, host.top_k, x=x, w_router=host.w_router,
                     b_router=host.b_router, n_slots=K, exp_slot=exp_slot if K else None,
                     slot_exp=slot_exp if K else None, slot_state=slot_state if K else None, hot_gu=host.hot_gu,
                     hot_down=host.hot_down, s_hot=host.s_hot, cold_gu=host.cold_gu, cold_down=host.cold_down,
                     s_cold=host.s_cold), pool_digests_host(host)


def pool_digests_host(host) -> dict:
    return {n: sha(getattr(host, n)) if getattr(host, n) is not None else ""
            for n in ("hot_gu", "hot_down", "cold_gu", "cold_down")}


def main_block():
    """The Gemma-4 MoE block norms (gemma4.cpp:394-427) through the reference: ggml_rms_norm rows
    (plain, with a weight, with a scale and a weight), and whole blocks (the reference's rms_norm /
    scale / mul nodes around its MoE graph) on the mini shape and at decode_t4_mixed's real shape."""
    r = Ref()
    rng = np.random.default_rng(20261202)
    fx = {}
    d = 1024
    x = rng.normal(0, 1, (6, d)).astype(np.float32)
    x *= np.array([[1.0], [30.0], [1e-3], [1e3], [1.0], [7.0]], np.float32)
    x[4] = 0.0                     # zero row: scale 1 / sqrt(eps), output zero
    x[5, ::3] = 0.0
    w = (1.0 + rng.normal(0, 0.1, d)).astype(np.float32)
    c = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    fx["rms_x"], fx["rms_w"], fx["rms_c"] = x, w, np.float32(c)
    fx["rms_plain"] = r.rms_norm(x, workload.NORM_EPS)
    fx["rms_weight"] = r.rms_norm(x, workload.NORM_EPS, w)
    fx["rms_router"] = r.rms_norm(x, workload.NORM_EPS, w, c)
    for name, T in (("mini_mixed", 16), ("decode_t4_mixed", 4)):
        cfg = workload.CONFIGS[name]
        xb = workload.make_block_input(cfg, n_tokens=T, stream=77)
        spec, dig = block_spec(cfg, xb)
        nrm = workload.block_norms(cfg)
        want = ("logits", "ids", "weights", "gate_up", "down") if name == "mini_mixed" else ("logits", "ids", "weights")
        res = r.gemma4_block(spec, nrm, n_threads=8, want=want)
        fx[f"{name}_x"] = xb
        for k in want + ("moe", "out", "x_expert", "x_router"):
            fx[f"{name}_{k}"] = res[k]
        for k, v in dig.items():
            fx[f"{name}_sha_{k}"] = np.array(v)
        print(name, "done")
    path = os.path.join(HERE, "golden_block.npz")
    np.savez_compressed(path, **fx)
    print("wrote", path, os.path.getsize(path), "bytes")


def main_types():
    """IQ2_XXS and Q8_0 expert weights (the other types the product files use): the tables, reference
    dequantised rows, and a mini layer whose cold class is IQ2_XXS gate_up / IQ4_NL down and whose
    hot class is Q8_0 gate_up and down, through the reference's MUL_MAT_ID graph."""
    r = Ref()
    write_tables(*extract_tables(r), *extract_iq2xxs_tables(r))
    rng = np.random.default_rng(20261203)
    fx = {}
    for t, n in ((IQ2_XXS, 512), (Q8_0, 64)):
        w = rng.normal(0, 0.02, (6, n)).astype(np.float32)
        w[1] *= 1e-3
        w[2, 3] = 0.5
        q = r.quantize(t, w)
        fx[f"deq_{t}_src"] = q
        fx[f"deq_{t}_f32"] = np.stack([r.dequantize(t, q[i], n) for i in range(len(q))])
    cfg = workload.CONFIGS["mini_mixed"]
    E, d, nff, hot = cfg.n_expert, cfg.d_model, cfg.n_ff, list(cfg.hot)
    cold_gu, cold_dn, hot_gu, hot_dn = [], [], [], []
    for e in range(E):
        gu, dn = workload.expert_f32(cfg, 0, e)
        cold_gu.append(r.quantize(IQ2_XXS, gu))
        cold_dn.append(r.quantize(IQ4_NL, dn))
        if e in hot:
            hot_gu.append(r.quantize(Q8_0, gu))
            hot_dn.append(r.quantize(Q8_0, dn))
    x = workload.make_input(cfg, n_tokens=12, stream=5)
    K = len(hot)
    exp_slot = np.full(E, -1, np.int32)
    exp_slot[hot] = np.arange(K, dtype=np.int32)
    spec = LayerSpec(d, nff, E, cfg.top_k, x=x, w_router=workload._normal((cfg.seed, 0, 1 << 20), (E, d), 0.02),
                     n_slots=K, exp_slot=exp_slot, slot_exp=np.array(hot, np.int32),
                     slot_state=np.full(K, 2, np.int32), hot_type_gu=Q8_0, hot_type_down=Q8_0,
                     hot_gu=np.stack(hot_gu), hot_down=np.stack(hot_dn), s_hot=np.ones(K, np.float32),
                     cold_type_gu=IQ2_XXS, cold_type_down=IQ4_NL, cold_gu=np.stack(cold_gu),
                     cold_down=np.stack(cold_dn), s_cold=np.ones(E, np.float32))
    res = r.moe_layer(spec, n_threads=4)
    for k, v in res.items():
        fx[f"types_{k}"] = v
    fx["types_x"] = x
    for n in ("hot_gu", "hot_down", "cold_gu", "cold_down"):   # the pools are regenerated by the tests
        fx[f"types_sha_{n}"] = np.array(sha(getattr(spec, n)))
    # real shape, the product files' cold class: decode_t4_iq2xxs (cold gate_up IQ2_XXS from the
    # reference quantiser, digest pinned; the other pools are digest-pinned by golden.npz)
    cfg = workload.CONFIGS["decode_t4_iq2xxs"]
    host = workload.build_layer(cfg)
    hot_set = set(cfg.hot)
    r.quantize(IQ2_XXS, np.zeros((1, 256), np.float32))   # the reference's IQ2_XXS tables, once

    def cold_row(e):
        return e, (None if e in hot_set else r.quantize(IQ2_XXS, workload.expert_f32(cfg, 0, e)[0]))
    with ThreadPoolExecutor(8) as ex:
        cold = dict(ex.map(cold_row, range(cfg.n_expert)))
    cold_gu = np.zeros_like(host.cold_gu)
    for e, q in cold.items():
        if q is not None:
            cold_gu[e] = q
    fx["real_sha_cold_gu"] = np.array(sha(cold_gu))
    x = workload.make_input(cfg)
    from oracle import LayerSpec as _LS
    exp_slot, slot_exp, slot_state = host.residency()
    spec = _LS(host.d_model, host.n_ff, host.n_expert, host.top_k, x=x, w_router=host.w_router, b_router=host.b_router,
               n_slots=host.n_slots, exp_slot=exp_slot, slot_exp=slot_exp, slot_state=slot_state, hot_gu=host.hot_gu,
               hot_down=host.hot_down, s_hot=host.s_hot, cold_type_gu=IQ2_XXS, cold_gu=cold_gu,
               cold_down=host.cold_down, s_cold=host.s_cold)
    res = r.moe_layer(spec, n_threads=8, want=("logits", "ids", "weights"))
    for k in ("logits", "ids", "weights", "out"):
        fx[f"real_{k}"] = res[k]
    fx["real_x"] = x
    path = os.path.join(HERE, "golden_types.npz")
    np.savez_compressed(path, **fx)
    print("wrote", path, os.path.getsize(path), "bytes")


def token_digests(a: np.ndarray, T: int) -> np.ndarray:
    """Per-token 64-bit digests (leading 8 bytes of SHA-256) of a [T * k, n] f32 array in pair order."""
    rows = a.reshape(T, -1)
    return np.array([np.frombuffer(hashlib.sha256(np.ascontiguousarray(rows[t]).tobytes()).digest()[:8], np.uint64)[0]
                     for t in range(T)], np.uint64)


def main_prefill():
    """The prefill workloads at their full token counts through the reference graph: routing, per-token
    digests of gate_up and of the GeGLU output (both bit-exact targets), and the outputs of every
    `step`-th token with the whole output's RMS (the parity bar's scale)."""
    r = Ref()
    fx = {}
    for name, step in (("prefill_t2048_q4k", 32), ("stack30_t256_mixed", 8)):
        cfg = workload.CONFIGS[name]
        pools = ref_pools(r, cfg)
        x = workload.make_input(cfg)
        T = x.shape[0]
        spec = layer_spec(cfg, pools, x)
        res = r.moe_layer(spec, n_threads=8, want=("logits", "ids", "weights", "gate_up", "act"))
        fx[f"{name}_ids"] = res["ids"]
        fx[f"{name}_logits_sha"] = np.array(sha(res["logits"]))
        fx[f"{name}_gate_up_digest"] = token_digests(res["gate_up"], T)
        fx[f"{name}_act_digest"] = token_digests(res["act"], T)
        fx[f"{name}_out_rows"] = np.arange(0, T, step, dtype=np.int32)
        fx[f"{name}_out"] = res["out"][::step]
        fx[f"{name}_out_rms"] = np.array(np.sqrt(np.mean(res["out"].astype(np.float64) ** 2)))
        for k, v in pool_digests(spec).items():
            fx[f"{name}_sha_{k}"] = np.array(v)
        print(name, "done")
    path = os.path.join(HERE, "golden_prefill.npz")
    np.savez_compressed(path, **fx)
    print("wrote", path, os.path.getsize(path), "bytes")


def main_dense():
    """Gemma-4's dense MLP (d_model 2816, inner width 2112, Q4_K gate / up, Q5_0 down) through the
    reference's own build_ffn nodes (ref_dense_ffn) and, as a one-expert layer, through its MoE graph:
    the pools' digests, per-token digests of gate_up and of the GeGLU output, sampled output rows and
    the output's RMS."""
    from oracle.oracle import dense_as_expert_spec
    r = Ref()
    g, u, w = workload.dense_mlp_f32()
    gq, uq, wq = r.quantize(Q4_K, g), r.quantize(Q4_K, u), r.quantize(Q5_0, w)
    T, step = 64, 4
    x = workload.make_dense_input(T)
    dense = r.dense_ffn(x, Q4_K, gq, uq, Q5_0, wq, n_threads=8)
    res = r.moe_layer(dense_as_expert_spec(x, Q4_K, gq, uq, Q5_0, wq), n_threads=8,
                      want=("ids", "weights", "gate_up", "act"))
    assert np.array_equal(res["out"].view(np.uint32), dense.view(np.uint32))
    fx = {"sha_gate": np.array(sha(gq)), "sha_up": np.array(sha(uq)), "sha_down": np.array(sha(wq)),
          "gate_up_digest": token_digests(res["gate_up"], T), "act_digest": token_digests(res["act"], T),
          "out_digest": token_digests(dense, T), "out_rows": np.arange(0, T, step, dtype=np.int32),
          "out": dense[::step], "out_rms": np.array(np.sqrt(np.mean(dense.astype(np.float64) ** 2)))}
    path = os.path.join(HERE, "golden_dense.npz")
    np.savez_compressed(path, **fx)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    if "--dense" in sys.argv:
        main_dense()
    elif "--prefill" in sys.argv:
        main_prefill()
    elif "--types" in sys.argv:
        main_types()
    elif "--block" in sys.argv:
        main_block()
    else:
        main()
