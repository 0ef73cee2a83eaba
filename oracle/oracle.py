"""TEST INFRASTRUCTURE — ctypes front-end for the two CPU oracles (see ``oracle/__init__.py``)."""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass, field

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_SO = os.path.join(HERE, "_ref", "libref_runner.so")
SIDECAR_SO = os.path.join(HERE, "_ref", "libsidecar_ref.so")
PORT_SO = os.path.join(HERE, "_build", "libmoe_oracle.so")

# ggml type ids (third_party/llama/ggml/include/ggml.h:390-432)
F32, F16, Q5_0, Q8_0, Q4_K, Q8_K, IQ2_XXS, IQ4_NL, IQ2_S = 0, 1, 6, 8, 12, 15, 16, 20, 22


class _Layer(C.Structure):
    _fields_ = [
        ("d_model", C.c_int32), ("n_ff", C.c_int32), ("n_expert", C.c_int32), ("top_k", C.c_int32),
        ("n_tokens", C.c_int32),
        ("x", C.c_void_p), ("w_router", C.c_void_p), ("b_router", C.c_void_p),
        ("n_slots", C.c_int32), ("exp_slot", C.c_void_p), ("slot_exp", C.c_void_p), ("slot_state", C.c_void_p),
        ("hot_type_gu", C.c_int32), ("hot_type_down", C.c_int32),
        ("hot_gu", C.c_void_p), ("hot_down", C.c_void_p), ("s_hot", C.c_void_p),
        ("cold_type_gu", C.c_int32), ("cold_type_down", C.c_int32),
        ("cold_gu", C.c_void_p), ("cold_down", C.c_void_p), ("s_cold", C.c_void_p),
        ("n_threads", C.c_int32),
        ("ids_in", C.c_void_p), ("gate_up_in", C.c_void_p),
        ("x_router", C.c_void_p), ("gelu_tanh", C.c_int32),
    ]


class _LayerOut(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("logits", "probs", "ids", "weights", "gate_up", "act", "down", "out")]


def _ptr(a):
    return None if a is None else a.ctypes.data


@dataclass
class LayerSpec:
    """Host-side (numpy) description of one MoE layer; mirrors ``oracle_layer``."""
    d_model: int
    n_ff: int
    n_expert: int
    top_k: int
    x: np.ndarray                       # f32 [T, d_model]
    w_router: np.ndarray                # f32 [E, d_model]
    b_router: np.ndarray | None = None  # f32 [E]
    n_slots: int = 0
    exp_slot: np.ndarray | None = None  # i32 [E]
    slot_exp: np.ndarray | None = None  # i32 [K]
    slot_state: np.ndarray | None = None  # i32 [K]
    hot_type_gu: int = Q4_K
    hot_type_down: int = Q5_0
    hot_gu: np.ndarray | None = None    # u8 [K, 2*n_ff, row]
    hot_down: np.ndarray | None = None  # u8 [K, d_model, row]
    s_hot: np.ndarray | None = None
    cold_type_gu: int = IQ2_S
    cold_type_down: int = IQ4_NL
    cold_gu: np.ndarray | None = None   # u8 [E, 2*n_ff, row]
    cold_down: np.ndarray | None = None
    s_cold: np.ndarray | None = None
    ids_in: np.ndarray | None = None      # i32 [T, k]: routing taken as given (port oracle only)
    gate_up_in: np.ndarray | None = None  # f32 [T*k, 2*n_ff]: gate_up taken as given (port oracle only)
    x_router: np.ndarray | None = None    # f32 [T, d_model]: router input when it differs from x
    gelu_tanh: bool = False               # port oracle: tanh-form GELU instead of the fp16 table
    keep: list = field(default_factory=list)

    @property
    def n_tokens(self) -> int:
        return int(self.x.shape[0])

    def to_c(self, n_threads: int = 1) -> _Layer:
        L = _Layer()
        L.d_model, L.n_ff, L.n_expert, L.top_k = self.d_model, self.n_ff, self.n_expert, self.top_k
        L.n_tokens = self.n_tokens
        arrs = dict(
            x=np.ascontiguousarray(self.x, np.float32),
            w_router=np.ascontiguousarray(self.w_router, np.float32),
            b_router=None if self.b_router is None else np.ascontiguousarray(self.b_router, np.float32),
            exp_slot=None if self.exp_slot is None else np.ascontiguousarray(self.exp_slot, np.int32),
            slot_exp=None if self.slot_exp is None else np.ascontiguousarray(self.slot_exp, np.int32),
            slot_state=None if self.slot_state is None else np.ascontiguousarray(self.slot_state, np.int32),
            hot_gu=None if self.hot_gu is None else np.ascontiguousarray(self.hot_gu),
            hot_down=None if self.hot_down is None else np.ascontiguousarray(self.hot_down),
            s_hot=None if self.s_hot is None else np.ascontiguousarray(self.s_hot, np.float32),
            cold_gu=None if self.cold_gu is None else np.ascontiguousarray(self.cold_gu),
            cold_down=None if self.cold_down is None else np.ascontiguousarray(self.cold_down),
            s_cold=None if self.s_cold is None else np.ascontiguousarray(self.s_cold, np.float32),
            ids_in=None if self.ids_in is None else np.ascontiguousarray(self.ids_in, np.int32),
            gate_up_in=None if self.gate_up_in is None else np.ascontiguousarray(self.gate_up_in, np.float32),
            x_router=None if self.x_router is None else np.ascontiguousarray(self.x_router, np.float32),
        )
        self.keep = list(arrs.values())
        for k, v in arrs.items():
            setattr(L, k, _ptr(v))
        L.gelu_tanh = int(self.gelu_tanh)
        L.n_slots = self.n_slots
        L.hot_type_gu, L.hot_type_down = self.hot_type_gu, self.hot_type_down
        L.cold_type_gu, L.cold_type_down = self.cold_type_gu, self.cold_type_down
        L.n_threads = n_threads
        return L


@dataclass
class BlockNorms:
    """The Gemma-4 MoE block norms (f32 [d_model] each) and the rms_norm epsilon."""
    pre_norm: np.ndarray       # ffn_pre_norm_2
    router_scale: np.ndarray   # ffn_gate_inp_s
    post_norm: np.ndarray      # ffn_post_norm_2
    eps: float = 1e-6


class _Oracle:
    prefix = ""

    def __init__(self, so: str):
        self.lib = C.CDLL(so)
        p = self.prefix
        f = self._fn
        self._row_size = f(p + "row_size", C.c_size_t, [C.c_int32, C.c_int64])
        self._deq = f(p + "dequantize_row", None, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64])
        self._qact = f(p + "quantize_act", None, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64])
        self._vdt = f(p + "vec_dot_type", C.c_int32, [C.c_int32])
        self._vdot = f(p + "vec_dot", C.c_float, [C.c_int32, C.c_int64, C.c_void_p, C.c_void_p])
        self._layer = f(p + "moe_layer", C.c_int, [C.POINTER(_Layer), C.POINTER(_LayerOut)])
        self._rms = f(p + "rms_norm", None, [C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_int64, C.c_int64,
                                             C.c_float])

    def _fn(self, name, res, args):
        fn = getattr(self.lib, name)
        fn.restype = res
        fn.argtypes = args
        return fn

    def row_size(self, t: int, n: int) -> int:
        return int(self._row_size(t, n))

    def dequantize(self, t: int, data: np.ndarray, n: int) -> np.ndarray:
        data = np.ascontiguousarray(data)
        out = np.empty(n, np.float32)
        self._deq(t, data.ctypes.data, out.ctypes.data, n)
        return out

    def vec_dot_type(self, wtype: int) -> int:
        return int(self._vdt(wtype))

    def quantize_act(self, vdt: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(self.row_size(vdt, x.size), np.uint8)
        self._qact(vdt, x.ctypes.data, out.ctypes.data, x.size)
        return out

    def vec_dot(self, wtype: int, n: int, w_row: np.ndarray, xq: np.ndarray) -> float:
        return float(self._vdot(wtype, n, np.ascontiguousarray(w_row).ctypes.data,
                                np.ascontiguousarray(xq).ctypes.data))

    def rms_norm(self, x: np.ndarray, eps: float, w: np.ndarray | None = None, s: float = 1.0) -> np.ndarray:
        """Row-wise ((x / sqrt(mean(x^2) + eps)) * s) * w of a 2-D f32 array (ggml_rms_norm, then
        ggml_scale when s != 1 and ggml_mul when w is given)."""
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty_like(x)
        wp = None if w is None else np.ascontiguousarray(w, np.float32)
        self._rms(x.ctypes.data, None if wp is None else wp.ctypes.data, s, out.ctypes.data, x.shape[0], x.shape[1],
                  eps)
        return out

    def gemma4_block(self, spec: LayerSpec, norms: "BlockNorms", n_threads: int = 1,
                     want=("logits", "ids", "weights", "gate_up", "act", "down")) -> dict:
        """The Gemma-4 MoE block around the layer (third_party/llama/src/models/gemma4.cpp:394-427):
        spec.x is the block input (attn_out); the experts see rms_norm(x) * pre_norm (:394-396),
        the router rms_norm(x) * (1 / sqrtf(d)) * router_scale (:399-402), and the output is
        rms_norm(moe) * post_norm (:423-425). Result keys as moe_layer plus "moe" (before the output
        norm), "x_expert" and "x_router". Each norm is one call of this oracle's rms_norm (the reference
        build runs the reference's own rms_norm, scale and mul nodes)."""
        eps = float(np.float32(norms.eps))
        c = float(np.float32(1.0) / np.sqrt(np.float32(spec.d_model)))   # 1.0f / sqrtf((float) n_embd)
        x_expert = self.rms_norm(spec.x, eps, norms.pre_norm)
        x_router = self.rms_norm(spec.x, eps, norms.router_scale, c)
        inner = LayerSpec(**{f: getattr(spec, f) for f in spec.__dataclass_fields__ if f != "keep"})
        inner.x, inner.x_router = x_expert, x_router
        res = self.moe_layer(inner, n_threads=n_threads, want=want)
        res["moe"] = res["out"]
        res["out"] = self.rms_norm(res["out"], eps, norms.post_norm)
        res["x_expert"], res["x_router"] = x_expert, x_router
        return res

    def moe_layer(self, spec: LayerSpec, n_threads: int = 1, want=("logits", "probs", "ids", "weights",
                                                                     "gate_up", "act", "down")) -> dict:
        T, E, k, d, nff = spec.n_tokens, spec.n_expert, spec.top_k, spec.d_model, spec.n_ff
        shapes = dict(logits=((T, E), np.float32), probs=((T, E), np.float32), ids=((T, k), np.int32),
                      weights=((T, k), np.float32), gate_up=((T * k, 2 * nff), np.float32),
                      act=((T * k, nff), np.float32), down=((T * k, d), np.float32), out=((T, d), np.float32))
        res = {n: np.zeros(*shapes[n]) for n in list(want) + ["out"]}
        o = _LayerOut()
        for n, a in res.items():
            setattr(o, n, a.ctypes.data)
        L = spec.to_c(n_threads)
        rc = self._layer(C.byref(L), C.byref(o))
        if rc != 1:
            raise RuntimeError(f"{type(self).__name__}.moe_layer failed ({rc})")
        return res


class Ref(_Oracle):
    """The reference's ggml-cpu path, built from the reference sources (oracle/_ref)."""
    prefix = "ref_"

    def __init__(self):
        super().__init__(REF_SO)
        self._quant = self._fn("ref_quantize", C.c_size_t, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64])
        self._quant_im = self._fn("ref_quantize_imatrix", C.c_size_t,
                                  [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p])
        self._gelu = self._fn("ref_gelu_table", C.c_uint16, [C.c_uint16])
        self.lib.ref_init()

    def quantize(self, t: int, w: np.ndarray, imatrix: np.ndarray | None = None) -> np.ndarray:
        """Reference quantiser ggml_quantize_chunk (ggml.c:7761) over rows of ``w`` (f32 [..., n]).
        IQ2_XXS needs an importance matrix; without one given, a uniform one is used."""
        w = np.ascontiguousarray(w, np.float32)
        n = w.shape[-1]
        nrow = w.size // n
        out = np.zeros(nrow * self.row_size(t, n), np.uint8)
        if imatrix is None and t == IQ2_XXS:
            imatrix = np.ones(n, np.float32)
        if imatrix is None:
            self._quant(t, w.ctypes.data, out.ctypes.data, nrow, n)
        else:
            im = np.ascontiguousarray(imatrix, np.float32)
            self._quant_im(t, w.ctypes.data, out.ctypes.data, nrow, n, im.ctypes.data)
        return out.reshape(*w.shape[:-1], self.row_size(t, n))

    def gelu_table(self) -> np.ndarray:
        return np.array([self._gelu(h) for h in range(1 << 16)], np.uint16)

    def dense_ffn(self, x, gu_type, w_gate, w_up, dn_type, w_down, n_threads: int = 4) -> np.ndarray:
        """The Gemma-4 dense MLP's FFN nodes (build_ffn, GELU / PAR): W_down geglu(W_gate x, W_up x)."""
        x = np.ascontiguousarray(x, np.float32)
        T, d = x.shape
        nff = w_gate.shape[0]
        fn = self._fn("ref_dense_ffn", C.c_int, [C.c_void_p, C.c_int64, C.c_int64, C.c_int64, C.c_int32, C.c_void_p,
                                                 C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int])
        out = np.zeros((T, d), np.float32)
        ws = [np.ascontiguousarray(w) for w in (w_gate, w_up, w_down)]
        assert fn(x.ctypes.data, T, d, nff, gu_type, ws[0].ctypes.data, ws[1].ctypes.data, dn_type, ws[2].ctypes.data,
                  out.ctypes.data, n_threads) == 1
        return out


def dense_as_expert_spec(x, gu_type, w_gate, w_up, dn_type, w_down, n_expert: int = 32) -> LayerSpec:
    """A dense GeGLU MLP as a one-expert MoE layer: a single hot slot holding [gate rows; up rows] and
    the down matrix, zero router weights with a bias that puts every token on expert 0, top-1 (its
    normalised weight is then exactly 1.0) and scale 1, so the layer output is the MLP's output."""
    T, d = x.shape
    nff = w_gate.shape[0]
    bias = np.full(n_expert, -1e4, np.float32)
    bias[0] = 0.0
    exp_slot = np.full(n_expert, -1, np.int32)
    exp_slot[0] = 0
    return LayerSpec(d, nff, n_expert, 1, x=x, w_router=np.zeros((n_expert, d), np.float32), b_router=bias, n_slots=1,
                     exp_slot=exp_slot, slot_exp=np.zeros(1, np.int32), slot_state=np.full(1, 2, np.int32),
                     hot_type_gu=gu_type, hot_type_down=dn_type,
                     hot_gu=np.concatenate([w_gate, w_up])[None], hot_down=np.asarray(w_down)[None],
                     s_hot=np.ones(1, np.float32))


class Port(_Oracle):
    """This repository's plain-C restatement of the path (oracle/moe_oracle.c)."""
    prefix = "oracle_"

    def __init__(self):
        if not os.path.exists(PORT_SO):
            build_port()
        super().__init__(PORT_SO)
        self._topk = self._fn("oracle_topk", None, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p])
        self._gelu = self._fn("oracle_gelu_table", C.c_uint16, [C.c_uint16])
        self._geglu = self._fn("oracle_geglu", None, [C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p])

    def topk(self, v: np.ndarray, k: int) -> np.ndarray:
        v = np.ascontiguousarray(v, np.float32)
        out = np.zeros(k, np.int32)
        self._topk(v.ctypes.data, v.size, k, out.ctypes.data)
        return out

    def gelu_table(self) -> np.ndarray:
        return np.array([self._gelu(h) for h in range(1 << 16)], np.uint16)

    def geglu(self, gate: np.ndarray, up: np.ndarray) -> np.ndarray:
        gate = np.ascontiguousarray(gate, np.float32)
        up = np.ascontiguousarray(up, np.float32)
        out = np.empty_like(gate)
        self._geglu(gate.size, out.ctypes.data, gate.ctypes.data, up.ctypes.data)
        return out


class Sidecar:
    """The reference's CPU sidecar (src/moe_sidecar.cpp, O2), built into oracle/_ref with
    oracle/sidecar_runner.cpp: per routed pair gate_up -> tanh GeGLU -> down on the host cores
    (ggml-cpu's vec_dot, the sidecar's own kernels for IQ2_XXS / IQ4_NL), at most 32 pairs a job."""

    def __init__(self, n_workers: int = 8):
        self.lib = C.CDLL(SIDECAR_SO)
        self.lib.sidecar_init.restype = C.c_int
        self.lib.sidecar_init.argtypes = [C.c_int]
        self.lib.sidecar_ffn.restype = C.c_int
        self.lib.sidecar_ffn.argtypes = [C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p,
                                         C.c_void_p, C.c_uint64, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_uint64,
                                         C.c_int32, C.c_void_p, C.c_void_p]
        if not self.lib.sidecar_init(n_workers):
            raise RuntimeError("sidecar init failed")
        self.n_workers = n_workers

    def ffn(self, x, pool_ids, pairs, k, gu, gu_type, dn, dn_type, d, nff):
        """Raw down outputs [len(pairs), d] of pairs p (token p // k) on pool entries pool_ids."""
        x = np.ascontiguousarray(x, np.float32)
        gu, dn = np.ascontiguousarray(gu), np.ascontiguousarray(dn)
        out = np.zeros((len(pairs), d), np.float32)
        for s in range(0, len(pairs), 32):
            ids = np.ascontiguousarray(pool_ids[s:s + 32], np.int32)
            cd = np.ascontiguousarray(pairs[s:s + 32], np.int32)
            # the job writes pair i's row at y[i * d]; its error path clears 4096 floats per pair
            y = np.zeros((len(ids), max(d, 4096)), np.float32)
            ns = C.c_int64()
            got = self.lib.sidecar_ffn(0, len(ids), ids.ctypes.data, cd.ctypes.data, k, x.shape[0], x.ctypes.data,
                                       gu.ctypes.data, gu[0].nbytes, gu_type, d, nff, dn.ctypes.data, dn[0].nbytes,
                                       dn_type, y.ctypes.data, C.byref(ns))
            if got != len(ids):
                raise RuntimeError(f"sidecar job computed {got} of {len(ids)} pairs")
            out[s:s + len(ids)] = y.reshape(-1)[:len(ids) * d].reshape(len(ids), d)
        return out

    def layer(self, spec: LayerSpec, ids: np.ndarray, weights: np.ndarray) -> np.ndarray:
        """The layer output with the given routing (O1's): each pair through the sidecar on its class's
        pool, then the down scale, the routing weight and the slot-order add, each product rounded
        (the reference's mul / mul / add-chain nodes)."""
        T, k, d = spec.n_tokens, spec.top_k, spec.d_model
        flat = ids.reshape(-1)
        hot = np.zeros(len(flat), bool)
        widx = flat.copy()
        if spec.n_slots and spec.exp_slot is not None:
            for p, e in enumerate(flat):
                s = int(spec.exp_slot[e])
                if 0 <= s < spec.n_slots and spec.slot_state[s] == 2 and spec.slot_exp[s] == e:
                    hot[p], widx[p] = True, s
        y = np.zeros((len(flat), d), np.float32)
        for cls in (True, False):
            sel = np.nonzero(hot == cls)[0]
            if not len(sel):
                continue
            gu, dn = (spec.hot_gu, spec.hot_down) if cls else (spec.cold_gu, spec.cold_down)
            tg, td = (spec.hot_type_gu, spec.hot_type_down) if cls else (spec.cold_type_gu, spec.cold_type_down)
            sc = spec.s_hot if cls else spec.s_cold
            yy = self.ffn(spec.x, widx[sel], sel, k, gu, tg, dn, td, d, spec.n_ff)
            if sc is not None:
                yy = (yy * sc[widx[sel]][:, None].astype(np.float32)).astype(np.float32)
            y[sel] = yy
        w = weights.reshape(-1).astype(np.float32)
        prod = (y * w[:, None]).astype(np.float32).reshape(T, k, d)
        out = prod[:, 0].copy()
        for j in range(1, k):
            out = (out + prod[:, j]).astype(np.float32)
        return out


def sidecar_available() -> bool:
    return os.path.exists(SIDECAR_SO)


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def port_available() -> bool:
    return os.path.exists(PORT_SO)


def build_port() -> None:
    subprocess.run(["make", "-s", "-C", HERE, "port"], check=True)
