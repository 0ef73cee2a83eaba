"""Expert loading from files: one Gemma-4 MoE layer from a GGUF (router, block norms, the cold
class's stacked expert tensors) and the hot class's pages from an expert store
(experts.index / experts.pack), through libmoeb200.so's native GGUF directory, store reader and
file -> HBM loaders.

The tensors follow the reference's Gemma-4 loader (third_party/llama/src/models/gemma4.cpp:168-203,
llama-model.cpp:1117-1121): blk.<il>.ffn_gate_inp.weight [n_embd, E] f32, ffn_gate_inp.scale,
pre_ffw_norm_2.weight, post_ffw_norm_2.weight [n_embd] f32, ffn_gate_up_exps.weight
[n_embd, 2*n_ff, E] (or ffn_gate_exps + ffn_up_exps [n_embd, n_ff, E]), ffn_down_exps.weight
[n_ff, n_embd, E], optional ffn_down_exps.scale [E] and ffn_gate_inp.bias [E] (the router bias
build_moe_ffn adds to the logits, llama-graph.cpp:1544-1545). Store pages are addressed (layer, kind,
is_scale, expert) with kind 0 gate_up, 1 down (moert/include/moert/store.h:63-73).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import capi
from .capi import MoebError
from .layer import BlockNorms, HostLayer

KIND_GATE_UP, KIND_DOWN = 0, 1


def _lib():
    return capi.lib()


def _err(code: int, what: str) -> MoebError:
    return MoebError(code, f"{what}: {_lib().moeb_last_error().decode()}")


class Gguf:
    """A GGUF file's key/values and tensor directory (moeb_gguf_*)."""

    def __init__(self, path: str):
        self.path = path
        self.h = _lib().moeb_gguf_open(path.encode())
        if not self.h:
            raise _err(-1, "moeb_gguf_open")

    def close(self):
        if self.h:
            _lib().moeb_gguf_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:   # interpreter shutdown: the library binding may already be gone
            pass

    def tensor(self, name: str) -> capi.GgufTensor | None:
        t = capi.GgufTensor()
        return t if _lib().moeb_gguf_find_tensor(self.h, name.encode(), C.byref(t)) == 0 else None

    def u32(self, key: str, default=None):
        v = C.c_uint32()
        return int(v.value) if _lib().moeb_gguf_get_u32(self.h, key.encode(), C.byref(v)) == 0 else default

    def f32(self, key: str, default=None):
        v = C.c_float()
        return float(v.value) if _lib().moeb_gguf_get_f32(self.h, key.encode(), C.byref(v)) == 0 else default

    def str(self, key: str, default=None):
        buf = C.create_string_buffer(256)
        return buf.value.decode() if _lib().moeb_gguf_get_str(self.h, key.encode(), buf, 256) == 0 else default

    def read(self, name: str) -> np.ndarray:
        """The tensor's bytes (u8)."""
        t = self.tensor(name)
        if t is None:
            raise MoebError(-1, f"tensor {name} not in {self.path}")
        return np.fromfile(self.path, dtype=np.uint8, count=int(t.nbytes), offset=int(t.offset))


class Store:
    """An expert store reader (moert_store_reader_*)."""

    def __init__(self, index_path: str, expect_source_uuid: int = 0):
        self.h = _lib().moert_store_reader_open(index_path.encode(), expect_source_uuid)
        if not self.h:
            raise MoebError(-1, f"cannot open expert store {index_path}")

    def close(self):
        if self.h:
            _lib().moert_store_reader_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:   # interpreter shutdown: the library binding may already be gone
            pass

    def info(self, layer: int, kind: int, is_scale: int, expert: int):
        """(quant_type, nbytes, shape) of a page, or None when absent."""
        qt, nb, shape = C.c_int32(), C.c_uint64(), (C.c_int64 * 4)()
        if not _lib().moert_store_reader_page_info(self.h, layer, kind, is_scale, expert, C.byref(qt), C.byref(nb),
                                                   shape):
            return None
        return int(qt.value), int(nb.value), tuple(int(x) for x in shape)

    def page(self, layer: int, kind: int, is_scale: int, expert: int, verify: bool = True) -> np.ndarray:
        inf = self.info(layer, kind, is_scale, expert)
        if inf is None:
            raise MoebError(-1, f"store has no page (layer {layer}, kind {kind}, scale {is_scale}, expert {expert})")
        out = np.empty(inf[1], np.uint8)
        got = _lib().moert_store_reader_read(self.h, layer, kind, is_scale, expert, out.ctypes.data, out.size,
                                             int(verify))
        if got != out.size:
            raise MoebError(-1, f"store page read failed (layer {layer}, kind {kind}, expert {expert})")
        return out


def write_store(index_path: str, pack_path: str, pages, *, n_layers: int, n_expert: int, arch: str = "gemma4",
                n_embd: int = 0, n_ff_exp: int = 0, source_uuid: int = 0, pack_uuid: int = 0) -> None:
    """Writes an expert store (moert_store_writer_*). pages: iterable of dicts with layer, expert,
    kind, is_scale, quant_type, source_quant, shape (tuple), data (bytes-like)."""
    lib = _lib()
    info = capi.StoreInfo(0, source_uuid, arch.encode()[:15], n_layers, n_expert, n_embd, n_ff_exp, pack_uuid, 0)
    w = lib.moert_store_writer_open(index_path.encode(), pack_path.encode(), C.byref(info))
    if not w:
        raise MoebError(-1, f"cannot create expert store {index_path}")
    ok = True
    for p in pages:
        data = np.ascontiguousarray(np.frombuffer(p["data"], np.uint8) if not isinstance(p["data"], np.ndarray)
                                    else p["data"].view(np.uint8).reshape(-1))
        shape = (C.c_int64 * 4)(*p["shape"])
        ok = ok and bool(lib.moert_store_writer_add_page(w, p["layer"], p["expert"], p["kind"], p["is_scale"],
                                                         p["quant_type"], p.get("source_quant", p["quant_type"]),
                                                         p.get("flags", 0), shape, len(p["shape"]), data.ctypes.data,
                                                         data.size))
    if not lib.moert_store_writer_close(w) or not ok:
        raise MoebError(-1, f"writing expert store {index_path} failed")


def layer_tensor_names(il: int) -> dict:
    b = f"blk.{il}."
    return dict(router=b + "ffn_gate_inp.weight", router_bias=b + "ffn_gate_inp.bias", router_scale=b + "ffn_gate_inp.scale",
                pre_norm=b + "pre_ffw_norm_2.weight", post_norm=b + "post_ffw_norm_2.weight",
                gate_up=b + "ffn_gate_up_exps.weight", gate=b + "ffn_gate_exps.weight", up=b + "ffn_up_exps.weight",
                down=b + "ffn_down_exps.weight", down_scale=b + "ffn_down_exps.scale")


def _hparams(g: Gguf) -> dict:
    arch = g.str("general.architecture")
    if arch is None:
        raise MoebError(-1, f"{g.path}: no general.architecture")
    hp = dict(arch=arch, d_model=g.u32(f"{arch}.embedding_length"), n_expert=g.u32(f"{arch}.expert_count"),
              top_k=g.u32(f"{arch}.expert_used_count"), n_ff=g.u32(f"{arch}.expert_feed_forward_length"),
              eps=g.f32(f"{arch}.attention.layer_norm_rms_epsilon", 1e-6))
    missing = [k for k, v in hp.items() if v is None]
    if missing:
        raise MoebError(-1, f"{g.path}: missing hyperparameters {missing}")
    return hp


def _f32(g: Gguf, name: str, shape) -> np.ndarray:
    t = g.tensor(name)
    if t is None or t.type != 0:
        raise MoebError(-1, f"{g.path}: {name} missing or not f32")
    return g.read(name).view(np.float32).reshape(shape)


def _norms(g: Gguf, names: dict, d: int, eps: float) -> BlockNorms | None:
    if not all(g.tensor(names[n]) is not None for n in ("pre_norm", "router_scale", "post_norm")):
        return None
    return BlockNorms(pre_norm=_f32(g, names["pre_norm"], (d,)), router_scale=_f32(g, names["router_scale"], (d,)),
                      post_norm=_f32(g, names["post_norm"], (d,)), eps=eps)


def _cold_meta(g: Gguf, names: dict, hp: dict):
    """Types and per-expert byte strides of the stacked expert tensors (validating their shapes)."""
    d, nff, E = hp["d_model"], hp["n_ff"], hp["n_expert"]
    gu = g.tensor(names["gate_up"])
    if gu is not None:
        if tuple(gu.ne[:3]) != (d, 2 * nff, E):
            raise MoebError(-1, f"{names['gate_up']}: shape {tuple(gu.ne[:3])} != {(d, 2 * nff, E)}")
        gu_parts = [gu]
    else:
        gate, up = g.tensor(names["gate"]), g.tensor(names["up"])
        if gate is None or up is None:
            raise MoebError(-1, f"{g.path}: no gate_up (or gate + up) expert tensors for this layer")
        if tuple(gate.ne[:3]) != (d, nff, E) or tuple(up.ne[:3]) != (d, nff, E) or gate.type != up.type:
            raise MoebError(-1, "gate / up expert tensors disagree in shape or type")
        gu_parts = [gate, up]
    dn = g.tensor(names["down"])
    if dn is None or tuple(dn.ne[:3]) != (nff, d, E):
        raise MoebError(-1, f"{names['down']}: missing or shape != {(nff, d, E)}")
    return gu_parts, dn


def load_host_layer(gguf_path: str, il: int, store_index: str | None = None, hot_ids=()):
    """Layer `il` into host memory: (HostLayer, BlockNorms or None). The cold pool holds every
    expert from the GGUF's stacked tensors; the hot pool holds hot_ids (slot order) from the store."""
    g = Gguf(gguf_path)
    try:
        hp = _hparams(g)
        names = layer_tensor_names(il)
        d, nff, E = hp["d_model"], hp["n_ff"], hp["n_expert"]
        gu_parts, dn = _cold_meta(g, names, hp)
        parts = [g.read(names["gate_up"] if len(gu_parts) == 1 else n).reshape(E, -1)
                 for n in ([names["gate_up"]] if len(gu_parts) == 1 else [names["gate"], names["up"]])]
        cold_gu = np.concatenate(parts, axis=1).reshape(E, 2 * nff, -1)   # gate rows first
        cold_down = g.read(names["down"]).reshape(E, d, -1)
        s_cold = _f32(g, names["down_scale"], (E,)) if g.tensor(names["down_scale"]) is not None else None
        router = _f32(g, names["router"], (E, d))
        bias = _f32(g, names["router_bias"], (E,)) if g.tensor(names["router_bias"]) is not None else None
        norms = _norms(g, names, d, hp["eps"])
        cold_types = (gu_parts[0].type, dn.type)
    finally:
        g.close()
    hot_ids = np.asarray(list(hot_ids), np.int32)
    hot_gu = hot_down = s_hot = None
    hot_types = (capi.Q4_K, capi.Q5_0)
    if len(hot_ids):
        if store_index is None:
            raise MoebError(-1, "hot experts given without an expert store")
        st = Store(store_index)
        try:
            hot_types = (st.info(il, KIND_GATE_UP, 0, int(hot_ids[0]))[0], st.info(il, KIND_DOWN, 0, int(hot_ids[0]))[0])
            hot_gu = np.stack([st.page(il, KIND_GATE_UP, 0, int(e)) for e in hot_ids]).reshape(len(hot_ids), 2 * nff, -1)
            hot_down = np.stack([st.page(il, KIND_DOWN, 0, int(e)) for e in hot_ids]).reshape(len(hot_ids), d, -1)
            if st.info(il, KIND_DOWN, 1, int(hot_ids[0])) is not None:
                s_hot = np.concatenate([st.page(il, KIND_DOWN, 1, int(e)).view(np.float32) for e in hot_ids])
        finally:
            st.close()
    host = HostLayer(d_model=d, n_ff=nff, n_expert=E, top_k=hp["top_k"], w_router=router, b_router=bias,
                     hot_ids=hot_ids, hot_gu=hot_gu, hot_down=hot_down, cold_gu=cold_gu, cold_down=cold_down,
                     hot_type_gu=hot_types[0], hot_type_down=hot_types[1], cold_type_gu=cold_types[0],
                     cold_type_down=cold_types[1], s_hot=s_hot, s_cold=s_cold)
    return host, norms


def load_layer(gguf_path: str, il: int, store_index: str | None = None, hot_ids=(), device="cuda",
               use_norms: bool = True, stream=None):
    """Layer `il` straight into HBM: the cold pool from the GGUF's stacked expert tensors
    (moeb_load_file_range), the hot pool's slots from the store (moeb_load_store_pages); the small
    f32 tensors through host memory. Returns (MoELayer, bytes loaded into the pools)."""
    import torch

    from .layer import MoELayer
    lib = _lib()
    dev = torch.device(device)
    if dev.index is None:
        dev = torch.device(dev.type, torch.cuda.current_device())
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    g = Gguf(gguf_path)
    total = 0

    def check(n, what):
        if n < 0:
            raise _err(int(n), what)
        return int(n)
    try:
        hp = _hparams(g)
        names = layer_tensor_names(il)
        d, nff, E = hp["d_model"], hp["n_ff"], hp["n_expert"]
        gu_parts, dn = _cold_meta(g, names, hp)
        gu_row = int(gu_parts[0].nbytes) // (E * (2 * nff if len(gu_parts) == 1 else nff))
        cold_gu = torch.empty((E, 2 * nff, gu_row), dtype=torch.uint8, device=dev)
        if len(gu_parts) == 1:
            total += check(lib.moeb_load_file_range(gguf_path.encode(), gu_parts[0].offset, gu_parts[0].nbytes,
                                                    cold_gu.data_ptr(), s.cuda_stream), "gate_up load")
        else:   # separate gate and up tensors: each lands in a scratch pool, then rows are merged
            for j, t in enumerate(gu_parts):
                part = torch.empty((E, nff, gu_row), dtype=torch.uint8, device=dev)
                total += check(lib.moeb_load_file_range(gguf_path.encode(), t.offset, t.nbytes, part.data_ptr(),
                                                        s.cuda_stream), "gate / up load")
                cold_gu[:, j * nff:(j + 1) * nff].copy_(part)
        cold_down = torch.empty((E, d, int(dn.nbytes) // (E * d)), dtype=torch.uint8, device=dev)
        total += check(lib.moeb_load_file_range(gguf_path.encode(), dn.offset, dn.nbytes, cold_down.data_ptr(),
                                                s.cuda_stream), "down load")
        s_cold = (torch.from_numpy(_f32(g, names["down_scale"], (E,)).copy()).to(dev)
                  if g.tensor(names["down_scale"]) is not None else None)
        router = _f32(g, names["router"], (E, d)).copy()
        bias = _f32(g, names["router_bias"], (E,)).copy() if g.tensor(names["router_bias"]) is not None else None
        norms = _norms(g, names, d, hp["eps"]) if use_norms else None
        cold_types = (gu_parts[0].type, dn.type)
    finally:
        g.close()
    hot_ids = np.asarray(list(hot_ids), np.int32)
    pools = dict(cold_gu=cold_gu, cold_down=cold_down, s_cold=s_cold, hot_gu=None, hot_down=None, s_hot=None)
    hot_types = (capi.Q4_K, capi.Q5_0)
    if len(hot_ids):
        if store_index is None:
            raise MoebError(-1, "hot experts given without an expert store")
        st = Store(store_index)
        try:
            ids = np.ascontiguousarray(hot_ids)
            K = len(ids)
            for kind, key, rows in ((KIND_GATE_UP, "hot_gu", 2 * nff), (KIND_DOWN, "hot_down", d)):
                qt, nb, _ = st.info(il, kind, 0, int(ids[0]))
                buf = torch.empty((K, rows, nb // rows), dtype=torch.uint8, device=dev)
                total += check(lib.moeb_load_store_pages(st.h, il, kind, 0, ids.ctypes.data, K, buf.data_ptr(), nb, 1,
                                                         s.cuda_stream), "store page load")
                pools[key] = buf
                hot_types = (qt, hot_types[1]) if kind == KIND_GATE_UP else (hot_types[0], qt)
            if st.info(il, KIND_DOWN, 1, int(ids[0])) is not None:
                sc = torch.empty(K, dtype=torch.float32, device=dev)
                check(lib.moeb_load_store_pages(st.h, il, KIND_DOWN, 1, ids.ctypes.data, K, sc.data_ptr(), 4, 1,
                                                s.cuda_stream), "store scale load")
                pools["s_hot"] = sc
        finally:
            st.close()
    host = HostLayer(d_model=d, n_ff=nff, n_expert=E, top_k=hp["top_k"], w_router=router, b_router=bias,
                     hot_ids=hot_ids, hot_gu=None, hot_down=None, cold_gu=None, cold_down=None,
                     hot_type_gu=hot_types[0], hot_type_down=hot_types[1], cold_type_gu=cold_types[0],
                     cold_type_down=cold_types[1], s_hot=None, s_cold=None)
    return MoELayer(host, dev, norms=norms, pools=pools), total
