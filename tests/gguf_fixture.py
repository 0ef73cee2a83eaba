"""TEST INFRASTRUCTURE — files for the expert-loading tests: a GGUF v3 writer (the layout of the
reference's gguf_write_to_file, third_party/llama/ggml/src/gguf.cpp:1400-1640; tests/test_load.py
checks the bytes against the reference's own writer) and a Gemma-4 layer written as a GGUF (the
cold class, router, block norms) plus an expert store (the hot class)."""
from __future__ import annotations

import struct

import numpy as np

# GGUF value types (gguf.h:53-68)
U32, I32, F32, STR = 4, 5, 6, 8


def _s(b: bytes) -> bytes:
    return struct.pack("<Q", len(b)) + b


def write_gguf(path: str, kvs, tensors, alignment: int = 32) -> None:
    """kvs: [(key, gguf type, value)]; tensors: [(name, ggml type, ne tuple, raw bytes)], written
    in order, each data block padded to `alignment`."""
    out = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(kvs)))
    for key, t, v in kvs:
        out += _s(key.encode()) + struct.pack("<I", t)
        out += {U32: lambda: struct.pack("<I", v), I32: lambda: struct.pack("<i", v),
                F32: lambda: struct.pack("<f", v), STR: lambda: _s(v.encode())}[t]()
    off = 0
    for name, typ, ne, data in tensors:
        out += _s(name.encode()) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}q", *ne)
        out += struct.pack("<IQ", typ, off)
        off += (len(data) + alignment - 1) // alignment * alignment
    out += bytes(-len(out) % alignment)
    for _, _, _, data in tensors:
        out += bytes(data) + bytes(-len(data) % alignment)
    with open(path, "wb") as f:
        f.write(out)


def layer_files(host, norms, gguf_path: str, store_index: str, il: int = 0, n_layers: int = 1,
                split_gate_up: bool = False, eps: float = 1e-6) -> None:
    """Writes `host` (a llapis_b200 HostLayer) as layer `il` of a Gemma-4 GGUF and its hot experts
    as an expert store (gate_up kind 0, down kind 1, the down scale as a kind-1 scale page)."""
    from llapis_b200.loader import write_store
    d, nff, E = host.d_model, host.n_ff, host.n_expert
    b = f"blk.{il}."
    kvs = [("general.architecture", STR, "gemma4"), ("gemma4.block_count", U32, n_layers),
           ("gemma4.embedding_length", U32, d), ("gemma4.expert_count", U32, E),
           ("gemma4.expert_used_count", U32, host.top_k), ("gemma4.expert_feed_forward_length", U32, nff),
           ("gemma4.attention.layer_norm_rms_epsilon", F32, eps)]
    ts = [(b + "ffn_gate_inp.weight", 0, (d, E), host.w_router.astype(np.float32).tobytes())]
    if host.b_router is not None:
        ts += [(b + "ffn_gate_inp.bias", 0, (E,), host.b_router.astype(np.float32).tobytes())]
    if norms is not None:
        ts += [(b + "ffn_gate_inp.scale", 0, (d,), norms.router_scale.astype(np.float32).tobytes()),
               (b + "pre_ffw_norm_2.weight", 0, (d,), norms.pre_norm.astype(np.float32).tobytes()),
               (b + "post_ffw_norm_2.weight", 0, (d,), norms.post_norm.astype(np.float32).tobytes())]
    gu = np.ascontiguousarray(host.cold_gu)
    if split_gate_up:
        ts += [(b + "ffn_gate_exps.weight", host.cold_type_gu, (d, nff, E), gu[:, :nff].tobytes()),
               (b + "ffn_up_exps.weight", host.cold_type_gu, (d, nff, E), gu[:, nff:].tobytes())]
    else:
        ts += [(b + "ffn_gate_up_exps.weight", host.cold_type_gu, (d, 2 * nff, E), gu.tobytes())]
    ts += [(b + "ffn_down_exps.weight", host.cold_type_down, (nff, d, E), np.ascontiguousarray(host.cold_down).tobytes())]
    if host.s_cold is not None:
        ts += [(b + "ffn_down_exps.scale", 0, (E,), host.s_cold.astype(np.float32).tobytes())]
    write_gguf(gguf_path, kvs, ts)
    pages = []
    for slot, e in enumerate(host.hot_ids.tolist()):
        pages.append(dict(layer=il, expert=e, kind=0, is_scale=0, quant_type=host.hot_type_gu, source_quant=host.hot_type_gu,
                          shape=(d, 2 * nff), data=np.ascontiguousarray(host.hot_gu[slot])))
        pages.append(dict(layer=il, expert=e, kind=1, is_scale=0, quant_type=host.hot_type_down,
                          source_quant=host.hot_type_down, shape=(nff, d), data=np.ascontiguousarray(host.hot_down[slot])))
        if host.s_hot is not None:
            pages.append(dict(layer=il, expert=e, kind=1, is_scale=1, quant_type=0, source_quant=0, shape=(1,),
                              data=np.ascontiguousarray(host.s_hot[slot:slot + 1].astype(np.float32))))
    pack = store_index[:-len(".experts.index")] + ".experts.pack"
    write_store(store_index, pack, pages, n_layers=n_layers, n_expert=E, n_embd=d, n_ff_exp=nff, pack_uuid=0x5eed)
