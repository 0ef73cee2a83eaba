"""ctypes binding of libmoeb200.so (include/moeb200.h, include/moert_cuda.h).

The library is the product: every compute entry runs sm_100a kernels and fails loudly (MoebError)
when it cannot — there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os

from . import build as _build

# ggml type ids (third_party/llama/ggml/include/ggml.h:390-432)
Q5_0, Q4_K, IQ4_NL, IQ2_S, Q8_0, Q8_K, IQ2_XXS = 6, 12, 20, 22, 8, 15, 16

ERRORS = {0: "OK", -1: "EINVAL", -2: "ENODEV", -3: "ECUDA", -4: "ESPACE", -5: "EDEVICE", -6: "ETYPE"}


class MoebError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"moeb error {ERRORS.get(code, code)}: {msg}")
        self.code = code


class Pool(C.Structure):
    _fields_ = [("type_gu", C.c_int32), ("type_down", C.c_int32), ("n", C.c_int32), ("_pad", C.c_int32),
                ("w_gu", C.c_void_p), ("w_down", C.c_void_p), ("s_down", C.c_void_p)]


class Layer(C.Structure):
    _fields_ = [("d_model", C.c_int32), ("n_ff", C.c_int32), ("n_expert", C.c_int32), ("top_k", C.c_int32),
                ("w_router", C.c_void_p), ("b_router", C.c_void_p), ("hot", Pool), ("cold", Pool),
                ("exp_slot", C.c_void_p), ("slot_exp", C.c_void_p), ("slot_state", C.c_void_p)]


class LayerAux(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("logits", "ids", "weights", "counts", "offsets", "perm", "gate_up", "down")]


class Norms(C.Structure):
    """moeb_norms: the Gemma-4 MoE block norms (device pointers to f32 [d_model])."""
    _fields_ = [("pre_norm", C.c_void_p), ("router_scale", C.c_void_p), ("post_norm", C.c_void_p),
                ("eps", C.c_float), ("_pad", C.c_int32)]


class StoreInfo(C.Structure):
    """moert_store_info (include/moert_store.h)."""
    _fields_ = [("format_version", C.c_uint32), ("source_uuid", C.c_uint64), ("arch", C.c_char * 16),
                ("n_layers", C.c_int32), ("n_expert", C.c_int32), ("n_embd", C.c_uint64), ("n_ff_exp", C.c_uint64),
                ("pack_uuid", C.c_uint64), ("record_count", C.c_uint64)]


class GgufTensor(C.Structure):
    """moeb_gguf_tensor (include/moeb200.h)."""
    _fields_ = [("type", C.c_int32), ("n_dims", C.c_int32), ("ne", C.c_int64 * 4), ("offset", C.c_uint64),
                ("nbytes", C.c_uint64)]


_lib = None

# name -> (restype, argtypes); every symbol include/*.h declares
SIGNATURES = {
    "moeb_init": (C.c_int, []),
    "moeb_last_error": (C.c_char_p, []),
    "moeb_version": (C.c_char_p, []),
    "moeb_device_error": (C.c_int32, [C.c_void_p]),
    "moeb_layer_workspace_size": (C.c_size_t, [C.POINTER(Layer), C.c_int32]),
    "moeb_layer_path": (C.c_int32, [C.POINTER(Layer), C.c_int32]),
    "moeb_layer_forward": (C.c_int, [C.POINTER(Layer), C.c_void_p, C.c_int32, C.c_void_p, C.POINTER(LayerAux),
                                     C.c_void_p, C.c_size_t, C.c_void_p]),
    "moeb_layer_forward_gemma4": (C.c_int, [C.POINTER(Layer), C.POINTER(Norms), C.c_void_p, C.c_int32, C.c_void_p,
                                            C.POINTER(LayerAux), C.c_void_p, C.c_size_t, C.c_void_p]),
    "moeb_rms_norm": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_float, C.c_float, C.c_void_p,
                                C.c_void_p]),
    "moeb_ffn_block_workspace_size": (C.c_size_t, [C.POINTER(Layer), C.POINTER(Layer), C.c_int32]),
    "moeb_ffn_block_gemma4": (C.c_int, [C.POINTER(Layer), C.POINTER(Norms), C.POINTER(Layer), C.POINTER(Norms),
                                        C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p,
                                        C.c_void_p]),
    "moeb_layer_forward_static": (C.c_int, [C.POINTER(Layer), C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p]),
    "moeb_set_prefill_min_tokens": (C.c_int32, [C.c_int32]),
    "moeb_set_mid_max_pairs": (C.c_int32, [C.c_int32]),
    "moeb_set_mid_max_pairs_down": (C.c_int32, [C.c_int32]),
    "moeb_layer_route": (C.c_int, [C.POINTER(Layer), C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
                                   C.c_void_p, C.c_size_t, C.c_void_p]),
    "moeb_route_workspace_size": (C.c_size_t, [C.POINTER(Layer), C.c_int32]),
    "moeb_routed_workspace_size": (C.c_size_t, [C.POINTER(Layer), C.c_int32]),
    "moeb_layer_forward_routed": (C.c_int, [C.POINTER(Layer), C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p,
                                            C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "moeb_layer_forward_routed_q8k": (C.c_int, [C.POINTER(Layer), C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p,
                                                C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "moeb_prefill_profile": (C.c_int, [C.c_int32]),
    "moeb_prefill_profile_read": (C.c_int, [C.POINTER(C.c_float), C.c_int32]),
    "moeb_bind_pools": (C.c_int, [C.c_int32, C.c_int32, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p, C.c_int32,
                                  C.c_int32]),
    "moeb_router_topk": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "moeb_dispatch": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p,
                                C.c_void_p]),
    "moeb_dequantize": (C.c_int, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p]),
    "moeb_quantize_act": (C.c_int, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p]),
    "moeb_quantize_weights": (C.c_size_t, [C.c_int32, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_int32]),
    "moeb_row_size": (C.c_size_t, [C.c_int32, C.c_int64]),
    "moeb_gguf_open": (C.c_void_p, [C.c_char_p]),
    "moeb_gguf_close": (None, [C.c_void_p]),
    "moeb_gguf_find_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(GgufTensor)]),
    "moeb_gguf_get_u32": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_uint32)]),
    "moeb_gguf_get_f32": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_float)]),
    "moeb_gguf_get_str": (C.c_int, [C.c_void_p, C.c_char_p, C.c_char_p, C.c_size_t]),
    "moeb_load_file_range": (C.c_int64, [C.c_char_p, C.c_uint64, C.c_uint64, C.c_void_p, C.c_void_p]),
    "moeb_load_store_pages": (C.c_int64, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_int32,
                                          C.c_void_p, C.c_uint64, C.c_int32, C.c_void_p]),
    "moert_store_probe": (C.c_int32, [C.c_char_p, C.POINTER(StoreInfo)]),
    "moert_store_verify": (C.c_int64, [C.c_char_p]),
    "moert_store_writer_open": (C.c_void_p, [C.c_char_p, C.c_char_p, C.POINTER(StoreInfo)]),
    "moert_store_writer_add_page": (C.c_int32, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                                C.c_int32, C.c_uint32, C.POINTER(C.c_int64), C.c_int32, C.c_void_p,
                                                C.c_uint64]),
    "moert_store_writer_close": (C.c_int32, [C.c_void_p]),
    "moert_store_fnv1a64": (C.c_uint64, [C.c_void_p, C.c_uint64, C.c_uint64]),
    "moert_store_reader_open": (C.c_void_p, [C.c_char_p, C.c_uint64]),
    "moert_store_reader_free": (None, [C.c_void_p]),
    "moert_store_reader_geometry": (C.c_int32, [C.c_void_p, C.POINTER(C.c_int32), C.POINTER(C.c_int32)]),
    "moert_store_reader_page_nbytes": (C.c_uint64, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
    "moert_store_reader_page_info": (C.c_int32, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                                 C.POINTER(C.c_int32), C.POINTER(C.c_uint64), C.POINTER(C.c_int64)]),
    "moert_store_reader_read": (C.c_uint64, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                             C.c_uint64, C.c_int32]),
    "moert_cuda_configure": (None, [C.c_void_p]),
    "moert_ffn_moe": (None, [C.c_void_p, C.c_void_p]),
    "moert_cuda_route_counts_enable": (C.c_int32, [C.c_int32, C.c_int32]),
    "moert_cuda_route_counts_fetch": (C.c_int32, [C.c_void_p, C.c_int32]),
    "moert_cuda_host_register_pinned": (C.c_int32, [C.c_void_p, C.c_uint64]),
    "moert_cuda_host_unregister": (None, [C.c_void_p]),
    "moert_cuda_host_register_mapped": (C.c_int32, [C.c_void_p, C.c_uint64]),
    "moert_cuda_host_map": (C.c_void_p, [C.c_void_p, C.c_uint64]),
    "moert_cuda_stats_get": (None, [C.c_void_p]),
    "moert_cuda_dir_init": (C.c_int32, [C.c_int32, C.c_int32, C.c_int32]),
    "moert_cuda_dir_async": (C.c_int32, [C.c_void_p, C.c_void_p, C.c_uint64]),
    "moert_cuda_dir_mark": (C.c_int64, []),
    "moert_cuda_dir_poll": (C.c_int64, [C.c_int32]),
    "moert_cuda_publish_h2d": (C.c_int32, [C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "moert_cuda_dir_stats_get": (None, [C.c_void_p]),
    "moert_cuda_dir_gate": (C.c_int64, [C.c_int32, C.c_int64]),
    "moert_cuda_set_hot_table": (None, [C.c_int32, C.c_int32, C.c_void_p, C.c_int32, C.c_int32]),
}


def lib(build_if_missing: bool = True) -> C.CDLL:
    """Loads libmoeb200.so (building it in-tree first when the sources changed)."""
    global _lib
    if _lib is None:
        path = _build.LIB
        if build_if_missing:
            try:
                path = _build.build()
            except (RuntimeError, OSError) as exc:
                if not os.path.exists(path):
                    raise MoebError(-2, f"libmoeb200.so is not built and cannot be built: {exc}") from exc
        if not os.path.exists(path):
            raise MoebError(-2, f"{path} missing: run `python -m llapis_b200.build`")
        _lib = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(_lib, name)
            fn.restype = res
            fn.argtypes = args
    return _lib


def check(code: int) -> None:
    if code != 0:
        raise MoebError(code, lib().moeb_last_error().decode())


def row_size(wtype: int, n: int) -> int:
    return int(lib().moeb_row_size(wtype, n))
