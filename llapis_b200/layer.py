"""Host-side MoE layer over libmoeb200.so: the HBM-resident precision classes, the residency mirror
and one call per layer forward (moeb_layer_forward), mirroring what LLapis's build_moe_ffn +
moe_dual hook compute for one Gemma-4 MoE layer (third_party/llama/src/llama-graph.cpp:1507-1851).

PyTorch provides device memory and streams only; all compute is the library's sm_100a kernels.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from . import capi
from .capi import IQ2_S, IQ4_NL, Q4_K, Q5_0

READY = 2  # moert_slot_state READY (moert/include/moert/policy.h:46)


@dataclass
class HostLayer:
    """Quantised weights of one layer in host memory (ggml layouts)."""
    d_model: int
    n_ff: int
    n_expert: int
    top_k: int
    w_router: np.ndarray                  # f32 [E, d]
    b_router: np.ndarray | None           # f32 [E]
    hot_ids: np.ndarray                   # i32 [K] experts held by the hot class, slot order
    hot_gu: np.ndarray | None             # u8 [K, 2nff, row]
    hot_down: np.ndarray | None           # u8 [K, d, row]
    cold_gu: np.ndarray | None            # u8 [E, 2nff, row]
    cold_down: np.ndarray | None
    hot_type_gu: int = Q4_K
    hot_type_down: int = Q5_0
    cold_type_gu: int = IQ2_S
    cold_type_down: int = IQ4_NL
    s_hot: np.ndarray | None = None       # f32 [K]
    s_cold: np.ndarray | None = None      # f32 [E]

    @property
    def n_slots(self) -> int:
        return int(len(self.hot_ids))

    def residency(self):
        """exp_slot / slot_exp / slot_state of the moe_dual mirror for this layout."""
        exp_slot = np.full(self.n_expert, -1, np.int32)
        exp_slot[self.hot_ids] = np.arange(self.n_slots, dtype=np.int32)
        return exp_slot, self.hot_ids.astype(np.int32), np.full(self.n_slots, READY, np.int32)

    def hot_mask(self) -> np.ndarray:
        m = np.zeros(self.n_expert, bool)
        m[self.hot_ids] = True
        return m

    def expert_bytes(self, e: int) -> int:
        """Weight bytes a forward reads for expert e (gate_up + down of its class)."""
        if self.hot_mask()[e]:
            return (2 * self.n_ff * capi.row_size(self.hot_type_gu, self.d_model)
                    + self.d_model * capi.row_size(self.hot_type_down, self.n_ff))
        return (2 * self.n_ff * capi.row_size(self.cold_type_gu, self.d_model)
                + self.d_model * capi.row_size(self.cold_type_down, self.n_ff))


@dataclass
class BlockNorms:
    """The norms around a Gemma-4 MoE block (third_party/llama/src/models/gemma4.cpp:394-427), f32
    [d_model] each: the experts see rms_norm(x) * pre_norm (ffn_pre_norm_2), the router
    rms_norm(x) / sqrt(d_model) * router_scale (ffn_gate_inp_s), and the block output is
    rms_norm(moe) * post_norm (ffn_post_norm_2)."""
    pre_norm: np.ndarray
    router_scale: np.ndarray
    post_norm: np.ndarray
    eps: float = 1e-6


def _dev(a, device):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(device)


def _ptr(t):
    return None if t is None else t.data_ptr()


class MoELayer:
    """One MoE layer resident on a CUDA device. With `norms` the forward is the whole Gemma-4 MoE
    block (moeb_layer_forward_gemma4): x is the block input and the output is normed."""

    def __init__(self, host: HostLayer, device: str | torch.device = "cuda", norms: BlockNorms | None = None,
                 pools: dict | None = None):
        """pools: device tensors already holding the weights (hot_gu, hot_down, cold_gu, cold_down,
        s_hot, s_cold; llapis_b200.loader fills them from files); the host arrays of those names
        are then not uploaded."""
        self.host = host
        self.norms = norms
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device(self.device.type, torch.cuda.current_device())
        capi.lib()
        with torch.cuda.device(self.device):
            capi.check(capi.lib().moeb_init())
        h = host
        exp_slot, slot_exp, slot_state = h.residency()
        weights = ("hot_gu", "hot_down", "cold_gu", "cold_down", "s_hot", "s_cold")
        self.t = dict(
            w_router=_dev(h.w_router.astype(np.float32), self.device),
            b_router=_dev(None if h.b_router is None else h.b_router.astype(np.float32), self.device),
            **{n: (pools.get(n) if pools is not None else _dev(getattr(h, n), self.device)) for n in weights},
            exp_slot=_dev(exp_slot, self.device) if h.n_slots else None,
            slot_exp=_dev(slot_exp, self.device) if h.n_slots else None,
            slot_state=_dev(slot_state, self.device) if h.n_slots else None,
        )
        t = self.t
        L = capi.Layer()
        L.d_model, L.n_ff, L.n_expert, L.top_k = h.d_model, h.n_ff, h.n_expert, h.top_k
        L.w_router, L.b_router = _ptr(t["w_router"]), _ptr(t["b_router"])
        L.hot = capi.Pool(h.hot_type_gu, h.hot_type_down, h.n_slots if t["hot_gu"] is not None else 0, 0,
                          _ptr(t["hot_gu"]), _ptr(t["hot_down"]), _ptr(t["s_hot"]))
        L.cold = capi.Pool(h.cold_type_gu, h.cold_type_down, h.n_expert if t["cold_gu"] is not None else 0, 0,
                           _ptr(t["cold_gu"]), _ptr(t["cold_down"]), _ptr(t["s_cold"]))
        L.exp_slot, L.slot_exp, L.slot_state = _ptr(t["exp_slot"]), _ptr(t["slot_exp"]), _ptr(t["slot_state"])
        self.c = L
        self.cn = None
        if norms is not None:
            for n in ("pre_norm", "router_scale", "post_norm"):
                t[n] = _dev(np.asarray(getattr(norms, n), np.float32).reshape(h.d_model), self.device)
            self.cn = capi.Norms(_ptr(t["pre_norm"]), _ptr(t["router_scale"]), _ptr(t["post_norm"]), float(norms.eps), 0)
        self._ws = None
        self._rws = None

    def prefill_path(self, n_tokens: int) -> bool:
        """Whether moeb_layer_forward runs n_tokens on the prefill (tensor-core GEMM) path."""
        return int(capi.lib().moeb_layer_path(C.byref(self.c), max(int(n_tokens), 1))) == 1

    def mid_path(self, n_tokens: int, kind: int = 0) -> bool:
        """Whether a prefill-path forward of n_tokens runs projection `kind` (0 gate_up, 1 down) on the
        mid-size kernels (int8 MMAs on the weight codes) rather than the tcgen05 GEMM: fewer routed
        pairs per expert than the library's bound (moeb_set_mid_max_pairs / _down) and a covered
        shape (tile and work-unit counts, mirrored from the library)."""
        h = self.host
        P = n_tokens * h.top_k
        lib = capi.lib()
        m = int(lib.moeb_set_mid_max_pairs(0) if kind == 0 else lib.moeb_set_mid_max_pairs_down(0))   # 1: off
        tiles = P // 128 + h.n_expert + 1
        chunk = 2 if kind == 0 else 4
        return (self.prefill_path(n_tokens) and m > 1 and P < m * h.n_expert and h.d_model % 256 == 0
                and h.n_ff % 32 == 0 and h.n_ff <= 1024 and tiles <= 512 and P // (8 * chunk) + tiles <= 1024)

    def launches(self, n_tokens: int) -> int:
        """Kernels one forward of n_tokens launches. Prefill path: router, top-k, then the routed half
        (routed_launches; with the block norms their kernel takes the activation quantiser's place).
        Decode path: one cooperative fused kernel per 8-token chunk."""
        if n_tokens <= 0:
            return 0
        return 2 + self.routed_launches(n_tokens) if self.prefill_path(n_tokens) else (n_tokens + 7) // 8

    def routed_launches(self, n_rows: int) -> int:
        """Kernels of the routed expert half (moeb_layer_forward_routed[_q8k]): dispatch, activation
        quantisation (or the Q8_K rows' unpacking), gate_up (tcgen05: B-image gather, Q4_K min-term
        kernel, GEMM; mid-size: operand images, GEMM), down (GeGLU images + GEMM on either path),
        combine."""
        if n_rows <= 0:
            return 0
        return 1 + 1 + (2 if self.mid_path(n_rows, 0) else 3) + 2 + 1

    def workspace_bytes(self, n_tokens: int) -> int:
        return int(capi.lib().moeb_layer_workspace_size(C.byref(self.c), n_tokens))

    def workspace(self, n_tokens: int) -> torch.Tensor:
        need = self.workspace_bytes(n_tokens)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, aux: dict | None = None,
                stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """x: f32 [T, d_model] on the layer's device. aux: optional dict of preallocated device tensors
        among logits [T,E], ids [T,k] i32, weights [T,k], counts [E], offsets [E+1], perm [T*k],
        gate_up [T*k, 2nff], down [T*k, d]."""
        assert x.dtype == torch.float32 and x.is_contiguous() and x.device == self.device
        T = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        ws = self.workspace(T)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        a = None
        if aux:
            a = capi.LayerAux(*[_ptr(aux.get(n)) for n, _ in capi.LayerAux._fields_])
        ap = C.byref(a) if a is not None else None
        if self.cn is not None:
            rc = capi.lib().moeb_layer_forward_gemma4(C.byref(self.c), C.byref(self.cn), x.data_ptr(), T,
                                                      out.data_ptr(), ap, ws.data_ptr(), ws.numel(), s.cuda_stream)
        else:
            rc = capi.lib().moeb_layer_forward(C.byref(self.c), x.data_ptr(), T, out.data_ptr(), ap, ws.data_ptr(),
                                               ws.numel(), s.cuda_stream)
        capi.check(rc)
        return out

    __call__ = forward

    def route(self, x: torch.Tensor, stream: torch.cuda.Stream | None = None):
        """Router logits, top-k ids and normalised weights of x (moeb_layer_route)."""
        assert x.dtype == torch.float32 and x.is_contiguous() and x.device == self.device
        T, h = x.shape[0], self.host
        logits = torch.empty((T, h.n_expert), dtype=torch.float32, device=self.device)
        ids = torch.empty((T, h.top_k), dtype=torch.int32, device=self.device)
        w = torch.empty((T, h.top_k), dtype=torch.float32, device=self.device)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        lib = capi.lib()
        need = int(lib.moeb_route_workspace_size(C.byref(self.c), T))
        if self._rws is None or self._rws.numel() < need:
            self._rws = torch.empty(need, dtype=torch.uint8, device=self.device)
        capi.check(lib.moeb_layer_route(C.byref(self.c), x.data_ptr(), T, logits.data_ptr(), ids.data_ptr(),
                                        w.data_ptr(), self._rws.data_ptr(), self._rws.numel(), s.cuda_stream))
        return logits, ids, w

    def forward_routed(self, x: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
                       stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """The expert half on given routing (moeb_layer_forward_routed): ids [n, k] i32 with -1 for
        experts held elsewhere, w [n, k] f32."""
        assert x.dtype == torch.float32 and x.is_contiguous() and x.device == self.device
        assert ids.dtype == torch.int32 and w.dtype == torch.float32 and ids.is_contiguous() and w.is_contiguous()
        n = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        if n == 0:
            return out
        need = int(capi.lib().moeb_routed_workspace_size(C.byref(self.c), n))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        capi.check(capi.lib().moeb_layer_forward_routed(C.byref(self.c), x.data_ptr(), n, ids.data_ptr(), w.data_ptr(),
                                                        out.data_ptr(), self._ws.data_ptr(), self._ws.numel(),
                                                        s.cuda_stream))
        return out

    def quantize_q8k(self, x: torch.Tensor, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """x's Q8_K rows (uint8 [T, d / 256 * 292], ggml block_q8_K), the bytes the experts consume."""
        assert x.dtype == torch.float32 and x.is_contiguous() and x.device == self.device
        T, d = x.shape
        out = torch.empty((T, capi.row_size(capi.Q8_K, d)), dtype=torch.uint8, device=self.device)
        if T:
            s = stream if stream is not None else torch.cuda.current_stream(self.device)
            capi.check(capi.lib().moeb_quantize_act(capi.Q4_K, x.data_ptr(), out.data_ptr(), T, d, s.cuda_stream))
        return out

    def forward_routed_q8k(self, xq: torch.Tensor, ids: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None,
                           stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        """forward_routed on rows already quantised to Q8_K (moeb_layer_forward_routed_q8k)."""
        assert xq.dtype == torch.uint8 and xq.is_contiguous() and xq.device == self.device
        assert ids.dtype == torch.int32 and w.dtype == torch.float32 and ids.is_contiguous() and w.is_contiguous()
        n = xq.shape[0]
        if out is None:
            out = torch.empty((n, self.host.d_model), dtype=torch.float32, device=self.device)
        if n == 0:
            return out
        need = int(capi.lib().moeb_routed_workspace_size(C.byref(self.c), n))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        capi.check(capi.lib().moeb_layer_forward_routed_q8k(C.byref(self.c), xq.data_ptr(), n, ids.data_ptr(),
                                                            w.data_ptr(), out.data_ptr(), self._ws.data_ptr(),
                                                            self._ws.numel(), s.cuda_stream))
        return out

    def device_error(self) -> int:
        s = torch.cuda.current_stream(self.device)
        return int(capi.lib().moeb_device_error(s.cuda_stream))


class FfnBlock:
    """The feed-forward part of a Gemma-4 MoE block (moeb_ffn_block_gemma4): out = the MoE block
    (`moe`, a MoELayer with its norms) + the dense MLP branch (`mlp`, a one-expert MoELayer with the
    dense norms ffn_norm / ffn_post_norm_1), the dense branch on a side stream when one is given."""

    def __init__(self, moe: MoELayer, mlp: MoELayer):
        assert moe.cn is not None and mlp.cn is not None, "both branches need their block norms"
        assert moe.device == mlp.device
        self.moe, self.mlp, self.device = moe, mlp, moe.device
        self._ws = None

    def workspace(self, n_tokens: int) -> torch.Tensor:
        need = int(capi.lib().moeb_ffn_block_workspace_size(C.byref(self.moe.c), C.byref(self.mlp.c), n_tokens))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.device)
        return self._ws

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None,
                side_stream: torch.cuda.Stream | None = None) -> torch.Tensor:
        assert x.dtype == torch.float32 and x.is_contiguous() and x.device == self.device
        T = x.shape[0]
        if out is None:
            out = torch.empty_like(x)
        ws = self.workspace(T)
        s = stream if stream is not None else torch.cuda.current_stream(self.device)
        capi.check(capi.lib().moeb_ffn_block_gemma4(C.byref(self.moe.c), C.byref(self.moe.cn), C.byref(self.mlp.c),
                                                    C.byref(self.mlp.cn), x.data_ptr(), T, out.data_ptr(),
                                                    ws.data_ptr(), ws.numel(), s.cuda_stream,
                                                    side_stream.cuda_stream if side_stream is not None else None))
        return out

    __call__ = forward
