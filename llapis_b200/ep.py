"""Expert-parallel MoE layer over torch.distributed (one process per GPU, NCCL over NVLink).

Expert e lives on rank floor(e * G / E) (contiguous blocks); every rank holds the router and a
shard of the batch. One forward:

  1. route the local tokens (replicated router: moeb_layer_route);
  2. dispatch: for every (token, rank) pair with at least one of the token's top-k experts on that
     rank, send the token's row once, with its k expert ids (-1 where the expert lives elsewhere)
     and routing weights -- one all-to-all of fixed-size blocks;
  3. each rank runs the expert half on what it received (moeb_layer_forward_routed), which sums
     its own experts' weighted outputs per row in slot order;
  4. combine: all-to-all-v of those partial rows back to their source rank, which adds them in
     rank order.

This mirrors the reference's single-GPU arithmetic except for the final order of additions: the
reference adds all k weighted outputs in slot order, here the slot-ordered partial sums of each
rank are added in rank order (a difference of float rounding only).

Inside a Gemma-4 block (norms given), the source rank norms its tokens before step 1 (the router
input rms_norm(x) / sqrt(d) * ffn_gate_inp_s, the expert input rms_norm(x) * ffn_pre_norm_2) and the
combined rows after step 4 (rms_norm(out) * ffn_post_norm_2, gemma4.cpp:394-427): the output norm
needs every rank's partial rows, so it cannot run inside the experts' kernels as on one GPU.

Failure handling: with a Heartbeat, every rank announces each step in the process group's store
before it launches anything, and waits (bounded) for the others' announcements; a rank that left
(announced through Heartbeat.leave, or silent past the deadline) raises RankFailure on the others
before their next collective, so no rank blocks in a collective that can never complete. A
collective that fails anyway (the process group's own timeout) is reported as RankFailure too.

The data path is collectives of fixed size (rows out, with a small message of their ids and
weights, and partial rows back): each rank sends every rank a block of T rows, its own rows first
and absent rows (ids all -1) after them, so no split sizes cross to the host and a step needs no
host synchronisation. The
bookkeeping (which rows go where) is a handful of device-side index operations.
"""
from __future__ import annotations

import time
from datetime import timedelta

import numpy as np
import torch
import torch.distributed as dist


class RankFailure(RuntimeError):
    """A peer rank left or stopped answering; raised before this rank's next collective."""


class Heartbeat:
    """Per-step liveness through a torch.distributed Store (the process group's TCP store).

    beat(step) records this rank at `step`, then waits until every other rank has recorded it too,
    polling the store (a few ms apart) for at most deadline_s; a rank that called leave() fails the
    wait at once. Keys older than two steps are deleted, so the store stays small."""

    def __init__(self, store, rank: int, world: int, deadline_s: float = 30.0, prefix: str = "ep"):
        self.store, self.rank, self.world, self.deadline_s, self.prefix = store, rank, world, deadline_s, prefix

    def _key(self, step: int, r: int) -> str:
        return f"{self.prefix}/s{step}/r{r}"

    def _left(self, r: int) -> str:
        return f"{self.prefix}/left/r{r}"

    def beat(self, step: int) -> None:
        self.store.set(self._key(step, self.rank), b"1")
        others = [r for r in range(self.world) if r != self.rank]
        t_end = time.monotonic() + self.deadline_s
        pause = 1e-4
        while True:
            gone = [r for r in others if self.store.check([self._left(r)])]
            if gone:
                raise RankFailure(f"rank(s) {gone} left the expert-parallel group before step {step}")
            missing = [r for r in others if not self.store.check([self._key(step, r)])]
            if not missing:
                break
            if time.monotonic() > t_end:
                raise RankFailure(f"rank(s) {missing} did not reach step {step} within {self.deadline_s:.1f} s")
            time.sleep(pause)
            pause = min(2 * pause, 5e-3)
        if step >= 2:
            self.store.delete_key(self._key(step - 2, self.rank))

    def leave(self) -> None:
        """Announce that this rank takes no further steps (call between steps)."""
        self.store.set(self._left(self.rank), b"1")


def owner(e: torch.Tensor, n_expert: int, world: int) -> torch.Tensor:
    """Rank holding expert e: contiguous blocks of n_expert / world experts."""
    return (e * world) // n_expert


def local_experts(rank: int, n_expert: int, world: int) -> np.ndarray:
    e = np.arange(n_expert)
    return e[(e * world) // n_expert == rank].astype(np.int32)


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_splits, in_splits, group):
    dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)
    return out


def presence(ids: torch.Tensor, n_expert: int, world: int):
    """[world, T] bool: whether token t has at least one of its top-k experts on rank r, and the
    per-rank counts (device tensors: no host synchronisation)."""
    T, k = ids.shape
    dest = owner(ids.long(), n_expert, world)                                  # [T, k]
    present = torch.zeros((world, T), dtype=torch.bool, device=ids.device)
    # the value as a device tensor: a Python scalar would be copied from the host (not capturable)
    present.index_put_((dest.t().reshape(-1), torch.arange(T, device=ids.device).repeat(k)),
                       torch.ones((), dtype=torch.bool, device=ids.device))
    return dest, present, present.sum(dim=1)


def dispatch_plan(ids: torch.Tensor, n_expert: int, world: int, n_sent: int | None = None):
    """For local routing ids [T, k]: the (rank, token) pairs to send, rank-major then token order,
    the per-rank counts, and each sent row's ids with experts of other ranks masked to -1. With
    n_sent (the total, already known on the host) the compaction needs no host synchronisation."""
    dest, present, counts = presence(ids, n_expert, world)
    if n_sent is None:
        r_idx, t_idx = present.nonzero(as_tuple=True)                          # rank-major, tokens ascending
    else:
        nz = torch.nonzero_static(present, size=n_sent)
        r_idx, t_idx = nz[:, 0], nz[:, 1]
    sent_ids = torch.where(dest[t_idx] == r_idx[:, None], ids[t_idx], torch.full_like(ids[t_idx], -1))
    return r_idx, t_idx, counts, sent_ids


class EPMoE:
    """One layer's expert-parallel forward for this rank.

    route_fn(x) -> (ids [T, k] i32, w [T, k] f32) and experts_fn(rows, ids, w) -> partial rows are
    the local compute; by default they are a MoELayer's route / forward_routed (sm_100a kernels).
    Tests on CPU pass host functions instead, over a gloo group."""

    def __init__(self, n_expert: int, top_k: int, route_fn, experts_fn, group=None, norm_in=None, norm_out=None,
                 heartbeat: Heartbeat | None = None, encode_fn=None):
        """norm_in(x) -> (router input, expert input) and norm_out(rows) -> rows: the Gemma-4 block
        norms (None: the plain layer). heartbeat: per-step liveness checks (None: none).
        encode_fn(x) -> wire rows: what the dispatch sends for each expert-input row (None: the f32
        row); experts_fn then receives those rows."""
        self.E, self.k = n_expert, top_k
        self.route_fn, self.experts_fn = route_fn, experts_fn
        self.encode_fn = encode_fn
        self.norm_in, self.norm_out = norm_in, norm_out
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.heartbeat = heartbeat
        self.step = 0
        self.timing = {}

    @classmethod
    def from_layer(cls, layer, group=None, norms=None, heartbeat: Heartbeat | None = None, wire: str = "q8k"):
        """From a plain MoELayer (no norms of its own); with `norms` (BlockNorms) the forward is the
        Gemma-4 MoE block, its norms computed by moeb_rms_norm on the source rank. wire "q8k": the
        dispatch carries each row's Q8_K bytes (quantised once on the source rank: the bytes the
        experts consume, 3.5x smaller than f32 at d_model 2816, identical results); "f32": f32 rows."""
        norm_in = norm_out = None
        if norms is not None:
            from . import capi

            dev, d = layer.device, layer.host.d_model
            pre, rsc, post = (torch.from_numpy(np.asarray(getattr(norms, n), np.float32).reshape(d)).to(dev)
                              for n in ("pre_norm", "router_scale", "post_norm"))
            eps = float(norms.eps)
            c = float(np.float32(1.0) / np.sqrt(np.float32(d)))   # 1.0f / sqrtf((float) n_embd)

            def rms(v, w, scale):
                out = torch.empty_like(v)
                capi.check(capi.lib().moeb_rms_norm(v.data_ptr(), v.shape[0], d, w.data_ptr(), scale, eps,
                                                    out.data_ptr(), torch.cuda.current_stream(dev).cuda_stream))
                return out

            def norm_in(x):
                return rms(x, rsc, c), rms(x, pre, 1.0)

            def norm_out(rows):
                return rms(rows, post, 1.0)
        if wire == "q8k":
            return cls(layer.host.n_expert, layer.host.top_k, lambda x: layer.route(x)[1:],
                       lambda rows, ids, w: layer.forward_routed_q8k(rows, ids, w), group, norm_in, norm_out, heartbeat,
                       encode_fn=layer.quantize_q8k)
        assert wire == "f32", wire
        return cls(layer.host.n_expert, layer.host.top_k, lambda x: layer.route(x)[1:],
                   lambda rows, ids, w: layer.forward_routed(rows, ids, w), group, norm_in, norm_out, heartbeat)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        step = self.step
        self.step += 1
        if self.heartbeat is not None:
            self.heartbeat.beat(step)
        try:
            return self._forward(x)
        except RuntimeError as e:   # a collective that failed (peer gone, process-group timeout)
            if isinstance(e, RankFailure):
                raise
            raise RankFailure(f"expert-parallel step {step} failed: {e}") from e

    def _forward(self, x: torch.Tensor) -> torch.Tensor:
        G, d, k, dev = self.world, x.shape[1], self.k, x.device
        T = x.shape[0]
        if self.norm_in is not None:
            x_router, x = self.norm_in(x)
        else:
            x_router = x
        ids, w = self.route_fn(x_router)
        dest, present, _ = presence(ids, self.E, G)                        # [T, k], [G, T]
        # Fixed-capacity messages: each rank gets a block of T rows (its rows first, in token order,
        # then absent rows with every id -1), so the exchange needs no split sizes on the host and
        # the step runs without any host synchronisation.
        pos = torch.cumsum(present.to(torch.int32), dim=1) - 1             # slot of token t in rank r's block
        base = torch.arange(G, device=dev, dtype=torch.int64)[:, None] * T
        dump = G * T                                                       # one spare row takes the absent pairs
        idx = torch.where(present, base + pos.long(), torch.full_like(base + pos.long(), dump)).reshape(-1)
        mine = dest.t()[:, :, None] == torch.arange(G, device=dev)[None, None, :]   # [k, T, G]
        mine = mine.permute(2, 1, 0)                                                 # [G, T, k]
        sids = torch.where(mine, ids[None].expand(G, T, k), torch.full((G, T, k), -1, dtype=ids.dtype, device=dev))
        sw = torch.where(mine, w[None].expand(G, T, k), torch.zeros((G, T, k), dtype=w.dtype, device=dev))
        # rows: gathered straight into the send buffer through the inverse of idx (absent rows repeat
        # token 0; their ids are all -1, so nothing reads them); ids and weights: a small second message
        inv = torch.zeros(G * T + 1, dtype=torch.int64, device=dev)
        inv.index_put_((idx,), torch.arange(T, device=dev).repeat(G))
        wire = self.encode_fn(x) if self.encode_fn is not None else x
        sent_x = wire.index_select(0, inv[:G * T])
        meta = torch.empty((G * T + 1, 2 * k), dtype=torch.float32, device=dev)
        meta[:G * T, :k] = torch.full((), -1, dtype=torch.int32, device=dev).view(torch.float32)   # absent ids
        meta.index_put_((idx,), torch.cat([sids.to(torch.int32).view(torch.float32), sw.float()], dim=2).reshape(G * T, 2 * k))
        recv_x = torch.empty((G * T, wire.shape[1]), dtype=wire.dtype, device=dev)
        recv_meta = torch.empty((G * T, 2 * k), dtype=torch.float32, device=dev)
        _a2a(recv_x, sent_x, None, None, self.group)
        _a2a(recv_meta, meta[:G * T], None, None, self.group)
        recv_ids = recv_meta[:, :k].contiguous().view(torch.int32)
        recv_w = recv_meta[:, k:].contiguous()
        # the local experts' weighted sums per received row (absent rows give zeros)
        partial = self.experts_fn(recv_x, recv_ids, recv_w)
        back = torch.empty((G * T, d), dtype=x.dtype, device=dev)
        _a2a(back, partial.contiguous(), None, None, self.group)
        # combine in rank order
        out = torch.zeros_like(x)
        for r in range(G):
            got = back[(r * T + pos[r].clamp(min=0)).long()]
            out += torch.where(present[r][:, None], got, torch.zeros_like(got))
        if self.norm_out is not None:
            out = self.norm_out(out)
        return out

    __call__ = forward
