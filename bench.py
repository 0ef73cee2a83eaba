"""Benchmark of the B200 MoE-FFN layer (router -> dispatch -> grouped gate_up -> GeGLU -> down ->
combine) on the configurations of BASELINE.json.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--impl ours|reference]

One JSON line on rank 0. A "step" is one layer forward over the config's tokens. `value` is
layer-tokens/s summed over ranks, device-timed with CUDA events on the launching stream (inputs
resident in HBM, L2 flushed between steps with a 256 MiB write that is not timed). `e2e` is the
same metric through the public API with the step's input copied from pinned host memory and the
output read back inside the timed region.

The metric is quoted at T=2048 and T=1: the default line is the T=2048 prefill layer
(prefill_t2048_q4k) and carries the T=1 decode layer (decode_t1_iq2s) as `secondary`. At N > 1
the default layer runs expert-parallel (experts sharded over the ranks, NCCL all-to-all dispatch
and combine) with 2048 tokens per rank (weak scaling; at N = 4 that is the T=8192 expert-parallel
config). Other decode configs do not shard: at N > 1 every rank runs an independent replica.
`--impl reference` times the reference's own CPU implementation (ggml-cpu built from the
reference sources, oracle/_ref) on this host's cores, with weights from the reference's own
quantiser; it never loads this repository's library.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

DEFAULT_CONFIG = "prefill_t2048_q4k"
SECONDARY_CONFIG = "decode_t1_iq2s"   # the metric's T=1 point, reported beside the default line
METRIC = "moe_layer_tokens_per_s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--config", default=DEFAULT_CONFIG)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-graph", action="store_true", help="launch eagerly instead of replaying a CUDA graph")
    p.add_argument("--cpu-sample-s", type=float, default=15.0, help="CPU baseline budget (seconds)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-secondary", action="store_true", help="skip the T=1 decode line of the default run")
    p.add_argument("--block-norms", action="store_true",
                   help="the whole Gemma-4 MoE block: pre / router-input / output rms_norms fused into the layer "
                        "(moeb_layer_forward_gemma4); input is the block input (attn_out)")
    p.add_argument("--ffn-block", action="store_true",
                   help="the Gemma-4 feed-forward block: the MoE block plus the dense MLP branch (d_model 2816, "
                        "inner width 2112) on a side stream (moeb_ffn_block_gemma4), against each branch alone "
                        "and both in turn")
    return p.parse_args()


def dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))


class Clocks:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(2)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


def measured_traffic(workload_name):
    """dram__bytes_read.sum + dram__bytes_write.sum of one launch of the dominant kernel, from the
    ncu capture summarised in profiles/ (None when no capture of this workload is committed)."""
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(workload_name)
    except (OSError, ValueError):
        return None


def reference_spec(host, x):
    from oracle import LayerSpec
    exp_slot, slot_exp, slot_state = host.residency()
    K = host.n_slots
    return LayerSpec(host.d_model, host.n_ff, host.n_expert, host.top_k, x=x, w_router=host.w_router,
                     b_router=host.b_router, n_slots=K, exp_slot=exp_slot if K else None,
                     slot_exp=slot_exp if K else None, slot_state=slot_state if K else None, hot_gu=host.hot_gu,
                     hot_down=host.hot_down, s_hot=host.s_hot, cold_gu=host.cold_gu, cold_down=host.cold_down,
                     s_cold=host.s_cold)


def time_reference(host, x, warmup, steps, budget_s, n_threads=None, norms=None):
    """The reference CPU path (oracle/_ref: the ggml-cpu MUL_MAT_ID graph of build_moe_ffn; with
    norms, also the block's rms_norm / scale / mul nodes) on this host's cores: `warmup` untimed
    forwards, then up to `steps` timed ones within `budget_s`."""
    from oracle import Ref, ref_available
    if not ref_available():
        return None
    r = Ref()
    spec = reference_spec(host, x)
    nt = n_threads or os.cpu_count() or 1

    def fwd():
        if norms is not None:
            r.gemma4_block(spec, norms, n_threads=nt, want=())
        else:
            r.moe_layer(spec, n_threads=nt, want=())
    for _ in range(max(1, warmup)):
        fwd()
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < max(1, steps) and (len(times) < 2 or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        fwd()
        times.append(time.perf_counter() - t0)
    value = x.shape[0] * len(times) / sum(times)
    return {"value": value, "unit": "tokens/s", "cores": nt, "kind": "reference",
            "sample": f"{len(times)} layer forwards of {x.shape[0]} tokens each, ggml-cpu O1 graph built from the "
                      f"reference sources, {nt} threads", "ms_per_forward": 1e3 * sum(times) / len(times)}


def time_sidecar(host, x, budget_s, n_threads=None):
    """The reference's CPU sidecar (O2: src/moe_sidecar.cpp, oracle/_ref/libsidecar_ref.so) for a
    decode batch (at most 4 tokens, 32 pairs a job): each routed pair's gate_up -> tanh GeGLU ->
    down on the host cores, then scale, weight and slot-order add. Routing is O1's, computed once
    outside the timed region. A second CPU baseline beside O1; never raises."""
    try:
        from oracle import Ref, Sidecar, ref_available, sidecar_available
        if not (ref_available() and sidecar_available()) or x.shape[0] > 4:
            return None
        nt = min(16, n_threads or os.cpu_count() or 1)
        spec = reference_spec(host, x)
        o1 = Ref().moe_layer(spec, n_threads=nt, want=("ids", "weights"))
        sc = Sidecar(nt)
        sc.layer(spec, o1["ids"], o1["weights"])   # warm
        times = []
        t_end = time.perf_counter() + budget_s
        while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 1000):
            t0 = time.perf_counter()
            sc.layer(spec, o1["ids"], o1["weights"])
            times.append(time.perf_counter() - t0)
        times.sort()
        med = times[len(times) // 2]
        return {"value": x.shape[0] / med, "unit": "tokens/s", "cores": nt, "kind": "reference",
                "sample": f"{len(times)} forwards of {x.shape[0]} tokens (median), the reference's moe_sidecar on "
                          f"{nt} threads; routing (O1) outside the timed region; tanh GeGLU",
                "ms_per_forward": 1e3 * med}
    except Exception as exc:   # a baseline must not take the bench line down with it
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}


def reference_layer_spec(cfg, x):
    """The config's layer for the reference arm, built without this repository's library: the same
    seeded f32 weights (llapis_b200.workload, numpy only) quantised by the reference's own
    ggml_quantize_chunk (oracle/_ref), in parallel over the host cores (ctypes releases the GIL),
    cached per expert on disk under its own key."""
    from concurrent.futures import ThreadPoolExecutor

    from llapis_b200 import workload
    from oracle import LayerSpec, Ref
    from oracle.oracle import IQ4_NL, Q4_K, Q5_0
    ref = Ref()
    E, d, nff = cfg.n_expert, cfg.d_model, cfg.n_ff
    hot = [int(e) for e in cfg.hot]
    is_hot = np.zeros(E, bool)
    is_hot[hot] = True
    ct = cfg.cold_gu_type

    def one(e):
        def make():
            gu, dn = workload.expert_f32(cfg, 0, e)
            ta, tb = (Q4_K, Q5_0) if is_hot[e] else (ct, IQ4_NL)
            return np.concatenate([ref.quantize(ta, gu).reshape(-1), ref.quantize(tb, dn).reshape(-1)])
        return workload._cached(f"ref-v1|{cfg.seed}|0|{e}|{d}|{nff}|{int(is_hot[e])}|{ct}", make)

    with ThreadPoolExecutor(max_workers=os.cpu_count() or 1) as ex:
        blobs = list(ex.map(one, range(E)))
    hgu, hdn = 2 * nff * ref.row_size(Q4_K, d), d * ref.row_size(Q5_0, nff)
    cgu, cdn = 2 * nff * ref.row_size(ct, d), d * ref.row_size(IQ4_NL, nff)
    K = len(hot)
    pools = {"hot_gu": [], "hot_down": [], "cold_gu": np.zeros((E, 2 * nff, cgu // (2 * nff)), np.uint8),
             "cold_down": np.zeros((E, d, cdn // d), np.uint8)}
    for e in hot:
        pools["hot_gu"].append(blobs[e][:hgu].reshape(2 * nff, -1))
        pools["hot_down"].append(blobs[e][hgu:hgu + hdn].reshape(d, -1))
    for e in range(E):
        if not is_hot[e]:
            pools["cold_gu"][e] = blobs[e][:cgu].reshape(2 * nff, -1)
            pools["cold_down"][e] = blobs[e][cgu:cgu + cdn].reshape(d, -1)
    n_cold = E - K
    exp_slot = np.full(E, -1, np.int32)
    exp_slot[hot] = np.arange(K, dtype=np.int32)
    b_router = None
    if cfg.bias_s is not None:
        b_router = (-cfg.bias_s * np.log1p(np.arange(E, dtype=np.float64))).astype(np.float32)
    return LayerSpec(d, nff, E, cfg.top_k, x=x, w_router=workload._normal((cfg.seed, 0, 1 << 20), (E, d), 0.02),
                     b_router=b_router, n_slots=K, exp_slot=exp_slot if K else None,
                     slot_exp=np.array(hot, np.int32) if K else None,
                     slot_state=np.full(K, 2, np.int32) if K else None,
                     hot_gu=np.stack(pools["hot_gu"]) if K else None,
                     hot_down=np.stack(pools["hot_down"]) if K else None,
                     s_hot=np.ones(K, np.float32) if K else None, cold_type_gu=ct,
                     cold_gu=pools["cold_gu"] if n_cold else None, cold_down=pools["cold_down"] if n_cold else None,
                     s_cold=np.ones(E, np.float32) if n_cold else None)


def run_reference(args):
    """--impl reference: the reference's CPU implementation of the path (oracle/_ref: ggml-cpu's
    MUL_MAT_ID graph of build_moe_ffn, built from the reference sources) on all host threads, each
    step a bounded sample (<= 256 tokens) of the config's batch. Rank 0 only under torchrun."""
    rank, _, world = dist_env()
    if rank != 0:
        return 0
    from oracle import Ref, ref_available
    if not ref_available():
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref (reference ggml-cpu build) missing"}))
        return 0
    from llapis_b200 import workload
    cfg = workload.CONFIGS[args.config]
    norms = workload.block_norms(cfg) if args.block_norms else None
    x = (workload.make_block_input(cfg) if norms else workload.make_input(cfg))[:256]
    spec = reference_layer_spec(cfg, x)
    r = Ref()
    nt = os.cpu_count() or 1

    def fwd():
        if norms is not None:
            r.gemma4_block(spec, norms, n_threads=nt, want=())
        else:
            r.moe_layer(spec, n_threads=nt, want=())
    for _ in range(max(1, args.warmup)):
        fwd()
    times = []
    t_end = time.perf_counter() + 120.0
    while len(times) < max(1, args.steps) and (len(times) < 2 or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        fwd()
        times.append(time.perf_counter() - t0)
    v = x.shape[0] * len(times) / sum(times)
    cb = {"value": v, "unit": "tokens/s", "cores": nt, "kind": "reference",
          "sample": f"{len(times)} layer forwards of {x.shape[0]} tokens each (a bounded sample of the {cfg.n_tokens}-token "
                    f"batch), ggml-cpu O1 graph built from the reference sources, weights from the reference "
                    f"quantiser, {nt} threads", "ms_per_forward": 1e3 * sum(times) / len(times)}
    line = {"metric": METRIC, "value": v, "unit": "tokens/s", "n_gpus": args.gpus, "steps": len(times),
            "warmup": args.warmup, "ms_per_step": cb["ms_per_forward"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "q8 int dot / f32", "data": "synthetic (seeded)",
            "config": {"workload": cfg.name, "n_tokens": cfg.n_tokens, "layers": 1,
                       "sample_tokens_per_step": int(x.shape[0]), "block_norms": norms is not None},
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))
    return 0


def local_shard(host, rank, world):
    """This rank's experts of a layer whose experts all sit in the hot class (expert-parallel)."""
    import dataclasses
    from llapis_b200.ep import local_experts
    mine = local_experts(rank, host.n_expert, world)
    assert host.n_slots == host.n_expert and np.array_equal(host.hot_ids, np.arange(host.n_expert))
    return dataclasses.replace(host, hot_ids=mine, hot_gu=host.hot_gu[mine], hot_down=host.hot_down[mine],
                               s_hot=host.s_hot[mine], cold_gu=None, cold_down=None, s_cold=None)


def run_ep(args, cfg, tokens_per_rank=None):
    """Expert-parallel prefill: experts sharded over the ranks, tokens split T/G per rank, NCCL
    all-to-all dispatch and combine (llapis_b200/ep.py). With tokens_per_rank the batch grows with
    the ranks (T = tokens_per_rank x G, weak scaling: the default T=2048 layer at N > 1); without,
    the config's T is split (strong scaling: the T=8192 expert-parallel config)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from llapis_b200 import capi, workload
    from llapis_b200.ep import EPMoE
    from llapis_b200.layer import MoELayer

    rank, local, world = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    else:
        dist.init_process_group("nccl", init_method="tcp://127.0.0.1:%d" % _free_port(), rank=0, world_size=1,
                                timeout=timedelta(seconds=300), device_id=dev)
    host = workload.build_layer(cfg)
    layer = MoELayer(local_shard(host, rank, world), dev)
    x_all = workload.make_input(cfg, n_tokens=tokens_per_rank * world if tokens_per_rank else None)
    T = x_all.shape[0]
    assert T % world == 0
    x_host = x_all[rank * (T // world):(rank + 1) * (T // world)]
    x = torch.from_numpy(x_host).to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    ep = EPMoE.from_layer(layer, group=None)
    s = torch.cuda.current_stream(dev)

    def timed(fn, steps):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for i in range(steps):
            flush.zero_()
            ev[i][0].record(s)
            fn()
            ev[i][1].record(s)
        torch.cuda.synchronize()
        return float(sum(a.elapsed_time(b) for a, b in ev))

    for _ in range(args.warmup):
        ep(x)
    torch.cuda.synchronize()
    dist.barrier()
    # one step as a CUDA graph (router, the exchange's bookkeeping, the three all-to-alls and both
    # expert halves): the fixed-size exchange needs no host synchronisation, so the whole step
    # captures; every rank captures at the same point (NCCL calls are recorded, not run)
    graph, graph_note = None, "eager launches"
    if not args.no_graph:
        try:
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(cap):
                for _ in range(3):
                    ep(x)
            torch.cuda.current_stream(dev).wait_stream(cap)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                ep(x)
            torch.cuda.synchronize()
            graph_note = "one CUDA graph per step (NCCL all-to-alls captured)"
        except RuntimeError as e:   # capture refused: time the eager step instead
            graph = None            # (the only reference: a graph holding NCCL calls must not outlive the group)
            graph_note = f"eager launches (graph capture failed: {str(e)[:120]})"
        dist.barrier()
    step = graph.replay if graph is not None else (lambda: ep(x))
    with Clocks(local) as clk:
        # keep the GPU loaded while the sampler takes its first readings: a FIXED number of steps,
        # the same on every rank (each step holds collectives, so ranks must take the same count)
        for _ in range(160):
            step()
        torch.cuda.synchronize()
        dev_ms = timed(step, args.steps)
    dist.barrier()
    # compute-only: the same local expert work on the rows this rank received, without communication
    recv_probe = {}

    orig = ep.experts_fn

    def experts_only():
        orig(recv_probe["x"], recv_probe["ids"], recv_probe["w"])

    ep.experts_fn = lambda rx, ri, rw: (recv_probe.update(x=rx, ids=ri, w=rw), orig(rx, ri, rw))[1]
    ep(x)
    torch.cuda.synchronize()
    ep.experts_fn = orig
    recv_rows = int(recv_probe["x"].shape[0])
    comp_ms = timed(experts_only, args.steps) if recv_rows else 0.0
    # kernel profile of this rank's expert half
    lib = capi.lib()
    names = ("router", "topk", "dispatch", "actq", "gather", "gate_up", "geglu", "down", "combine")
    buf = (C.c_float * len(names))()
    lib.moeb_prefill_profile(1)
    experts_only()
    capi.check(lib.moeb_prefill_profile_read(buf, len(names)))
    lib.moeb_prefill_profile(0)
    kernels_ms = dict(zip(names, buf[:]))
    # end to end: pinned host shard in, result out
    x_pin = torch.from_numpy(x_host).pin_memory()
    o_pin = torch.empty_like(x_pin).pin_memory()

    def e2e_step():
        xe = x_pin.to(dev, non_blocking=True)
        o_pin.copy_(ep(xe), non_blocking=True)

    e2e_ms = timed(e2e_step, args.steps)
    tot = torch.tensor([dev_ms, comp_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    # every reference to a graph holding NCCL calls goes before the process group does (else the exit
    # waits for good)
    del step, graph
    torch.cuda.synchronize()
    dev_ms, comp_ms, e2e_ms = tot.tolist()
    hbm, tflops_peak, peak_kind = measured_peaks()
    avg_ms = dev_ms / args.steps
    flops = workload.layer_flops(host, T)
    ach = flops / (avg_ms / 1e3) / 1e12
    if rank == 0:
        line = {
            "metric": METRIC, "value": T * args.steps / (dev_ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": avg_ms, "higher_is_better": True,
            "scaling": "weak" if tokens_per_rank else "strong", "vs_baseline": None,
            "dtype": "int8 x q4/q5 integer dots on fp16-exact tcgen05 MMAs / f32",
            "data": "synthetic (seeded N(0,0.02) weights quantised to ggml formats, bf16-valued N(0,1) activations)",
            "config": {"workload": cfg.name, "n_tokens": T, "layers": 1, "d_model": cfg.d_model,
                       "n_expert": cfg.n_expert, "top_k": cfg.top_k, "parallelism": f"ep{world}",
                       "experts_per_gpu": cfg.n_expert // world, "tokens_per_gpu": T // world,
                       "l2": "flushed between steps (256 MiB write, not timed)", "cuda_graph": graph_note,
                       "wire": "Q8_K rows out, f32 partial rows back"},
            "e2e": {"value": T * args.steps / (e2e_ms / 1e3), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(x_host.nbytes) * world, "d2h_bytes_per_step": int(x_host.nbytes) * world},
            # per step: router + top-k, the Q8_K quantisation of the sent rows, then the routed expert half
            "gpu_launches": (2 + 1 + layer.routed_launches(recv_rows)) * args.steps,
            "roofline": {"bound": "tensor", "achieved": ach, "peak": tflops_peak * world, "unit": "TFLOP/s",
                         "frac": ach / (tflops_peak * world), "traffic": None,
                         "peak_kind": f"{peak_kind} dense bf16 (burst) x {world} GPUs",
                         "scope": "whole job: layer FLOPs / step time",
                         "rank0_kernels_ms": kernels_ms},
            "exposed_comm_ms": avg_ms - comp_ms / args.steps, "compute_only_ms": comp_ms / args.steps,
            "cpu_baseline": None,
            "clocks": clk.summary(),
            "device_error": layer.device_error(),
        }
        print(json.dumps(line))
    dist.destroy_process_group()
    return 0


def run_stack(args, cfg):
    """a stack of n_layers MoE layers at T tokens on a residual stream
    (x + layer(rms_norm(x))). Every layer has its own seeded weights (seed, layer) and router."""
    import torch
    from llapis_b200 import workload
    from llapis_b200.layer import MoELayer

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    hosts = [workload.build_layer(cfg, layer=i) for i in range(cfg.n_layers)]
    layers = [MoELayer(h, dev) for h in hosts]
    host = hosts[0]
    x_host = workload.make_input(cfg)
    T = x_host.shape[0]
    x0 = torch.from_numpy(x_host).to(dev)
    bufs = [torch.empty_like(x0) for _ in range(2)]
    outs = torch.empty_like(x0)
    s = torch.cuda.current_stream(dev)
    for L in layers:
        L.workspace(T)

    normed = torch.empty_like(x0)

    def stack(x_in):
        # x_{l+1} = x_l + moe_l(rms_norm(x_l)): the pre-norm of a Gemma block (outside this path,
        # done here with torch) keeps every layer's input at unit scale
        x = x_in
        for i, L in enumerate(layers):
            torch.mul(x, torch.rsqrt(x.square().mean(dim=1, keepdim=True) + 1e-6), out=normed)
            L(normed, outs, stream=s)
            nxt = bufs[i & 1]
            torch.add(x, outs, out=nxt)
            x = nxt
        return x

    for _ in range(args.warmup):
        stack(x0)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with Clocks(0) as clk:
        for _ in range(5):
            stack(x0)
        torch.cuda.synchronize()
        for i in range(args.steps):
            ev[i][0].record(s)
            stack(x0)
            ev[i][1].record(s)
        torch.cuda.synchronize()
    dev_ms = float(sum(a.elapsed_time(b) for a, b in ev))
    x_pin = torch.from_numpy(x_host).pin_memory()
    o_pin = torch.empty_like(x_pin).pin_memory()
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps):
        ev2[i][0].record(s)
        o_pin.copy_(stack(x_pin.to(dev, non_blocking=True)), non_blocking=True)
        ev2[i][1].record(s)
    torch.cuda.synchronize()
    e2e_ms = float(sum(a.elapsed_time(b) for a, b in ev2))
    avg_ms = dev_ms / args.steps
    # algorithmic bytes of one pass: each layer streams its own routed unique experts (from its own
    # input in the stack) + router + activations
    stack_bytes = 0
    x = x0
    for i, L in enumerate(layers):
        torch.mul(x, torch.rsqrt(x.square().mean(dim=1, keepdim=True) + 1e-6), out=normed)
        ids = torch.empty((T, host.top_k), dtype=torch.int32, device=dev)
        L(normed, outs, aux={"ids": ids}, stream=s)
        stack_bytes += workload.algorithmic_bytes(hosts[i], ids.cpu().numpy(), T)
        x = x + outs
    hbm, tflops_peak, peak_kind = measured_peaks()
    ach = stack_bytes / (avg_ms / 1e3) / 1e9
    line = {
        "metric": METRIC, "value": T * args.steps / (dev_ms / 1e3), "unit": "tokens/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": avg_ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8 x q4/q5 integer dots on fp16-exact tcgen05 MMAs / f32",
        "data": f"synthetic ({cfg.n_layers} independently seeded layers, N(0,0.02) weights quantised to ggml "
                "formats; bf16-valued N(0,1) residual stream, RMS-normalised layer inputs)",
        "config": {"workload": cfg.name, "n_tokens": T, "layers": cfg.n_layers, "d_model": cfg.d_model,
                   "n_expert": cfg.n_expert, "top_k": cfg.top_k, "hot_experts": len(cfg.hot), "parallelism": "single",
                   "l2": f"inputs larger than L2 ({cfg.n_layers} layers of weights streamed per step)",
                   "path": path_label(layers[0], T),
                   "ms_per_layer": avg_ms / cfg.n_layers},
        "e2e": {"value": T * args.steps / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": int(x_host.nbytes),
                "d2h_bytes_per_step": int(x_host.nbytes)},
        "gpu_launches": (layers[0].launches(T)) * cfg.n_layers * args.steps,
        "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                     "traffic": None, "peak_kind": peak_kind,
                     "scope": f"whole stack: {stack_bytes} algorithmic bytes per step (each layer's routed "
                              "unique experts + router + activations)"},
        "cpu_baseline": None,
        "clocks": clk.summary(),
        "device_error": layers[0].device_error(),
    }
    print(json.dumps(line))
    return 0


def path_label(layer, T):
    """Which kernels a forward of T tokens runs (decode, or the prefill path's per-projection GEMMs)."""
    if not layer.prefill_path(T):
        return "decode (fused kernel)"
    kinds = ["mid-size int8 MMAs" if layer.mid_path(T, kind) else "tcgen05" for kind in (0, 1)]
    return f"prefill path: gate_up {kinds[0]}, down {kinds[1]}"


def _free_port():
    import socket
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    from llapis_b200 import workload as _wl
    if args.block_norms and (args.config.startswith("ep_") or _wl.CONFIGS[args.config].n_layers > 1):
        raise SystemExit("--block-norms covers the single-layer configs")
    if args.ffn_block:
        return run_ffn_block(args, _wl.CONFIGS[args.config])
    if args.config.startswith("ep_"):
        return run_ep(args, _wl.CONFIGS[args.config])
    if _wl.CONFIGS[args.config].n_layers > 1:
        return run_stack(args, _wl.CONFIGS[args.config])

    import torch
    import torch.distributed as dist

    from llapis_b200 import workload

    rank, local, world = dist_env()
    cfg = workload.CONFIGS[args.config]
    if world > 1 and cfg.name == DEFAULT_CONFIG:
        # the default layer at N > 1: expert-parallel, 2048 tokens per rank (weak scaling)
        return run_ep(args, cfg, tokens_per_rank=cfg.n_tokens)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    line = measure_layer(args, cfg, dev, rank, world, cpu_sample=not args.no_cpu_baseline)
    if cfg.name == DEFAULT_CONFIG and world == 1 and not args.no_secondary and not args.block_norms:
        sec = measure_layer(args, workload.CONFIGS[SECONDARY_CONFIG], dev, rank, world,
                            cpu_sample=not args.no_cpu_baseline)
        line["secondary"] = {k: sec[k] for k in ("metric", "value", "unit", "ms_per_step", "dtype", "config", "e2e",
                                                 "gpu_launches", "roofline", "cpu_baseline", "clocks", "device_error")}
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()
    return 0


def run_ffn_block(args, cfg):
    """The Gemma-4 feed-forward block at the config's T on one GPU: the MoE block (with its norms),
    the dense MLP branch alone, the block with both branches in turn on one stream, and the block
    with the dense branch on a side stream (concurrent with the MoE kernels). Device time per step
    (CUDA events on the launching stream, L2 flushed between steps, eager launches)."""
    import torch

    from llapis_b200 import workload
    from llapis_b200.layer import FfnBlock, MoELayer

    if cfg.n_layers > 1 or cfg.name.startswith("ep_"):
        raise SystemExit("--ffn-block covers the single-layer configs")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    moe = MoELayer(workload.build_layer(cfg), dev, norms=workload.block_norms(cfg))
    mlp = MoELayer(workload.build_dense_layer(), dev, norms=workload.dense_block_norms())
    blk = FfnBlock(moe, mlp)
    x = torch.from_numpy(workload.make_block_input(cfg)).to(dev)
    T = x.shape[0]
    out = torch.empty_like(x)
    s, side = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    variants = {"moe_block": lambda: moe(x, out, stream=s), "dense_mlp": lambda: mlp(x, out, stream=s),
                "sequential": lambda: blk(x, out, stream=s), "overlapped": lambda: blk(x, out, stream=s, side_stream=side)}
    res = {}
    with Clocks(0) as clk:
        for name, fn in variants.items():
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
            with torch.cuda.stream(s):
                for _ in range(max(3, args.warmup)):
                    flush.zero_()
                    fn()
                for i in range(args.steps):
                    flush.zero_()
                    ev[i][0].record(s)
                    fn()
                    ev[i][1].record(s)
            torch.cuda.synchronize()
            res[name] = float(np.mean([a.elapsed_time(b) for a, b in ev]))
    line = {"metric": "ffn_block_ms", "value": res["overlapped"], "unit": "ms", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": False, "dtype": "as the layer path",
            "data": "synthetic (seeded weights quantised to ggml formats, N(0,1) block input)",
            "config": {"workload": cfg.name, "n_tokens": T, "dense_n_ff": mlp.host.n_ff, "moe_path": path_label(moe, T),
                       "dense_path": path_label(mlp, T), "l2": "flushed between steps (256 MiB write, not timed)",
                       "cuda_graph": False},
            "ms": {k: round(v, 4) for k, v in res.items()},
            "overlap_saving_ms": round(res["sequential"] - res["overlapped"], 4),
            "tokens_per_s_overlapped": T / (res["overlapped"] * 1e-3), "clocks": clk.summary(),
            "device_error": moe.device_error()}
    print(json.dumps(line))
    return 0


def measure_layer(args, cfg, dev, rank, world, cpu_sample=True):
    """One single-GPU layer config (or one replica of it per rank): device-timed steps (CUDA-graph
    replay, L2 flushed between steps), the end-to-end steps through the public API, the roofline of
    the dominant kernel and the reference CPU baseline (rank 0, N=1). Returns the JSON line."""
    import torch
    import torch.distributed as dist

    from llapis_b200 import capi, workload
    from llapis_b200.layer import MoELayer

    local = dev.index
    host = workload.build_layer(cfg)
    norms = workload.block_norms(cfg) if args.block_norms else None
    layer = MoELayer(host, dev, norms=norms)
    x_host = workload.make_block_input(cfg) if norms else workload.make_input(cfg)
    T = x_host.shape[0]
    x = torch.from_numpy(x_host).to(dev)
    out = torch.empty_like(x)
    s = torch.cuda.Stream(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)   # > 126 MB L2

    # routing of this workload (for the algorithmic byte count)
    ids = torch.empty((T, host.top_k), dtype=torch.int32, device=dev)
    with torch.cuda.stream(s):
        layer(x, out, aux={"ids": ids}, stream=s)
    s.synchronize()
    alg_bytes = workload.algorithmic_bytes(host, ids.cpu().numpy(), T)
    launches_per_step = layer.launches(T)

    graph = None
    if not args.no_graph:
        layer.workspace(T)
        with torch.cuda.stream(s):
            for _ in range(3):
                layer(x, out, stream=s)
        s.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            layer(x, out, stream=s)
        s.synchronize()

    def step():
        if graph is not None:
            graph.replay()
        else:
            layer(x, out, stream=s)

    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            flush.zero_()
            step()
    s.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        # keep the GPU under this load until the sampler has a few readings (untimed)
        t_load = time.perf_counter()
        while len(clk.lines) < 3 and time.perf_counter() - t_load < 3.0:
            with torch.cuda.stream(s):
                for _ in range(50):
                    flush.zero_()
                    step()
            s.synchronize()
        with torch.cuda.stream(s):
            for i in range(args.steps):
                flush.zero_()
                ev[i][0].record(s)
                step()
                ev[i][1].record(s)
        s.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
    times_ms = [a.elapsed_time(b) for a, b in ev]
    dev_ms = float(sum(times_ms))

    # end to end through the public API: pinned host input -> layer -> host output, per step
    x_pin = torch.from_numpy(x_host).pin_memory()
    o_pin = torch.empty_like(x_pin).pin_memory()
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    x_e = torch.empty_like(x)
    o_e = torch.empty_like(x)
    with torch.cuda.stream(s):
        for i in range(args.warmup + args.steps):
            flush.zero_()
            if i >= args.warmup:
                ev2[i - args.warmup][0].record(s)
            x_e.copy_(x_pin, non_blocking=True)
            layer(x_e, o_e, stream=s)
            o_pin.copy_(o_e, non_blocking=True)
            if i >= args.warmup:
                ev2[i - args.warmup][1].record(s)
    s.synchronize()
    e2e_ms = float(sum(a.elapsed_time(b) for a, b in ev2))

    # prefill path: per-kernel CUDA-event durations on the launching stream (separate eager pass)
    prefill = layer.prefill_path(T)
    kernels_ms = None
    if prefill:
        lib = capi.lib()
        names = ("router", "topk", "dispatch", "actq", "gather", "gate_up", "geglu", "down", "combine")
        acc = np.zeros(len(names))
        buf = (C.c_float * len(names))()
        lib.moeb_prefill_profile(1)
        with torch.cuda.stream(s):
            for i in range(args.steps):
                flush.zero_()
                layer(x, out, stream=s)
                capi.check(lib.moeb_prefill_profile_read(buf, len(names)))
                acc += np.array(buf[:])
        lib.moeb_prefill_profile(0)
        kernels_ms = dict(zip(names, (acc / args.steps).tolist()))
    err = layer.device_error()

    tot = torch.tensor([dev_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    dev_ms, e2e_ms = tot.tolist()
    tokens = T * args.steps * world
    value = tokens / (dev_ms / 1e3)
    e2e = tokens / (e2e_ms / 1e3)
    hbm, tflops_peak, peak_kind = measured_peaks()
    avg_ms = dev_ms / args.steps
    achieved_gbs = alg_bytes / (avg_ms / 1e3) / 1e9
    if prefill:
        P = T * host.top_k
        kflops = {"gate_up": 2 * P * 2 * host.n_ff * host.d_model, "down": 2 * P * host.d_model * host.n_ff}
        top = max(kernels_ms, key=kernels_ms.get)
        if top in kflops:
            ach = kflops[top] / (kernels_ms[top] / 1e3) / 1e12
            roofline = {"bound": "tensor", "achieved": ach, "peak": tflops_peak, "unit": "TFLOP/s",
                        "frac": ach / tflops_peak, "traffic": measured_traffic(f"{cfg.name}:{top}"),
                        "peak_kind": f"{peak_kind} dense bf16 (burst); the kernel issues kind::f16 MMAs",
                        "kernel": top, "kernel_ms": kernels_ms[top],
                        "scope": f"pf_{top}_kernel, algorithmic FLOPs {kflops[top]} per launch "
                                 f"(2 x pairs x rows x K), CUDA events on the launching stream"}
        else:
            roofline = {"bound": "hbm", "achieved": None, "peak": hbm, "unit": "GB/s", "frac": None,
                        "traffic": None, "kernel": top, "kernel_ms": kernels_ms[top]}
        roofline["layer_tflops"] = workload.layer_flops(host, T) / (avg_ms / 1e3) / 1e12
        roofline["kernels_ms"] = kernels_ms
    else:
        roofline = {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm, "unit": "GB/s",
                    "frac": achieved_gbs / hbm, "traffic": measured_traffic(cfg.name), "peak_kind": peak_kind,
                    "scope": "whole layer forward (one cooperative fused kernel per 8-token chunk), "
                             f"algorithmic bytes {alg_bytes} per step"}

    cpu = None
    line = None
    if rank == 0 and world == 1 and cpu_sample:
        # a bounded sample: at most 256 tokens of the batch (the CPU cost per token is flat in T)
        cpu = time_reference(host, x_host[:256], 1, 1000, args.cpu_sample_s, norms=norms)
        if cpu is not None and norms is None and T <= 4:
            cpu["o2_sidecar"] = time_sidecar(host, x_host, min(5.0, args.cpu_sample_s))
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": avg_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int8 x q4/q5 integer dots on fp16-exact tcgen05 MMAs / f32" if prefill else "q8 int dot / f32",
            "data": "synthetic (seeded N(0,0.02) weights quantised to ggml formats, N(0,1) activations)",
            "config": {"workload": cfg.name, "n_tokens": T, "layers": 1, "d_model": cfg.d_model,
                       "n_expert": cfg.n_expert, "top_k": cfg.top_k, "hot_experts": len(cfg.hot),
                       "parallelism": f"replicas{world}" if world > 1 else "single",
                       "l2": "flushed between steps (256 MiB write, not timed)",
                       "path": path_label(layer, T), "block_norms": norms is not None,
                       "cuda_graph": graph is not None, "unique_experts": int(np.unique(ids.cpu().numpy()).size)},
            "e2e": {"value": e2e, "unit": "tokens/s", "h2d_bytes_per_step": int(x_host.nbytes),
                    "d2h_bytes_per_step": int(x_host.nbytes)},
            "gpu_launches": launches_per_step * args.steps,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "device_error": err,
        }
    del graph
    return line


if __name__ == "__main__":
    sys.exit(main())
