#!/usr/bin/env python
"""Benchmark of the B200 quantized-FFN path (one JSON line on rank 0).

Default workload: a 48-layer stack of qwen3next-shaped
MoE feed-forward layers (hidden 2048, 512 experts, top-10, intermediate 512,
shared expert, gate/up Q4_K, down Q6_K), decode batch 32, each layer
x <- x + MoE(rms_norm(x)) as in the qwen3next block (llambda.lisp
L5738-5746).  Weights are synthetic (seeded generator, 50 GB at N=1), made on
the device.  With --gpus N the 512 experts of every layer are split over N
ranks (expert parallel, 512/N each), every rank holds the replicated
activations, and the per-layer partial outputs are summed inside each
layer's combine kernel over NVLink peer memory (--reduce peer, default; the
step is then replayed from one CUDA graph) or by an NCCL all-reduce per layer
(--reduce nccl).

Reported:
  value         tokens/s of the whole job, device-resident, CUDA events,
                max over ranks
  e2e           the same through the C ABI with host buffers: one
                llambda_cuda_moe_session_run per layer per step, host copies
                inside the timed region
  roofline      the dominant kernel, the gate/up pass: its algorithmic bytes
                (gate and up rows of every distinct routed expert, plus the
                shared expert's) / its duration from CUDA events the sessions
                record around it on the launch stream, against the measured
                HBM peak; the routed down pass and the whole layer beside it
  parity        layer 0's output of the measured run against a reference on
                the same bytes: the CPU oracle at N=1 (inside the CPU leg),
                a single-device session of the whole layer at N>1
  ep_breakdown  per-layer stage times (router + top-k, gate/up, routed down,
                shared down, combine with the cross-rank exchange), eager
                launches with events between the stages, rank 0 and max over
                ranks
  extra         the other north-star workloads at the same N, each with
                value, e2e, rooflines and parity: config-5 decode batch 1,
                config-5 prefill batch 2048, config-4 decode batch 64
  kernels       dense dequant-GEMV roofline (configs 1 and 2) timed alone
  cpu_baseline  the CPU oracle (a C restatement of the reference path, AVX2,
                all host threads) on a bounded sample, rank 0 only

--impl reference times the reference's CPU path (the oracle port; the Lisp
reference cannot run here: no SBCL, Windows-only) on the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAKS_PATH = os.path.join(ROOT, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
NOMINAL_HBM_GBS = 8000.0
# ncu DRAM traffic (read + write) of one config-5 b32 layer's gate/up launch
# and routed down launch on one GPU
GATE_UP_TRAFFIC_BYTES_N1 = 279_900_000
DOWN_TRAFFIC_BYTES_N1 = 202_500_000
# the same for the prefill path's tcgen05 GEMM launches at batch 2048 (ncu,
# 2-layer capture of the same workload: DRAM read + write of one launch)
PF_GATE_UP_TRAFFIC_BYTES = {2048: 719_400_000}
PF_DOWN_TRAFFIC_BYTES = {2048: 614_700_000}
# the same for one dense GEMV launch (workload, tokens)
DENSE_TRAFFIC_BYTES = {("config1", 1): 33_100_000, ("config2", 1): 438_600_000,
                       ("config2", 8): 444_700_000}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--prefill-min", type=int, default=0,
                   help="batch size from which MoE calls take the tcgen05 prefill path "
                        "(0: the library default)")
    p.add_argument("--arch", default="qwen3next", choices=["qwen3next", "nemotron_h_moe"],
                   help="layer of the stack: qwen3next (config 3 / 5, the headline) or "
                        "nemotron_h_moe (config 4)")
    p.add_argument("--layers", type=int, default=48)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-kernels", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the extra workloads (decode b1, prefill b2048, config-4 b64)")
    p.add_argument("--reduce", choices=["peer", "nccl"], default="peer",
                   help="N > 1: sum the ranks' partial outputs in the combine kernel over "
                        "peer memory, or with an NCCL all-reduce per layer")
    p.add_argument("--no-graph", action="store_true",
                   help="launch every layer from Python instead of replaying one CUDA graph")
    p.add_argument("--workload", default="stack",
                   choices=["stack", "config1", "config2", "q8_0", "q5_0"],
                   help="stack: the config-5 MoE decode stack (the headline line); "
                        "config1/config2: one dense dequant-GEMV of --batch tokens; "
                        "q8_0/q5_0: a 32-value-block GEMV at Nemotron-H width 2688")
    return p.parse_args()


def hbm_peak():
    try:
        with open(PEAKS_PATH) as f:
            v = float(json.load(f)["hbm_gbs"])
        return v, "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------- distributed

def dist_setup(n_gpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus and world > 1:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=datetime.timedelta(seconds=300))
    else:
        torch.cuda.set_device(0)
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(v, world):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------- workload

def build_stack(cfg, layers, rank, world, seed, max_tokens, torch, peer=False):
    """Device-resident synthetic layers; returns (sessions, owned bytes)."""
    import llambda_b200 as LB
    from llambda_b200 import configs as CF
    from llambda_b200 import ep
    E = cfg.experts
    roles = ep.layer_roles(rank, world, E, peer)
    eb, ee = roles["expert_range"]
    sessions, keep = [], []
    norm_w = torch.ones(cfg.hidden, dtype=torch.float32)  # post_attention_norm, unit weights
    for layer in range(layers):
        s = CF.layer_seed(seed, layer)
        tensors = {}
        for name, t, ne0, ne1, ne2, stream, scale in CF.moe_tensor_specs(cfg):
            unit = 4 if t == LB.TYPE_F32 else (144 if t == LB.TYPE_Q4_K else 210)
            per = CF.tensor_units(t, ne0, ne1, 1)
            if ne2 > 1:
                first, count = per * eb, per * (ee - eb)   # only this rank's experts
            else:
                first, count = 0, per
            buf = torch.empty(count * unit + 256, dtype=torch.uint8, device="cuda")
            LB.synth_fill_device(t, s, stream, first, count, scale, buf)
            keep.append(buf)
            if name in ("exp_probs_b.bias", "ffn_gate_inp_shexp"):
                tensors[name] = buf
            else:
                # the session indexes experts globally: point at expert 0
                tensors[name] = (t, ne0, ne1, ne2, _ShiftedPtr(buf, -(per * unit * eb) if ne2 > 1 else 0))
        sess = LB.MoeSession.create(
            cfg.arch, cfg.hidden, cfg.top_k, tensors, weight_scale=cfg.weight_scale,
            weights_norm=cfg.weights_norm, on_device=True, expert_range=(eb, ee),
            shared_here=roles["shared_here"], max_tokens=max_tokens,
            input_norm=norm_w.cuda(), norm_epsilon=1e-6, add_residual=roles["add_residual"])
        sessions.append(sess)
    torch.cuda.synchronize()
    return sessions, keep


class _ShiftedPtr:
    """A device pointer offset from a torch buffer (expert shards index from
    the global expert 0)."""

    def __init__(self, buf, offset):
        self.buf, self.offset = buf, offset

    def data_ptr(self):
        return self.buf.data_ptr() + self.offset


# ----------------------------------------------------------------- kernels alone

def fill_block32(torch, buf, type_tag, nblocks, seed, LB):
    """Random Q5_0 / Q8_0 blocks in device memory: random bytes, then each
    block's fp16 d set to |N(0,1)| * 0.02 (no Inf/NaN)."""
    bb = LB._native.BLOCK32_BYTES[type_tag]
    g = torch.Generator(device="cuda").manual_seed(seed)
    blocks = buf[: nblocks * bb].view(nblocks, bb)
    blocks.copy_(torch.randint(0, 256, (nblocks, bb), dtype=torch.uint8, device="cuda",
                               generator=g))
    d = (torch.randn(nblocks, device="cuda", generator=g).abs() * 0.02).half()
    blocks[:, 0:2] = d.view(torch.uint8).view(nblocks, 2)


def time_dense_gemv(torch, LB, cfg, tokens, reps=20):
    """Dense GEMV (configs 1/2, Q5_0/Q8_0 shapes) timed alone; rotates weight
    copies past L2."""
    from llambda_b200 import configs as CF
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    wb = cfg.weight_bytes
    copies = max(1, math.ceil(3 * l2 / wb))
    bufs, sessions = [], []
    for c in range(copies):
        b = torch.empty(wb + 256, dtype=torch.uint8, device="cuda")
        if cfg.type in (LB.TYPE_Q5_0, LB.TYPE_Q8_0):
            fill_block32(torch, b, cfg.type, wb // LB._native.BLOCK32_BYTES[cfg.type], c, LB)
        else:
            unit = 144 if cfg.type == LB.TYPE_Q4_K else 210
            LB.synth_fill_device(cfg.type, c, CF.S_DENSE, 0, wb // unit, cfg.dscale, b)
        bufs.append(b)
        sessions.append(LB.ProjectionSession.from_device(cfg.type, cfg.cols, cfg.rows, b))
    x = torch.randn(tokens, cfg.cols, device="cuda")
    y = torch.empty(tokens, cfg.rows, device="cuda")
    stream = torch.cuda.current_stream()
    for i in range(3):
        sessions[i % copies].run_device(x, y, tokens, stream)
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    ev[0].record(stream)
    for i in range(reps):
        sessions[i % copies].run_device(x, y, tokens, stream)
    ev[1].record(stream)
    torch.cuda.synchronize()
    ms = ev[0].elapsed_time(ev[1]) / reps
    nbytes = cfg.algorithmic_bytes(tokens)
    # the same calls replayed from one CUDA graph: the kernels back to back
    # without the host's launch gaps between them
    ms_graph = None
    try:
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side, capture_error_mode="thread_local"):
            for i in range(reps):
                sessions[i % copies].run_device(x, y, tokens, side)
        graph.replay()
        torch.cuda.synchronize()
        ev[0].record(stream)
        graph.replay()
        ev[1].record(stream)
        torch.cuda.synchronize()
        ms_graph = ev[0].elapsed_time(ev[1]) / reps
        del graph
    except Exception:  # a call that cannot be captured keeps the eager figure only
        torch.cuda.synchronize()
    for s in sessions:
        s.close()
    del bufs
    torch.cuda.empty_cache()
    out = {"workload": cfg.name, "tokens": tokens, "us_per_launch": ms * 1e3,
           "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / (ms * 1e-3) / 1e9,
           "weight_copies_rotated": copies}
    if ms_graph is not None:
        out["us_per_launch_graph"] = ms_graph * 1e3
        out["achieved_gbs_graph"] = nbytes / (ms_graph * 1e-3) / 1e9
    return out


_S_ACT = 1  # generator stream of the activations (llambda_b200.configs.S_ACT)


# ----------------------------------------------------------------- CPU side

class HostLayer:
    """Layer 0 of a stack on the host, for the CPU oracle: the oracle's copy
    of the generator writes the same bytes the device generator wrote.  Used
    only by the CPU leg (rank 0, N=1) and the reference arm."""

    def __init__(self, cfg, layer_seed):
        from oracle import oracle as O
        from oracle.layers import host_layer, oracle_layer
        self.O, self.cfg = O, cfg
        self.tensors = host_layer(cfg, layer_seed)
        self.L = oracle_layer(cfg, self.tensors, input_norm=np.ones(cfg.hidden, np.float32),
                              eps=1e-6, residual=True)

    def x(self, act_seed, tokens):
        return self.O.synth_f32(act_seed, _S_ACT, 0, tokens * self.cfg.hidden, 1.0).reshape(
            tokens, self.cfg.hidden)

    def forward(self, x):
        return self.O.moe_forward(self.L, x, x.shape[0], self.cfg.top_k)

    def time(self, x, steps, warmup):
        """Median seconds of one forward of x on all host cores."""
        self.O.set_workers(os.cpu_count() or 1)
        for _ in range(warmup):
            self.forward(x)
        ts = []
        for _ in range(steps):
            t0 = time.perf_counter()
            self.forward(x)
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)


def parity_record(out, sel, ref, sel_ref, against, bar):
    """max|out - ref| / max|ref| over the checked tokens, and the share of
    tokens whose selected experts equal the reference's (rank order)."""
    den = float(np.max(np.abs(ref)))
    err = float(np.max(np.abs(out.astype(np.float64) - ref))) / (den if den > 0 else 1.0)
    match = float(np.mean(np.all(sel == sel_ref, axis=1)))
    return {"against": against, "max_rel": err, "bar": bar, "selection_match": match,
            "checked_tokens": int(out.shape[0]), "ok": bool(err <= bar and match == 1.0)}


# ----------------------------------------------------------------- stack measurement

class Ctx:
    def __init__(self, args, torch, LB, CF, rank, world, local):
        self.args, self.torch, self.LB, self.CF = args, torch, LB, CF
        self.rank, self.world, self.local = rank, world, local
        self.peer = world > 1 and args.reduce == "peer"
        self.collective = world > 1 and not self.peer
        self.dispatch = False  # token dispatch attached to the open stack


def open_stack(ctx, cfg, max_tokens):
    t0 = time.time()
    sessions, keep = build_stack(cfg, ctx.args.layers, ctx.rank, ctx.world, ctx.args.seed,
                                 max_tokens, ctx.torch, peer=ctx.peer)
    ctx.dispatch = False
    if ctx.peer:  # each layer's combine sums every rank's partial over NVLink
        from llambda_b200 import ep
        keep.append(ep.attach_peer_reduction(sessions))
        if max_tokens >= ctx.LB.prefill_min_tokens() * ctx.world:
            # prefill batches: each rank passes its own tokens, which travel to
            # their experts' owners and back (the token dispatch)
            keep.append(ep.attach_token_dispatch(sessions,
                                                 (max_tokens + ctx.world - 1) // ctx.world))
            ctx.dispatch = True
    ref0 = None
    if ctx.world > 1 and ctx.rank == 0:
        # the whole layer 0 (every expert, shared expert, residual) as one
        # single-device session: the parity reference of the N > 1 runs
        r, rkeep = build_stack(cfg, 1, 0, 1, ctx.args.seed, max_tokens, ctx.torch)
        ref0 = (r[0], rkeep)
    return sessions, keep, ref0, time.time() - t0


def close_stack(ctx, sessions, keep, ref0):
    for s in sessions:
        s.close()
    if ref0 is not None:
        ref0[0].close()
    del keep
    ctx.torch.cuda.synchronize()
    ctx.torch.cuda.empty_cache()


def measure(ctx, cfg, sessions, ref0, B, clocks=False, e2e_on=True):
    """One workload (B tokens through the stack) on every rank: timed steps,
    stage breakdown, rooflines, layer-0 output, e2e.  Returns rank 0's record
    (other ranks return theirs too; only rank 0 prints)."""
    torch, LB, CF, args = ctx.torch, ctx.LB, ctx.CF, ctx.args
    world, rank, NL = ctx.world, ctx.rank, len(sessions)
    H = cfg.hidden
    x0 = torch.empty(B, H, device="cuda")
    LB.synth_fill_device(LB.TYPE_F32, args.seed, CF.S_ACT, 0, B * H, 1.0, x0)
    # token dispatch (N > 1, prefill batches): each rank runs its own slice of
    # the batch through the stack; otherwise every rank holds all B tokens
    sharded = world > 1 and getattr(ctx, "dispatch", False) and B >= LB.prefill_min_tokens() * world
    from llambda_b200 import ep as _ep
    t_lo, t_hi = _ep.token_slice(rank, world, B) if sharded else (0, B)
    x_full = x0
    x0 = x0[t_lo:t_hi].contiguous()
    Bl = t_hi - t_lo
    bufs = [torch.empty(Bl, H, device="cuda") for _ in range(2)]
    stream = torch.cuda.current_stream()
    if world > 1:
        import torch.distributed as dist

    def step(record=None):
        st = torch.cuda.current_stream()  # the capture stream while a graph records
        cur = x0
        for li, s in enumerate(sessions):
            out = bufs[li % 2]
            if record is not None:
                record[li][0].record(st)
            s.run_device(cur, out, Bl, stream=st)
            if ctx.collective:
                dist.all_reduce(out)
            if record is not None:
                record[li][1].record(st)
            cur = out
        return cur

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # one CUDA graph replays the whole stack step (not with an NCCL all-reduce
    # per layer, which stays outside graphs)
    graph = None
    if not ctx.collective and not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        torch.cuda.synchronize()
    for s in sessions:
        if s.status() != 0:
            raise SystemExit("device status reported a failure (weight sum or a bounded wait)")
    sampler = ClockSampler(ctx.local) if clocks else None
    if sampler:
        sampler.start()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clk = sampler.stop() if sampler else None
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    value = B / (ms * 1e-3)
    del graph

    # eager pass with events around every layer and between its stages
    layer_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(NL)]
    for s in sessions:
        s.time_kernels(True)
    step(layer_ev)
    torch.cuda.synchronize()
    layer_ms = [a.elapsed_time(b) for a, b in layer_ev]
    kern_ms = [s.kernel_ms() for s in sessions]
    stages = [s.kernel_breakdown() for s in sessions]
    for s in sessions:
        s.time_kernels(False)
    names = tuple(stages[0].keys())  # the combine's phases too at N > 1
    mean_us = [statistics.mean(st[n] for st in stages) * 1e3 for n in names]
    mine = torch.tensor(mean_us + [statistics.mean(layer_ms) * 1e3], dtype=torch.float64,
                        device="cuda")
    if world > 1:
        dist.all_reduce(mine, op=dist.ReduceOp.MAX)
    breakdown = {"rank0_us": {n: round(v, 2) for n, v in zip(names + ("layer",),
                                                               mean_us + [statistics.mean(layer_ms) * 1e3])},
                 "max_over_ranks_us": {n: round(v, 2) for n, v in zip(names + ("layer",),
                                                                      mine.tolist())},
                 "how": "eager launches, CUDA events between the stages of every layer, "
                        "mean over layers"}

    # routing of the timed steps (identical every step: same x0) -> algorithmic
    # bytes; layer 0's output and selection for the parity check
    sel = torch.empty(Bl, cfg.top_k, dtype=torch.int32, device="cuda")
    eb, ee = rank * cfg.experts // world, (rank + 1) * cfg.experts // world

    def gathered(t):  # every rank's rows, in token order (the token dispatch)
        if not sharded:
            return t
        parts = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(parts, t.contiguous())
        return torch.cat(parts)

    distinct, own_distinct = [], []
    cur, layer0 = x0, None
    for li, s in enumerate(sessions):
        out = bufs[li % 2]
        s.run_device(cur, out, Bl, sel_dev=sel, stream=stream)
        if ctx.collective:
            dist.all_reduce(out)
        ss = gathered(sel).cpu().numpy()
        distinct.append(int(np.unique(ss[ss >= 0]).size))
        own_distinct.append(int(np.unique(ss[(ss >= eb) & (ss < ee)]).size))
        if li == 0:
            layer0 = (gathered(out).cpu().numpy().copy(), ss.copy())
        cur = out
    torch.cuda.synchronize()
    prefill = B >= LB.prefill_min_tokens()
    parity = None
    if ref0 is not None:  # N > 1: rank 0 checks against the single-device layer
        rout = torch.empty(B, H, device="cuda")
        rsel = torch.empty(B, cfg.top_k, dtype=torch.int32, device="cuda")
        ref0[0].run_device(x_full, rout, B, sel_dev=rsel, stream=stream)
        torch.cuda.synchronize()
        parity = parity_record(layer0[0], layer0[1], rout.cpu().numpy().astype(np.float64),
                               rsel.cpu().numpy(),
                               f"single-device session of the whole layer 0 (rank 0, "
                               f"{'bf16 prefill' if prefill else 'fp32 decode'} kernels)"
                               + (", all ranks' token slices gathered" if sharded else ""),
                               2e-2 if prefill else 1e-3)

    from llambda_b200 import ep as _ep
    streams_shared = _ep.layer_roles(rank, world, cfg.experts, ctx.peer)["shared_here"]
    layer_bytes = [cfg.router_bytes() + (cfg.shared_bytes() if streams_shared else 0)
                   + u * cfg.expert_bytes() + 2 * 4 * B * H for u in own_distinct]
    peak, peak_kind = hbm_peak()
    gu_bytes = [u * cfg.gate_up_bytes() + (cfg.shared_gate_up_bytes() if streams_shared else 0)
                for u in own_distinct]
    gu_ms = statistics.mean(k[0] for k in kern_ms)
    dn_bytes = [u * cfg.down_bytes() for u in own_distinct]
    dn_ms = statistics.mean(k[1] for k in kern_ms)
    achieved = (sum(gu_bytes) / NL) / (gu_ms * 1e-3) / 1e9
    layer_gbs = (sum(layer_bytes) / NL) / (statistics.mean(layer_ms) * 1e-3) / 1e9
    n1_q = world == 1 and cfg is CF.CONFIG3
    if prefill:
        gu_name = ("pf_gemm_kernel<Q4_K, gate+up> (tcgen05 bf16 grouped GEMM, routed + shared)"
                   if cfg.has_gate else
                   "pf_gemm_kernel<Q4_K, up> (tcgen05 bf16 grouped GEMM, routed + shared)")
        dn_name = "pf_gemm_kernel<Q6_K, down> (tcgen05 bf16 grouped GEMM, routed + shared)"
        gu_traffic = PF_GATE_UP_TRAFFIC_BYTES.get(B) if n1_q else None
        dn_traffic = PF_DOWN_TRAFFIC_BYTES.get(B) if n1_q else None
    else:
        gu_name = ("moe_up_slab_kernel (gate/up pass, Q4_K)" if cfg.has_gate
                   else "moe_up_slab_kernel (up pass, Q4_K)")
        dn_name = "moe_down_slab_kernel (routed, Q6_K)"
        gu_traffic = GATE_UP_TRAFFIC_BYTES_N1 if n1_q and B == 32 else None
        dn_traffic = DOWN_TRAFFIC_BYTES_N1 if n1_q and B == 32 else None
    roofline = {"bound": "hbm", "kernel": gu_name,
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "algorithmic_bytes_per_launch": int(sum(gu_bytes) / NL),
                "launch_us_mean": round(gu_ms * 1e3, 2),
                # DRAM read+write bytes of one gate/up launch at N=1 (ncu capture)
                "traffic": gu_traffic,
                "down": {"kernel": dn_name,
                         "achieved": round((sum(dn_bytes) / NL) / (dn_ms * 1e-3) / 1e9, 1),
                         "frac": round((sum(dn_bytes) / NL) / (dn_ms * 1e-3) / 1e9 / peak, 4),
                         "launch_us_mean": round(dn_ms * 1e3, 2),
                         "traffic": dn_traffic},
                "layer": {"achieved": round(layer_gbs, 1), "frac": round(layer_gbs / peak, 4),
                          "algorithmic_bytes": int(sum(layer_bytes) / NL),
                          "us_mean": round(statistics.mean(layer_ms) * 1e3, 2)}}

    e2e = None
    if e2e_on and not args.no_e2e:
        # page-locked host buffers (the library copies them by DMA, no staging)
        pinned = [x0.cpu().pin_memory()] + [torch.empty((Bl, H), dtype=torch.float32,
                                                        pin_memory=True) for _ in range(2)]
        x_host = pinned[0].numpy()
        gloo = dist.new_group(backend="gloo") if ctx.collective else None
        host_bufs = [t.numpy() for t in pinned[1:]]  # run-into destinations

        def e2e_step():
            cur_h = x_host
            for li, s in enumerate(sessions):
                out_h = s.run_into(host_bufs[li % 2], cur_h)
                if ctx.collective:
                    t = torch.from_numpy(out_h)
                    dist.all_reduce(t, group=gloo)
                    out_h = t.numpy()
                cur_h = out_h
            return cur_h

        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier(world)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            e2e_step()
        dt = max_over_ranks((time.perf_counter() - t0) / args.steps, world)
        e2e = {"value": B / dt, "unit": "tokens/s",
               "h2d_bytes_per_step": NL * Bl * H * 4, "d2h_bytes_per_step": NL * Bl * H * 4,
               "path": "llambda_cuda_moe_session_run per layer from and into preallocated "
                       "page-locked host float buffers (the reference's run-into convention)"}
    # decode: rms-norm + router, top-k with routing, gate/up, routed down, shared
    # down (ranks that compute a share of the shared expert), combine.
    # prefill: rms-norm, router K slices, their sum, top-k with routing, gather,
    # tile plan, gate/up, down, combine.
    # token dispatch: rms-norm, router K slices, their sum, top-k, send,
    # group, copy, tile plan, gate/up, down, done, wait, combine.
    per_layer = (13 if sharded else 9) if prefill else 5 + (1 if streams_shared else 0)
    if sharded:
        breakdown["mode"] = f"token dispatch: {Bl} of the {B} tokens on each rank"
    return {"value": value, "ms_per_step": ms, "clocks": clk, "roofline": roofline, "e2e": e2e,
            "parity": parity, "ep_breakdown": breakdown, "layer0": layer0,
            "gpu_launches": per_layer * NL * args.steps, "prefill": prefill,
            "distinct_experts_per_layer_mean": round(statistics.mean(distinct), 1)}


def workload_name(cfg, CF, NL, B, prefill):
    phase = "prefill" if prefill else "decode"
    if cfg is CF.CONFIG3:
        return f"config5_qwen3next_moe_stack_{NL}L_{phase}_b{B}"
    return f"config4_nemotron_h_moe_stack_{NL}L_{phase}_b{B}"


# ----------------------------------------------------------------- main arms

def run_reference(args):
    """--impl reference: the reference CPU path (the oracle port) on all host
    cores.  Each step is a bounded sample: the step's tokens through layer 0
    of the stack (the 48 layers have the same shape); `value` scales the
    measured layer time to the whole stack, and ms_per_step is the time each
    measured step actually took."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from llambda_b200 import configs as CF
    cfg = CF.CONFIG3 if args.arch == "qwen3next" else CF.CONFIG4
    B, NL = args.batch, args.layers
    cores = os.cpu_count() or 1
    host = HostLayer(cfg, CF.layer_seed(args.seed, 0))
    x = host.x(args.seed, B)
    host.O.set_workers(cores)
    for _ in range(max(1, args.warmup)):
        host.forward(x)
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        host.forward(x)
        ts.append(time.perf_counter() - t0)
    per_layer = sum(ts) / len(ts)
    value = B / (per_layer * NL)
    phase = "prefill" if B >= 128 else "decode"
    sample = (f"{B} {phase} tokens through layer 0 of the {NL}-layer stack per step (all "
              f"{NL} layers share its shape), layer time x {NL} (CPU oracle: C restatement of "
              f"llambda.lisp L4338-4658/L5321-5426, AVX2+FMA, {cores} OpenMP threads)")
    line = {"impl": "reference", "metric": f"MoE FFN {phase} tokens/s", "value": value,
            "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": per_layer * 1e3, "layers_timed": 1,
            "stack_ms_per_step": per_layer * NL * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": workload_name(cfg, CF, NL, B, B >= 128), "batch": B,
                       "layers": NL, "experts": cfg.experts, "top_k": cfg.top_k,
                       "hidden": cfg.hidden},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "note": "SBCL path unavailable on this box; the timed reference is the oracle port"}
    print(json.dumps(line), flush=True)
    return 0


def run_dense(args, torch, LB, CF):
    """--workload config1|config2: one dense dequant-GEMV (rank 0 only) with
    --batch tokens; value = algorithmic HBM GB/s (weights + inputs + outputs)."""
    cfg = {"config1": CF.CONFIG1, "config2": CF.CONFIG2, "q8_0": CF.DENSE_Q8_0,
           "q5_0": CF.DENSE_Q5_0}[args.workload]
    r = time_dense_gemv(torch, LB, cfg, args.batch, reps=max(args.steps, 1))
    peak, peak_kind = hbm_peak()
    line = {"metric": "dequant-GEMV HBM GB/s", "value": round(r["achieved_gbs"], 1),
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": 3,
            "ms_per_step": round(r["us_per_launch"] / 1e3, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": r["workload"], "tokens": args.batch,
                       "l2": f"{r['weight_copies_rotated']} weight copies rotated past L2"},
            "roofline": {"bound": "hbm", "achieved": round(r["achieved_gbs"], 1), "peak": peak,
                         "unit": "GB/s", "frac": round(r["achieved_gbs"] / peak, 4),
                         "peak_kind": peak_kind,
                         "traffic": DENSE_TRAFFIC_BYTES.get((args.workload, args.batch))},
            "e2e": None, "cpu_baseline": None, "gpu_launches": 2 * max(args.steps, 1)}
    if "achieved_gbs_graph" in r:  # the same calls back to back from one CUDA graph
        line["roofline"]["graph"] = {"us_per_launch": round(r["us_per_launch_graph"], 2),
                                     "achieved": round(r["achieved_gbs_graph"], 1),
                                     "frac": round(r["achieved_gbs_graph"] / peak, 4)}
    print(json.dumps(line), flush=True)
    return 0


def compact(rec, cfg, CF, NL, B, peak):
    """The record of an extra workload inside the main line."""
    r = rec["roofline"]
    return {"metric": f"MoE FFN {'prefill' if rec['prefill'] else 'decode'} tokens/s",
            "workload": workload_name(cfg, CF, NL, B, rec["prefill"]),
            "value": round(rec["value"], 2), "unit": "tokens/s",
            "ms_per_step": round(rec["ms_per_step"], 4),
            "dtype": "bf16" if rec["prefill"] else "f32",
            "e2e": rec["e2e"],
            "roofline": {"kernel": r["kernel"], "achieved": r["achieved"], "peak": peak,
                         "frac": r["frac"], "launch_us_mean": r["launch_us_mean"],
                         "traffic": r["traffic"], "down": r["down"], "layer": r["layer"]},
            "parity": rec["parity"], "ep_breakdown": rec["ep_breakdown"],
            "gpu_launches": rec["gpu_launches"],
            "distinct_experts_per_layer_mean": rec["distinct_experts_per_layer_mean"]}


def run_ours(args):
    import torch
    import llambda_b200 as LB
    from llambda_b200 import configs as CF
    if args.workload in ("config1", "config2", "q8_0", "q5_0"):
        if LB.probe() != 1:
            raise SystemExit("CUDA backend unavailable: " + LB._native.last_error())
        return run_dense(args, torch, LB, CF)
    rank, world, local = dist_setup(args.gpus)
    if LB.probe() != 1:
        raise SystemExit("CUDA backend unavailable: " + LB._native.last_error())
    ctx = Ctx(args, torch, LB, CF, rank, world, local)
    cfg = CF.CONFIG3 if args.arch == "qwen3next" else CF.CONFIG4
    if args.prefill_min:
        LB.set_prefill_min_tokens(args.prefill_min)
    B, NL = args.batch, args.layers
    extras_on = (not args.no_extras and cfg is CF.CONFIG3 and B == 32)
    extra_q = [("config5_decode_b1", 1), ("config5_prefill_b2048", 2048)] if extras_on else []
    max_tokens = max([B] + [b for _, b in extra_q])
    sessions, keep, ref0, setup_s = open_stack(ctx, cfg, max_tokens)
    main = measure(ctx, cfg, sessions, ref0, B, clocks=True)
    extra_recs = []
    for name, b in extra_q:
        extra_recs.append((name, cfg, b, measure(ctx, cfg, sessions, ref0, b)))
    close_stack(ctx, sessions, keep, ref0)
    if extras_on:  # config 4: the nemotron_h_moe stack at decode batch 64
        c4 = CF.CONFIG4
        s4, k4, r4, _ = open_stack(ctx, c4, 64)
        extra_recs.append(("config4_decode_b64", c4, 64, measure(ctx, c4, s4, r4, 64)))
        close_stack(ctx, s4, k4, r4)
    peak, _ = hbm_peak()

    kernels = None
    cpu = None
    if rank == 0 and world == 1:
        if not args.no_kernels:
            kernels = {}
            try:
                kernels["config1_b1"] = time_dense_gemv(torch, LB, CF.CONFIG1, 1)
                kernels["config2_b1"] = time_dense_gemv(torch, LB, CF.CONFIG2, 1)
                kernels["config2_b8"] = time_dense_gemv(torch, LB, CF.CONFIG2, 8)
                for v in kernels.values():
                    v["frac"] = round(v["achieved_gbs"] / peak, 4)
                    if "achieved_gbs_graph" in v:
                        v["frac_graph"] = round(v["achieved_gbs_graph"] / peak, 4)
            except Exception as e:  # memory pressure
                kernels["error"] = str(e)
        if not args.no_cpu_baseline:
            # the CPU leg: the oracle times layer 0 of the stack on all host
            # cores and, as the checker, recomputes layer 0 of every measured
            # workload on the same bytes (the parity of the N=1 runs)
            cores = os.cpu_count() or 1
            host = HostLayer(cfg, CF.layer_seed(args.seed, 0))
            per_layer = host.time(host.x(args.seed, B), steps=3, warmup=1)
            cpu = {"value": B / (per_layer * NL), "unit": "tokens/s", "cores": cores,
                   "kind": "port",
                   "sample": f"{B} tokens through layer 0 of the stack per sample "
                             f"({per_layer * 1e3:.1f} ms), scaled to {NL} layers"}
            recs = [(cfg, B, main)] + [(c, b, r) for _, c, b, r in extra_recs]
            hosts = {id(cfg): host}
            for c, b, r in recs:
                if id(c) not in hosts:
                    hosts[id(c)] = HostLayer(c, CF.layer_seed(args.seed, 0))
                h = hosts[id(c)]
                ref, sel_ref, _ = h.forward(h.x(args.seed, b))
                r["parity"] = parity_record(
                    r["layer0"][0], r["layer0"][1], ref, sel_ref,
                    "CPU oracle, layer 0 of the stack, same synthetic bytes",
                    2e-2 if r["prefill"] else 1e-3)

    line = {"metric": f"MoE FFN {'prefill' if main['prefill'] else 'decode'} tokens/s",
            "value": round(main["value"], 2), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(main["ms_per_step"], 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" if main["prefill"] else "f32", "data": "synthetic",
            "config": {"workload": workload_name(cfg, CF, NL, B, main["prefill"]),
                       "batch": B, "layers": NL, "experts": cfg.experts, "top_k": cfg.top_k,
                       "hidden": cfg.hidden,
                       "parallelism": f"ep{world}" + ("-peer" if ctx.peer else
                                                      "-nccl" if world > 1 else ""),
                       "l2": "weights streamed per step exceed L2 (no flush needed)",
                       "setup_s": round(setup_s, 1)},
            "roofline": main["roofline"], "e2e": main["e2e"], "cpu_baseline": cpu,
            "clocks": main["clocks"], "parity": main["parity"],
            "ep_breakdown": main["ep_breakdown"],
            "gpu_launches": main["gpu_launches"] + sum(r["gpu_launches"]
                                                       for _, _, _, r in extra_recs),
            "distinct_experts_per_layer_mean": main["distinct_experts_per_layer_mean"]}
    if extra_recs:
        line["extra"] = {name: compact(r, c, CF, NL, b, peak) for name, c, b, r in extra_recs}
    if kernels is not None:
        line["kernels"] = kernels
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
