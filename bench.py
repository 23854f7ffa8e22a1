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


def distinct_experts(sel: np.ndarray, E: int) -> int:
    return int(np.unique(sel[sel >= 0]).size)


# ----------------------------------------------------------------- CPU side

def cpu_layer_sample(cfg, seed, tokens):
    """One host layer (oracle generator) and a timed CPU forward of `tokens`."""
    from oracle import oracle as O
    from tests.helpers import host_layer, oracle_layer
    tensors = host_layer(cfg, seed)
    L = oracle_layer(cfg, tensors, input_norm=np.ones(cfg.hidden, np.float32), eps=1e-6,
                     residual=True)
    x = O.synth_f32(seed, 1, 0, tokens * cfg.hidden, 1.0).reshape(tokens, cfg.hidden)
    return O, L, x, tensors


def time_cpu_stack(cfg, layers, batch, seed, steps, warmup):
    """Seconds per layer for `batch` tokens through one layer on all host cores."""
    O, L, x, keep = cpu_layer_sample(cfg, seed, batch)
    O.set_workers(os.cpu_count() or 1)
    for _ in range(warmup):
        O.moe_forward(L, x, batch, cfg.top_k)
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        O.moe_forward(L, x, batch, cfg.top_k)
        ts.append(time.perf_counter() - t0)
    per_layer = statistics.median(ts)
    tok_s = batch / (per_layer * layers)
    return tok_s, per_layer


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
    for s in sessions:
        s.close()
    del bufs
    torch.cuda.empty_cache()
    return {"workload": cfg.name, "tokens": tokens, "us_per_launch": ms * 1e3,
            "algorithmic_bytes": nbytes, "achieved_gbs": nbytes / (ms * 1e-3) / 1e9,
            "weight_copies_rotated": copies}


# ----------------------------------------------------------------- main arms

def run_reference(args):
    """--impl reference: the reference CPU path (oracle port) on host cores."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from llambda_b200 import configs as CF
    cfg = CF.CONFIG3
    sample_tokens = args.batch
    cores = os.cpu_count() or 1
    O, L, x, keep = cpu_layer_sample(cfg, args.seed, sample_tokens)
    O.set_workers(cores)
    for _ in range(max(1, args.warmup)):
        O.moe_forward(L, x, sample_tokens, cfg.top_k)
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.moe_forward(L, x, sample_tokens, cfg.top_k)
        ts.append(time.perf_counter() - t0)
    per_layer = sum(ts) / len(ts)
    value = sample_tokens / (per_layer * args.layers)
    sample = (f"{sample_tokens} decode tokens through 1 of the {args.layers} qwen3next layers per "
              f"step, time x {args.layers} layers (CPU oracle: C restatement of llambda.lisp "
              f"L4338-4658/L5321-5426, AVX2+FMA, {cores} OpenMP threads)")
    line = {"impl": "reference", "metric": "MoE FFN decode tokens/s", "value": value,
            "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": per_layer * args.layers * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"config5_qwen3next_moe_stack_{args.layers}L_decode_b{args.batch}",
                       "batch": args.batch, "layers": args.layers},
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
    print(json.dumps(line), flush=True)
    return 0


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
    cfg = CF.CONFIG3 if args.arch == "qwen3next" else CF.CONFIG4
    if args.prefill_min:
        LB.set_prefill_min_tokens(args.prefill_min)
    B, NL = args.batch, args.layers
    t_setup = time.time()
    peer = world > 1 and args.reduce == "peer"
    sessions, keep = build_stack(cfg, NL, rank, world, args.seed, max(B, 1), torch, peer=peer)
    if peer:  # each layer's combine sums every rank's partial over NVLink
        from llambda_b200 import ep
        keep.append(ep.attach_peer_reduction(sessions))
    collective = world > 1 and not peer
    setup_s = time.time() - t_setup
    x0 = torch.empty(B, cfg.hidden, device="cuda")
    LB.synth_fill_device(LB.TYPE_F32, args.seed, CF.S_ACT, 0, B * cfg.hidden, 1.0, x0)
    bufs = [torch.empty(B, cfg.hidden, device="cuda") for _ in range(2)]
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
            s.run_device(cur, out, B, stream=st)
            if collective:
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
    if not collective and not args.no_graph:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        graph.replay()
        torch.cuda.synchronize()
    for s in sessions:
        if s.status() != 0:
            raise SystemExit("device status reported a non-positive router weight sum")
    layer_ev = [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(NL)]
    sampler = ClockSampler(local)
    sampler.start()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(args.steps):
        if graph is not None:
            graph.replay()
        else:
            step()
    e1.record(stream)
    torch.cuda.synchronize()
    barrier(world)
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    ms = max_over_ranks(ms, world)
    value = B / (ms * 1e-3)
    # per-layer times and, from CUDA events the sessions record on the same
    # stream, the gate/up and routed down kernels of every layer (launched eagerly)
    for s in sessions:
        s.time_kernels(True)
    step(layer_ev)
    torch.cuda.synchronize()
    layer_ms = [a.elapsed_time(b) for a, b in layer_ev]
    kern_ms = [s.kernel_ms() for s in sessions]
    for s in sessions:
        s.time_kernels(False)

    # routing of the timed steps (identical every step: same x0) -> algorithmic bytes
    sel = torch.empty(B, cfg.top_k, dtype=torch.int32, device="cuda")
    cur = x0
    distinct = []
    for li, s in enumerate(sessions):
        out = bufs[li % 2]
        s.run_device(cur, out, B, sel_dev=sel, stream=stream)
        if collective:
            dist.all_reduce(out)
        distinct.append(distinct_experts(sel.cpu().numpy(), cfg.experts))
        cur = out
    torch.cuda.synchronize()
    eb, ee = rank * cfg.experts // world, (rank + 1) * cfg.experts // world
    own_distinct = []
    cur = x0
    for li, s in enumerate(sessions):
        out = bufs[li % 2]
        s.run_device(cur, out, B, sel_dev=sel, stream=stream)
        if collective:
            dist.all_reduce(out)
        ss = sel.cpu().numpy()
        own_distinct.append(int(np.unique(ss[(ss >= eb) & (ss < ee)]).size))
        cur = out
    from llambda_b200 import ep as _ep
    streams_shared = _ep.layer_roles(rank, world, cfg.experts, peer)["shared_here"]
    layer_bytes = [cfg.router_bytes() + (cfg.shared_bytes() if streams_shared else 0)
                   + u * cfg.expert_bytes() + 2 * 4 * B * cfg.hidden for u in own_distinct]
    peak, peak_kind = hbm_peak()
    # the dominant kernel: the gate/up pass (its rows of every distinct routed
    # expert this rank owns, plus the shared expert's where it runs here)
    gu_bytes = [u * cfg.gate_up_bytes() + (cfg.shared_gate_up_bytes() if streams_shared else 0)
                for u in own_distinct]
    gu_ms = statistics.mean(k[0] for k in kern_ms)
    dn_bytes = [u * cfg.down_bytes() for u in own_distinct]
    dn_ms = statistics.mean(k[1] for k in kern_ms)
    achieved = (sum(gu_bytes) / NL) / (gu_ms * 1e-3) / 1e9
    layer_gbs = (sum(layer_bytes) / NL) / (statistics.mean(layer_ms) * 1e-3) / 1e9
    prefill = B >= LB.prefill_min_tokens()
    if prefill:
        gu_name = ("pf_gemm_kernel<Q4_K, gate+up> (tcgen05 bf16 grouped GEMM, routed + shared)"
                   if cfg.has_gate else
                   "pf_gemm_kernel<Q4_K, up> (tcgen05 bf16 grouped GEMM, routed + shared)")
        dn_name = "pf_gemm_kernel<Q6_K, down> (tcgen05 bf16 grouped GEMM, routed + shared)"
        gu_traffic = PF_GATE_UP_TRAFFIC_BYTES.get(B) if world == 1 and cfg is CF.CONFIG3 else None
        dn_traffic = PF_DOWN_TRAFFIC_BYTES.get(B) if world == 1 and cfg is CF.CONFIG3 else None
    else:
        gu_name = ("moe_up_slab_kernel (gate/up pass, Q4_K)" if cfg.has_gate
                   else "moe_up_slab_kernel (up pass, Q4_K)")
        dn_name = "moe_down_slab_kernel (routed, Q6_K)"
        gu_traffic = GATE_UP_TRAFFIC_BYTES_N1 if world == 1 and cfg is CF.CONFIG3 else None
        dn_traffic = DOWN_TRAFFIC_BYTES_N1 if world == 1 and cfg is CF.CONFIG3 else None
    roofline = {"bound": "hbm", "kernel": gu_name,
                "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                "algorithmic_bytes_per_launch": int(sum(gu_bytes) / NL),
                "launch_us_mean": round(gu_ms * 1e3, 2),
                # DRAM read+write bytes of one gate/up launch at N=1 (ncu capture)
                "traffic": gu_traffic,
                "down": {"kernel": dn_name,
                         "achieved": round((sum(dn_bytes) / NL) / (dn_ms * 1e-3) / 1e9, 1),
                         "launch_us_mean": round(dn_ms * 1e3, 2),
                         "traffic": dn_traffic},
                "layer": {"achieved": round(layer_gbs, 1), "frac": round(layer_gbs / peak, 4),
                          "algorithmic_bytes": int(sum(layer_bytes) / NL),
                          "us_mean": round(statistics.mean(layer_ms) * 1e3, 2)}}

    # e2e through the C ABI with host buffers (one call per layer per step)
    e2e = None
    if not args.no_e2e:
        # page-locked host buffers (the library copies them by DMA, no staging)
        pinned = [x0.cpu().pin_memory()] + [torch.empty(tuple(x0.shape), dtype=torch.float32,
                                                        pin_memory=True) for _ in range(2)]
        x_host = pinned[0].numpy()
        if world > 1:
            import torch.distributed as dist
            gloo = dist.new_group(backend="gloo")

        host_bufs = [t.numpy() for t in pinned[1:]]  # run-into destinations

        def e2e_step():
            cur_h = x_host
            for li, s in enumerate(sessions):
                out_h = s.run_into(host_bufs[li % 2], cur_h)
                if collective:
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
        dt = (time.perf_counter() - t0) / args.steps
        dt = max_over_ranks(dt, world)
        e2e = {"value": B / dt, "unit": "tokens/s",
               "h2d_bytes_per_step": NL * B * cfg.hidden * 4,
               "d2h_bytes_per_step": NL * B * cfg.hidden * 4,
               "path": "llambda_cuda_moe_session_run per layer from and into preallocated "
                       "page-locked host float buffers (the reference's run-into convention)"}

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
            except Exception as e:  # memory pressure at N=1 with the stack resident
                kernels["error"] = str(e)
        if not args.no_cpu_baseline:
            cores = os.cpu_count() or 1
            tok_s, per_layer = time_cpu_stack(cfg, NL, B, args.seed, steps=3, warmup=1)
            cpu = {"value": tok_s, "unit": "tokens/s", "cores": cores, "kind": "port",
                   "sample": f"{B} tokens through 1 qwen3next layer per sample "
                             f"({per_layer * 1e3:.1f} ms), scaled to {NL} layers"}

    # decode: rms-norm + router, top-k with routing, gate/up, routed down, shared
    # down (ranks that compute a share of the shared expert), combine.
    # prefill: rms-norm, router K slices, their sum, top-k with routing, gather,
    # tile plan, gate/up, down, combine.
    launches_per_layer = 9 if prefill else 5 + (1 if streams_shared else 0)
    phase = "prefill" if prefill else "decode"
    line = {"metric": f"MoE FFN {phase} tokens/s", "value": round(value, 2), "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16" if prefill else "f32", "data": "synthetic",
            "config": {"workload": (f"config5_qwen3next_moe_stack_{NL}L_{phase}_b{B}"
                                    if cfg is CF.CONFIG3 else
                                    f"config4_nemotron_h_moe_stack_{NL}L_{phase}_b{B}"),
                       "batch": B, "layers": NL, "experts": cfg.experts, "top_k": cfg.top_k,
                       "hidden": cfg.hidden,
                       "parallelism": f"ep{world}" + ("-peer" if peer else "-nccl" if world > 1 else ""),
                       "l2": "weights streamed per step exceed L2 (no flush needed)",
                       "setup_s": round(setup_s, 1)},
            "roofline": roofline, "e2e": e2e, "cpu_baseline": cpu, "clocks": clocks,
            "gpu_launches": launches_per_layer * NL * args.steps,
            "distinct_experts_per_layer_mean": round(statistics.mean(distinct), 1)}
    if kernels is not None:
        line["kernels"] = kernels
    if rank == 0:
        print(json.dumps(line), flush=True)
    for s in sessions:
        s.close()
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
