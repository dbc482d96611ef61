"""Benchmark of the Qwen3-MoE sparse block on B200 — one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (every N): benchmark config 2's block — H=2048, E=128 experts, top-8, I=768, bf16 —
with T=8192 tokens per rank and expert parallelism EP=N (16 experts per rank at N=8): weak
scaling, per-rank work fixed. One step = one ``MoE.forward`` of the drop-in module (router
GEMM, routing, dispatch, grouped SwiGLU experts, combine; at N>1 the all-to-all dispatch and
combine). Inputs: seeded synthetic tensors (no dataset exists for this path).

Reported:
* ``value``: tokens/s over all ranks, device-timed (CUDA events, barrier + synchronize on both
  sides, max over ranks), inputs resident in HBM;
* ``e2e``: the same metric through ``MoE.forward`` with the step's hidden states copied from
  pinned host memory and the output copied back inside the timed region;
* ``roofline``: the grouped gate_up GEMM (the dominant kernel), its algorithmic FLOPs per
  launch over its average event-timed duration, against the measured bf16 peak;
* ``cpu_baseline``: the numpy oracle (a restatement of the reference's CPU path) on a bounded
  sample of the same workload, on the host's cores (rank 0, N=1 only);
* ``decode_cfg1``: config 1 (T=64, single GPU) at N=1, HBM roofline.
``--impl reference`` times the reference algorithm on the host CPU (the oracle port), rank 0
only, on a sample of the same workload per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "MoE-block tokens/s (Qwen3-30B-A3B block, EP=N, T=8192/rank)"
UNIT = "tokens/s"
CFG = dict(T=8192, H=2048, E=128, k=8, I=768)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=CFG["T"], help="tokens per rank")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    return ap.parse_args()


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def ncu_traffic(kernel="gate_up"):
    """Per-launch DRAM bytes of the dominant kernel (``gate_up`` or ``fused``) at config 2 from
    the committed ncu summary, if it holds a figure for that kernel."""
    p = REPO / "profiles" / "ncu_traffic.txt"
    if not p.exists():
        return None
    vals = {}
    for line in p.read_text().splitlines():
        if "=" in line and not line.lstrip().startswith("#"):
            k, v = line.split("=", 1)
            vals[k.strip()] = v.strip()
    try:
        return float(vals[f"{kernel}_cfg2_bytes_per_launch"])
    except (KeyError, ValueError):
        return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"prism_clocks_{os.getpid()}.csv"

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self, gpus):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) not in gpus:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        self.path.unlink(missing_ok=True)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": sorted(reasons),
                "samples": len(sm)}


def workload_config(tokens_per_rank, world):
    """The ``config`` of both arms' JSON lines (benchmark config 2 at EP=world)."""
    return {"workload": "cfg2: Qwen3-30B-A3B MoE block H=2048 E=128 top-8 I=768",
            "tokens_per_rank": tokens_per_rank, "global_batch": tokens_per_rank * world,
            "ep": world, "parallelism": f"ep{world}",
            "l2": "inputs larger than L2: 1.2 GB of expert weights streamed per step"}


def launches_per_step(world, fused):
    """This library's kernels per MoE.forward (the router GEMM is torch's): route, plan (chunk,
    scan, scatter), then EP=1: permute, experts (2 launches, or 1 fused), combine; EP>1: counts
    all-gather, the fused expert launch with the exchange inside, wait for returned rows,
    combine."""
    experts = 1 if fused else 2
    return 1 + 3 + (1 + experts + 1 if world == 1 else 1 + experts + 1 + 1)


def dist_setup(n):
    import torch
    import torch.distributed as dist
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}: launch N>1 with torchrun")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def build_block(T, world, rank, device, cfg_id=2):
    import torch

    from prism_infer_b200 import synthetic
    from prism_infer_b200.engine.parallel import set_expert_parallel_size
    from prism_infer_b200.layers.moe import MoE
    H, E, k, I = CFG["H"], CFG["E"], CFG["k"], CFG["I"]
    seed = synthetic.config_seed(cfg_id)
    set_expert_parallel_size(world)
    El = E // world
    wg, wgu, wd = synthetic.make_weights_torch(H, E, I, seed, torch.bfloat16, device,
                                               expert_range=(rank * El, (rank + 1) * El))
    moe = MoE(H, I, E, k).to(device=device, dtype=torch.bfloat16)
    bank = moe.ep_moe if world > 1 else moe
    with torch.no_grad():
        moe.gate.weight.copy_(wg)
        bank.w_gate_up.copy_(wgu)
        bank.w_down.copy_(wd)
    x = synthetic.make_hidden_torch(T, H, synthetic.config_seed(cfg_id, rank), torch.bfloat16,
                                    device)
    return moe, x


def time_device(fn, steps, warmup, world, nvtx=None):
    """Device time of ``steps`` calls (ms, max over ranks). ``nvtx`` names an NVTX range around
    the timed calls (used to select them in an ncu launch list)."""
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        fn(-1)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if nvtx:
        torch.cuda.nvtx.range_push(nvtx)
    start.record()
    for i in range(steps):
        fn(i)
    end.record()
    if nvtx:
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ms = start.elapsed_time(end)
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def cpu_oracle_rate(sample_tokens, reps, seed=2000):
    """Tokens/s of the numpy oracle (fp32 restatement of the reference's MoE.forward) on
    ``sample_tokens`` tokens of the workload, best of ``reps``."""
    import numpy as np

    from oracle import moe_oracle as O
    from prism_infer_b200 import synthetic
    H, E, k, I = CFG["H"], CFG["E"], CFG["k"], CFG["I"]
    wts = synthetic.make_weights_np(H, E, I, seed)
    x = synthetic.make_hidden_np(sample_tokens, H, seed)
    best = math.inf
    for _ in range(reps):
        t0 = time.perf_counter()
        O.moe_forward(x, wts.w_gate, wts.w_gate_up, wts.w_down, k, True, "float32")
        best = min(best, time.perf_counter() - t0)
    del np
    return sample_tokens / best, best


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    sample = 256
    from oracle import moe_oracle as O
    from prism_infer_b200 import synthetic
    H, E, k, I = CFG["H"], CFG["E"], CFG["k"], CFG["I"]
    wts = synthetic.make_weights_np(H, E, I, 2000)
    x = synthetic.make_hidden_np(sample, H, 2000)
    for _ in range(max(1, min(args.warmup, 3))):                                   # warm-up
        O.moe_forward(x, wts.w_gate, wts.w_gate_up, wts.w_down, k, True, "float32")
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.moe_forward(x, wts.w_gate, wts.w_gate_up, wts.w_down, k, True, "float32")
    dt = time.perf_counter() - t0
    value = sample * args.steps / dt
    desc = (f"numpy oracle (fp32 restatement of prism_infer MoE.forward, moe.py:69-100) on "
            f"{sample} tokens of the workload per step, {cores} host threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {**workload_config(args.tokens, args.gpus),
                   "sample_tokens_per_step": sample},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": desc},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist

    from prism_infer_b200 import capi
    rank, world, local = dist_setup(args.gpus)
    device = torch.device("cuda", local)
    T = args.tokens
    H, E, k, I = CFG["H"], CFG["E"], CFG["k"], CFG["I"]
    moe, x = build_block(T, world, rank, device)
    peaks, peak_kind = load_peaks()

    # ---- device-resident timing with per-stage events ----
    steps, warmup = args.steps, args.warmup
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(steps)]
    for row in ev:
        for e in row:
            e.record()
    torch.cuda.synchronize()
    out_holder = {}

    def step(i):
        if i >= 0:
            capi.set_profile_events(ev[i])
        with torch.inference_mode():
            out_holder["y"] = moe(x)
        if i >= 0:
            capi.set_profile_events(None)

    sampler = ClockSampler() if rank == 0 else None
    if sampler:
        sampler.start()
    ms = time_device(step, steps, warmup, world, nvtx="prism_timed")
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    gpu_ids = ([int(v) for v in vis.split(",")][:world] if vis and all(
        v.strip().isdigit() for v in vis.split(",")) else list(range(world)))
    clocks = sampler.stop(gpu_ids) if sampler else None
    moe.check_device_error(device) if world == 1 else None

    # per-stage averages (ms) — slots: route, plan, permute, gate_up, down, combine
    # EP>1: "exchange" is the counts all-gather; the row dispatch and return run inside the
    # fused expert launch ("experts"), and "combine" includes waiting for every returned row
    names = ["route", "plan", "permute" if world == 1 else "exchange", "gate_up", "down",
             "combine"]
    stage_ms = {}
    for s, name in enumerate(names):
        vals = []
        for row in ev:
            try:
                vals.append(row[s].elapsed_time(row[s + 1]))
            except RuntimeError:
                pass
        stage_ms[name] = sum(vals) / len(vals) if vals else None

    fused = stage_ms["down"] is not None and stage_ms["down"] < 5e-3
    if fused:   # both expert GEMMs ran as one launch (slot 3 -> 4); slot 4 -> 5 is empty
        stage_ms["experts"] = stage_ms.pop("gate_up")
        stage_ms.pop("down")
    value = world * T * steps / (ms / 1e3)

    # ---- end to end through MoE.forward with host buffers ----
    # Every step copies its hidden states from pinned host memory and its output back. The
    # copies run on their own streams, double-buffered, so step i+1's upload and step i-1's
    # download overlap step i's forward (how a serving loop feeds the block).
    x_host = [x.detach().cpu().pin_memory() for _ in range(2)]
    y_host = [torch.empty_like(x_host[0]).pin_memory() for _ in range(2)]
    x_dev = [torch.empty_like(x) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    comp = torch.cuda.current_stream(device)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_done = [torch.cuda.Event() for _ in range(2)]
    ev_out = [torch.cuda.Event() for _ in range(2)]
    for e in ev_done + ev_out:
        e.record(comp)

    def e2e_step(i):
        b = i % 2
        s_in.wait_event(ev_done[b])          # x_dev[b] no longer read by step i-2
        with torch.cuda.stream(s_in):
            x_dev[b].copy_(x_host[b], non_blocking=True)
            ev_in[b].record(s_in)
        comp.wait_event(ev_in[b])
        with torch.inference_mode():
            y = moe(x_dev[b])
        ev_done[b].record(comp)
        s_out.wait_event(ev_done[b])
        s_out.wait_event(ev_out[b])          # y_host[b] free (step i-2's copy finished)
        with torch.cuda.stream(s_out):
            y_host[b].copy_(y, non_blocking=True)
            y.record_stream(s_out)
            ev_out[b].record(s_out)

    def e2e_loop_end():
        comp.wait_stream(s_out)

    def e2e_step_timed(i):
        e2e_step(i)
        if i == steps - 1 or i < 0:
            e2e_loop_end()

    ms_e2e = time_device(e2e_step_timed, steps, max(2, warmup // 2), world)
    e2e_value = world * T * steps / (ms_e2e / 1e3)

    # ---- roofline of the dominant kernel ----
    # fused engine (EP>1): both expert GEMMs in one launch, 6*H*I FLOP per routed row;
    # otherwise the gate_up GEMM launch, 4*H*I FLOP per routed row
    rows = T * k                       # routed rows per rank (EP: received rows ~ T*k)
    if fused:
        kflops = 2.0 * rows * H * (2 * I) + 2.0 * rows * I * H
        kms = stage_ms["experts"]
        kname = "fused_experts_kernel (gate_up + down, EP exchange inside)"
        algo = f"2*{rows}*{H}*{2 * I} + 2*{rows}*{I}*{H} = {kflops:.4g} FLOP per launch"
    else:
        kflops = 2.0 * rows * H * (2 * I)
        kms = stage_ms["gate_up"]
        kname = "grouped_gemm_sm100_kernel<gate_up>"
        algo = f"2*{rows}*{H}*{2 * I} = {kflops:.4g} FLOP per launch"
    achieved = kflops / (kms / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    traffic = ncu_traffic("fused" if fused else "gate_up")
    roofline = {"bound": "tensor", "kernel": kname,
                "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": f"{peak_kind} bf16_tflops (burst)",
                "traffic": traffic, "algorithmic": algo}
    block_flops = T * world * (2 * H * E + k * 6 * H * I)
    extra = {
        "stages_ms": stage_ms,
        "block_tflops": block_flops * steps / (ms / 1e3) / 1e12 / world,
        "block_frac_of_peak": block_flops * steps / (ms / 1e3) / 1e12 / world / peak,
    }
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    if world == 1:
        el = 2
        perm_bytes = T * H * el + rows * H * el + rows * 4
        comb_bytes = rows * H * el + T * H * el + rows * (4 + el)
        extra["hbm"] = {
            # bf16 fuses the permutation into the gate_up GEMM's gather loads
            "permute_gbs": (perm_bytes / (stage_ms["permute"] / 1e3) / 1e9
                            if stage_ms["permute"] > 1e-3 else "fused into gate_up"),
            "combine_gbs": comb_bytes / (stage_ms["combine"] / 1e3) / 1e9,
            "route_gbs": (T * E * el + T * k * (8 + el)) / (stage_ms["route"] / 1e3) / 1e9,
            "peak_gbs": hbm_peak,
        }

    # ---- config 1 decode (T=64) at N=1 ----
    if world == 1 and not args.no_decode:
        xd = x[:64].contiguous()

        def dec(_i):
            with torch.inference_mode():
                moe(xd)
        ms_dec = time_device(dec, 200, 20, 1)
        with torch.inference_mode():
            _, ids, _ = moe.route(xd)
        n_exp = int(torch.unique(ids).numel())
        wbytes = n_exp * 3 * H * I * 2
        t_step = ms_dec / 200 / 1e3
        extra["decode_cfg1"] = {"tokens": 64, "ms_per_step": ms_dec / 200,
                                "tokens_per_s": 64 / t_step,
                                "weight_bytes_per_step": wbytes,
                                "hbm_gbs": wbytes / t_step / 1e9,
                                "frac_of_hbm_peak": wbytes / t_step / 1e9 / hbm_peak}
        # the same step captured once in a CUDA graph and replayed (no host work per step)
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side), torch.inference_mode():
            for _ in range(2):
                moe(xd)
        torch.cuda.current_stream(device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.inference_mode(), torch.cuda.graph(graph):
            moe(xd)
        ms_g = time_device(lambda _i: graph.replay(), 200, 20, 1)
        extra["decode_cfg1"]["graph_ms_per_step"] = ms_g / 200
        extra["decode_cfg1"]["graph_hbm_gbs"] = wbytes / (ms_g / 200 / 1e3) / 1e9
        del graph

    # ---- CPU baseline (rank 0, N=1) ----
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cores = os.cpu_count() or 1
        sample = 512
        rate, best = cpu_oracle_rate(sample, 2)
        cpu = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
               "sample": f"numpy oracle, fp32, {sample} tokens of the workload, best of 2 "
                         f"({best:.2f} s each), {cores} host threads"}

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(T, world),
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2,
                "how": "MoE.forward; per step H2D of x from pinned host and D2H of the output, "
                       "on copy streams double-buffered against the forward"},
        "gpu_launches": steps * launches_per_step(world, fused),
        "clocks": clocks,
        **extra,
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
