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
  pinned host memory and the output copied back inside the timed region, next to the same
  copies timed alone (``copy_only``);
* ``roofline``: the dominant kernel (N=1: the grouped gate_up GEMM; N>1: the fused expert launch
  with the exchange inside), its algorithmic FLOPs per launch over its average event-timed
  duration, against the measured bf16 peak;
* ``parity``: after timing, on every rank — routing of every token compared bit for bit with
  torch's own CUDA softmax / top-k / renorm on the same logits (the reference's calls,
  prism_infer/layers/moe.py:74-81), the device error word, and sampled tokens' outputs against
  the reference's expert math run with torch ops (bf16 F.linear, SiluAndMul with one rounding,
  combine_weighted_sum) on the same routing;
* ``cfg3`` / ``cfg4``: benchmark configs 3 (Zipf-skewed routing, T=4096/rank) and 4
  (Qwen3-235B-A22B block, H=4096, I=1536, T=16384/rank) at the same EP size, each with its own
  parity; ``decode_cfg1``: config 1's batch (T=64 per rank) eager and replayed from a CUDA graph,
  against the HBM roofline of the expert weights it streams;
* ``a2a`` (N>1): NVLink bytes each rank sends per step, the dispatch window stamped inside the
  fused launch (%globaltimer) and the bandwidths they give;
* ``cpu_baseline``: the numpy restatement of the reference's CPU path on a bounded sample of the
  same workload, on the host's cores (rank 0, N=1 only).
``--impl reference`` times the reference algorithm on the host CPU (the numpy port; the
reference is Python over torch with no native code to build), rank 0 only, one full per-rank
batch (T=8192 tokens) per step, on every host thread it may use.
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
NVLINK_GBS = 770.0   # measured GPU-to-GPU copy bandwidth per direction (B200, NVLink 5)
CFGS = {
    2: dict(T=8192, H=2048, E=128, k=8, I=768, skew=False,
            name="cfg2: Qwen3-30B-A3B MoE block H=2048 E=128 top-8 I=768"),
    3: dict(T=4096, H=2048, E=128, k=8, I=768, skew=True,
            name="cfg3: cfg2 block, Zipf(1.2)-skewed routing, top expert ~8x mean load"),
    4: dict(T=16384, H=4096, E=128, k=8, I=1536, skew=False,
            name="cfg4: Qwen3-235B-A22B MoE block H=4096 E=128 top-8 I=1536"),
}
CFG = CFGS[2]
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
PARITY_MAX_ABS, PARITY_MEAN_REL = 2e-2, 1e-2     # bf16 tolerance of the north star


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=CFG["T"], help="tokens per rank")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-extra-configs", action="store_true")
    ap.add_argument("--no-ep1", action="store_true")
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
    return {"workload": CFG["name"],
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


def build_block(cfg_id, T, world, rank, device):
    """The drop-in ``MoE`` of benchmark config ``cfg_id`` with this rank's experts, and this
    rank's hidden states (seeded per config and rank)."""
    import torch

    from prism_infer_b200 import synthetic
    from prism_infer_b200.engine.parallel import set_expert_parallel_size
    from prism_infer_b200.layers.moe import MoE
    c = CFGS[cfg_id]
    H, E, k, I = c["H"], c["E"], c["k"], c["I"]
    seed = synthetic.config_seed(cfg_id)
    set_expert_parallel_size(world)
    El = E // world
    wg, wgu, wd = synthetic.make_weights_torch(H, E, I, seed, torch.bfloat16, device,
                                               skew=c["skew"], k=k,
                                               expert_range=(rank * El, (rank + 1) * El))
    moe = MoE(H, I, E, k).to(device=device, dtype=torch.bfloat16)
    bank = moe.ep_moe if world > 1 else moe
    with torch.no_grad():
        moe.gate.weight.copy_(wg)
        bank.w_gate_up.copy_(wgu)
        bank.w_down.copy_(wd)
    x = synthetic.make_hidden_torch(T, H, synthetic.config_seed(cfg_id, rank), torch.bfloat16,
                                    device, skew=c["skew"])
    return moe, x


def free_block(moe, world):
    import torch
    if world > 1 and moe.ep_moe is not None:
        moe.ep_moe.release()          # collective
    del moe
    torch.cuda.empty_cache()


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


def reduce_over_ranks(vals, op, world):
    """Elementwise reduction of a list of floats over the ranks (op: "max", "min", "sum")."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return list(vals)
    t = torch.tensor(vals, dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN,
                           "sum": dist.ReduceOp.SUM}[op])
    return t.tolist()


def check_device_error(moe, world, device):
    """Status of the block's device error word after the timed steps (0 = none)."""
    try:
        if world > 1:
            moe.ep_moe.check_device_error()
        else:
            moe.check_device_error(device)
        return 0
    except RuntimeError as e:
        msg = str(e)
        return int(msg.split("status ")[1].split(":")[0]) if "status " in msg else -1


def parity_check(moe, x, cfg_id, world, rank, device, n_sample=32):
    """Parity of one more step of ``moe`` on ``x`` (see the module docstring). Routing is checked
    for every token; outputs for ``n_sample`` tokens spread over the batch, against the reference's
    expert arithmetic on the same routing (a token's output depends only on its own row). Remote
    experts' weights are regenerated from their seeds. Returns the rank-reduced summary."""
    import torch
    import torch.nn.functional as F

    from prism_infer_b200 import capi, synthetic
    c = CFGS[cfg_id]
    H, E, k, I = c["H"], c["E"], c["k"], c["I"]
    T = x.shape[0]
    with torch.inference_mode():
        logits = moe.gate(x)
        out = moe(x)
        ids, w, _ = capi.route_topk(logits.contiguous(), k, True)
        # the reference's routing, moe.py:77-81, with torch's CUDA kernels
        p = F.softmax(logits, dim=-1, dtype=torch.float)
        rw, rid = torch.topk(p, k, dim=-1)
        rw = (rw / rw.sum(dim=-1, keepdim=True)).to(x.dtype)
        ids_mismatch = int((ids != rid).any(dim=-1).sum().item())
        w_mismatch = int((w != rw).any(dim=-1).sum().item())
        counts = torch.bincount(ids.reshape(-1), minlength=E)
        sample = torch.linspace(0, T - 1, n_sample, device=device).round().long().unique()
        xs, sid, sw = x[sample], rid[sample], rw[sample]
        seed = synthetic.config_seed(cfg_id)
        ys = torch.empty(sample.numel(), k, H, dtype=x.dtype, device=device)
        for e in torch.unique(sid).tolist():
            wgu, wd = synthetic.expert_weights_torch(H, I, seed, e, torch.bfloat16, device)
            tt, jj = torch.nonzero(sid == e, as_tuple=True)
            gu = F.linear(xs[tt], wgu)                                       # bf16, like cuBLAS
            act = (F.silu(gu[:, :I].float()) * gu[:, I:].float()).to(x.dtype)   # compiled: 1 rounding
            ys[tt, jj] = F.linear(act, wd)
        ref = (ys * sw.unsqueeze(-1)).sum(dim=1)              # combine_weighted_sum (:45-57)
        got = out[sample]
        d = (got.float() - ref.float()).abs()
        max_abs = float(d.max().item()) if d.numel() else 0.0
        rel_num = float(d.sum().item())
        rel_den = float(ref.float().abs().sum().item())
    status = check_device_error(moe, world, device)
    vals = reduce_over_ranks([ids_mismatch, w_mismatch, max_abs, rel_num, rel_den,
                              float(status != 0), float(T)], "sum", world)
    mx = reduce_over_ranks([max_abs, float(counts.max().item())], "max", world)
    load = reduce_over_ranks(counts.float().tolist(), "sum", world)
    mean_load = sum(load) / E
    res = {
        "ids_exact": vals[0] == 0, "weights_exact": vals[1] == 0,
        "tokens_routed_checked": int(vals[6]), "tokens_with_different_ids": int(vals[0]),
        "sampled_tokens_per_rank": int(sample.numel()), "max_abs": mx[0],
        "mean_rel": vals[3] / max(vals[4], 1e-30), "device_error_ranks": int(vals[5]),
        "tolerance": {"max_abs": PARITY_MAX_ABS, "mean_rel": PARITY_MEAN_REL},
        "max_expert_load_over_mean": max(load) / mean_load if mean_load else None,
        "ref_mean_abs": vals[4] / max(reduce_over_ranks([float(ref.numel())], "sum", world)[0], 1),
    }
    res["ok"] = bool(res["ids_exact"] and res["weights_exact"] and res["device_error_ranks"] == 0
                     and res["max_abs"] <= PARITY_MAX_ABS
                     and res["mean_rel"] <= PARITY_MEAN_REL)
    return res


def a2a_stats(moe, x, world, reps=5):
    """NVLink exchange of an EP step from the in-kernel stamps (``prism_moe_ep_read_stats``),
    averaged over ``reps`` steps; per-rank figures averaged over the ranks."""
    import torch
    H = x.shape[1]
    acc = [0.0] * 5
    for _ in range(reps):
        with torch.inference_mode():
            moe(x)
        st = moe.ep_moe.step_stats()
        disp_ns = max(st["dispatch_t1_ns"] - st["dispatch_t0_ns"], 1)
        fused_ns = max(st["fused_t1_ns"] - st["fused_t0_ns"], 1)
        sb, rb = st["send_rows"] * H * 2, st["recv_rows"] * H * 2
        acc = [a + b for a, b in zip(acc, [sb, rb, disp_ns, fused_ns,
                                           (sb + rb) / fused_ns])]
    acc = [a / reps for a in acc]
    tot = reduce_over_ranks(acc, "sum", world)
    mean = [t / world for t in tot]
    T, k = x.shape[0], CFGS[2]["k"]
    return {
        "dispatch_remote_bytes_per_rank": mean[0],
        "return_remote_bytes_per_rank": mean[1],
        "dispatch_bytes_without_dedup_per_rank": T * k * (world - 1) / world * H * 2,
        "dispatch_ms": mean[2] / 1e6,
        "fused_launch_ms": mean[3] / 1e6,
        "dispatch_gbs": mean[0] / mean[2],
        "nvlink_gbs_over_fused_launch": mean[4],
        "landing_zone_bytes_per_rank": moe.ep_moe.landing_bytes(),
        "how": "per rank: token rows pulled from other ranks (one per token and rank) and rows "
               "returned to them (one per routed entry) x H x 2 B; the no-dedup figure assumes "
               "uniform routing; dispatch window = first chunk claimed to last chunk stored "
               "(%globaltimer in the copy warps); mean over ranks and steps",
    }


def ep_path_one_gpu(moe, x, device, peak, steps=20, warmup=3):
    """The expert-parallel step (``prism_moe_ep_forward``) at ep_size 1 on the block's weights:
    the same kernels as at EP>1 (counts exchange, fused expert launch with its copy warps,
    return wait, combine), against this GPU's own landing zone. Shows what the exchange
    machinery costs without NVLink, and is the launch an ncu capture on one GPU sees."""
    import torch

    from prism_infer_b200.engine.parallel.expert_parallel import ExpertParallelMoE
    c = CFGS[2]
    bank = ExpertParallelMoE(c["H"], c["I"], c["E"], 1, 0, transport="p2p").to(device,
                                                                               torch.bfloat16)
    with torch.no_grad():
        bank.w_gate_up.copy_(moe.w_gate_up)
        bank.w_down.copy_(moe.w_down)
    holder = {}

    def step(_i):
        with torch.inference_mode():
            holder["y"] = bank.forward_p2p(x, router_logits=moe.gate(x), top_k=c["k"])
    ms = time_device(step, steps, warmup, 1)
    st = bank.step_stats()
    bank.check_device_error()
    with torch.inference_mode():
        same = bool(torch.equal(holder["y"], moe(x)))
    fused_ms = (st["fused_t1_ns"] - st["fused_t0_ns"]) / 1e6
    T = x.shape[0]
    kflops = 2.0 * T * c["k"] * c["H"] * 3 * c["I"]
    res = {"ms_per_step": ms / steps, "tokens_per_s": T / (ms / steps / 1e3),
           "fused_launch_ms": fused_ms,
           "fused_launch_tflops": kflops / (fused_ms / 1e3) / 1e12 if fused_ms > 0 else None,
           "fused_launch_frac_of_peak": (kflops / (fused_ms / 1e3) / 1e12 / peak
                                         if fused_ms > 0 else None),
           "output_equals_block_path": same,
           "how": "ExpertParallelMoE(ep_size=1).forward_p2p; fused launch span from its "
                  "%globaltimer stamps (last step)"}
    bank.release()
    return res


def sub_config(cfg_id, world, rank, device, peak, steps=10, warmup=3):
    """Throughput and parity of benchmark config ``cfg_id`` at EP=world."""
    c = CFGS[cfg_id]
    moe, x = build_block(cfg_id, c["T"], world, rank, device)
    import torch

    def step(_i):
        with torch.inference_mode():
            moe(x)
    ms = time_device(step, steps, warmup, world)
    t = ms / steps / 1e3
    flops = c["T"] * (2 * c["H"] * c["E"] + c["k"] * 6 * c["H"] * c["I"])
    res = {"workload": c["name"], "tokens_per_rank": c["T"], "ep": world, "steps": steps,
           "ms_per_step": ms / steps, "tokens_per_s": world * c["T"] / t,
           "block_tflops_per_gpu": flops / t / 1e12,
           "block_frac_of_peak": flops / t / 1e12 / peak}
    res["parity"] = parity_check(moe, x, cfg_id, world, rank, device, n_sample=16)
    if world > 1:
        res["a2a"] = a2a_stats(moe, x, world, reps=3)
    free_block(moe, world)
    return res


def cpu_oracle_rate(sample_tokens, reps, seed=2000):
    """Tokens/s of the numpy oracle (fp32 restatement of the reference's MoE.forward) on
    ``sample_tokens`` tokens of the workload, best of ``reps``."""
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
    return sample_tokens / best, best


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(args):
    """The reference's block on the host CPU: the numpy port of MoE.forward (fp32), one full
    per-rank batch per step, on every host thread this process may use. A launcher (torchrun)
    sets OMP_NUM_THREADS=1 before Python starts, so the BLAS pool is resized explicitly."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = host_threads()
    from threadpoolctl import threadpool_info, threadpool_limits

    from oracle import moe_oracle as O
    from prism_infer_b200 import synthetic
    H, E, k, I = CFG["H"], CFG["E"], CFG["k"], CFG["I"]
    T = args.tokens
    wts = synthetic.make_weights_np(H, E, I, 2000)
    x = synthetic.make_hidden_np(T, H, 2000)
    with threadpool_limits(limits=cores):
        used = max([d.get("num_threads", 1) for d in threadpool_info()] or [1])
        for _ in range(max(1, min(args.warmup, 2))):                             # warm-up
            O.moe_forward(x, wts.w_gate, wts.w_gate_up, wts.w_down, k, True, "float32")
        t0 = time.perf_counter()
        for _ in range(args.steps):
            O.moe_forward(x, wts.w_gate, wts.w_gate_up, wts.w_down, k, True, "float32")
        dt = time.perf_counter() - t0
    value = T * args.steps / dt
    desc = (f"numpy port of prism_infer MoE.forward (moe.py:69-100), fp32, {T} tokens "
            f"(one rank's full batch) per step, BLAS on {used} of {cores} host threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {**workload_config(T, args.gpus), "sample_tokens_per_step": T},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": used, "kind": "port",
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
    moe, x = build_block(2, T, world, rank, device)
    peaks, peak_kind = load_peaks()
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    hbm_peak = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))

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
    status_after_timing = check_device_error(moe, world, device)

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

    # ---- parity of the timed configuration, on every rank ----
    parity = parity_check(moe, x, 2, world, rank, device)
    parity["device_error_after_timing"] = int(reduce_over_ranks(
        [float(status_after_timing != 0)], "sum", world)[0])
    parity["ok"] = parity["ok"] and parity["device_error_after_timing"] == 0

    # ---- end to end through MoE.forward with host buffers ----
    # Every step copies its hidden states from pinned host memory and its output back. The
    # copies run on their own streams, double-buffered, so step i+1's upload and step i-1's
    # download overlap step i's forward (how a serving loop feeds the block).
    # The host side of the loop runs on the CPUs nearest this GPU, so the pinned buffers
    # sit on its NUMA node (the CPU set is put back afterwards).
    from prism_infer_b200.engine.affinity import local_to_gpu
    with local_to_gpu(device) as local_cpus:
        x_host = [x.detach().cpu().pin_memory() for _ in range(2)]
        y_host = [torch.empty_like(x_host[0]).pin_memory() for _ in range(2)]
        x_dev = [torch.empty_like(x) for _ in range(2)]
        y_dev = [torch.empty_like(x) for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
        comp = torch.cuda.current_stream(device)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_done = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]
        for e in ev_done + ev_out:
            e.record(comp)

        def e2e_step(i, forward=True):
            b = i % 2
            s_in.wait_event(ev_done[b])          # x_dev[b] no longer read by step i-2
            with torch.cuda.stream(s_in):
                x_dev[b].copy_(x_host[b], non_blocking=True)
                ev_in[b].record(s_in)
            comp.wait_event(ev_in[b])
            if forward:
                with torch.inference_mode():
                    y = moe(x_dev[b])
            else:
                y = y_dev[b]
            ev_done[b].record(comp)
            s_out.wait_event(ev_done[b])
            s_out.wait_event(ev_out[b])          # y_host[b] free (step i-2's copy finished)
            with torch.cuda.stream(s_out):
                y_host[b].copy_(y, non_blocking=True)
                if forward:
                    y.record_stream(s_out)
                ev_out[b].record(s_out)

        def e2e_timed(forward):
            def fn(i):
                e2e_step(i, forward)
                if i == steps - 1 or i < 0:
                    comp.wait_stream(s_out)
            return fn

        ms_e2e = time_device(e2e_timed(True), steps, max(2, warmup // 2), world)
        e2e_value = world * T * steps / (ms_e2e / 1e3)
        ms_copy = time_device(e2e_timed(False), steps, max(2, warmup // 2), world)

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
        "parity": parity,
    }
    if world == 1:
        el = 2
        perm_bytes = T * H * el + rows * H * el + rows * 4
        comb_bytes = rows * H * el + T * H * el + rows * (4 + el)
        extra["hbm"] = {
            "permute_gbs": (perm_bytes / (stage_ms["permute"] / 1e3) / 1e9
                            if stage_ms["permute"] > 1e-3 else "fused into gate_up"),
            "combine_gbs": comb_bytes / (stage_ms["combine"] / 1e3) / 1e9,
            "route_gbs": (T * E * el + T * k * (8 + el)) / (stage_ms["route"] / 1e3) / 1e9,
            "peak_gbs": hbm_peak,
        }
    else:
        extra["a2a"] = a2a_stats(moe, x, world)
        # The fused launch computes and exchanges at once: its target time is the slower of its
        # FLOPs at the tensor peak and the bytes each rank's NVLink carries per direction (rows
        # other ranks pull from it + outputs it stores into them; by symmetry the same inbound)
        # at the measured peer-copy bandwidth.
        link_bytes = (extra["a2a"]["dispatch_remote_bytes_per_rank"]
                      + extra["a2a"]["return_remote_bytes_per_rank"])
        t_tensor = kflops / (peak * 1e12) * 1e3
        t_link = link_bytes / (NVLINK_GBS * 1e9) * 1e3
        roofline["fused_target"] = {
            "bound": "nvlink" if t_link > t_tensor else "tensor",
            "tensor_ms": t_tensor, "nvlink_ms": t_link, "target_ms": max(t_tensor, t_link),
            "launch_ms": kms, "frac": max(t_tensor, t_link) / kms,
            "nvlink_bytes_per_direction_per_rank": link_bytes, "link_gbs": NVLINK_GBS,
            "link_source": "measured peer copy per direction on this pool's B200s (NVLink 5, "
                           "900 GB/s nominal)"}

    # ---- config 1 decode (T=64 per rank) ----
    # At N=1 the whole step streams the experts' weights (HBM roofline); at N>1 the same batch
    # runs through the expert-parallel step. Both eager and replayed from a CUDA graph captured
    # once (the EP epoch is counted on the device, so the captured step replays as is).
    if not args.no_decode:
        xd = x[:64].contiguous()

        def dec(_i):
            with torch.inference_mode():
                moe(xd)
        ms_dec = time_device(dec, 200, 20, world)
        with torch.inference_mode():
            _, ids, _ = moe.route(xd)
        hit = reduce_over_ranks(torch.bincount(ids.reshape(-1), minlength=E).float().tolist(),
                                "sum", world)
        El = E // world
        n_exp = sum(1 for e in range(rank * El, (rank + 1) * El) if hit[e] > 0)
        n_exp = int(reduce_over_ranks([float(n_exp)], "max", world)[0])
        wbytes = n_exp * 3 * H * I * 2
        t_step = ms_dec / 200 / 1e3
        extra["decode_cfg1"] = {"tokens_per_rank": 64, "ms_per_step": ms_dec / 200,
                                "tokens_per_s": world * 64 / t_step,
                                "weight_bytes_per_step_per_rank": wbytes,
                                "hbm_gbs": wbytes / t_step / 1e9,
                                "frac_of_hbm_peak": wbytes / t_step / 1e9 / hbm_peak}
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side), torch.inference_mode():
            for _ in range(2):
                moe(xd)
        torch.cuda.current_stream(device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.inference_mode(), torch.cuda.graph(graph):
            moe(xd)
        ms_g = time_device(lambda _i: graph.replay(), 200, 20, world)
        extra["decode_cfg1"]["graph_ms_per_step"] = ms_g / 200
        extra["decode_cfg1"]["graph_tokens_per_s"] = world * 64 / (ms_g / 200 / 1e3)
        extra["decode_cfg1"]["graph_hbm_gbs"] = wbytes / (ms_g / 200 / 1e3) / 1e9
        extra["decode_cfg1"]["device_error_ranks"] = int(reduce_over_ranks(
            [float(check_device_error(moe, world, device) != 0)], "sum", world)[0])
        del graph

    if world == 1 and not args.no_ep1:
        extra["ep_path_1gpu"] = ep_path_one_gpu(moe, x, device, peak)

    free_block(moe, world)
    del x_dev, y_dev

    # ---- benchmark configs 3 and 4 at the same EP size ----
    if not args.no_extra_configs:
        for cid in (3, 4):
            extra[f"cfg{cid}"] = sub_config(cid, world, rank, device, peak)

    # ---- CPU baseline (rank 0, N=1) ----
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        from threadpoolctl import threadpool_info, threadpool_limits
        cores = host_threads()
        sample = 512
        with threadpool_limits(limits=cores):
            used = max([d.get("num_threads", 1) for d in threadpool_info()] or [1])
            rate, best = cpu_oracle_rate(sample, 2)
        cpu = {"value": rate, "unit": UNIT, "cores": used, "kind": "port",
               "sample": f"numpy port of MoE.forward, fp32, {sample} tokens of the workload, "
                         f"best of 2 ({best:.2f} s each), BLAS on {used} host threads"}

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": steps,
        "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(T, world),
        "roofline": roofline,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2,
                "copy_only_ms_per_step": ms_copy / steps,
                "ms_per_step": ms_e2e / steps,
                "host_cpus_near_gpu": local_cpus,
                "how": "MoE.forward; per step H2D of x from pinned host and D2H of the output, "
                       "on copy streams double-buffered against the forward; copy_only: the "
                       "same copies with no forward; host_cpus_near_gpu: CPUs the host loop "
                       "and the pinned buffers were placed on (NVML affinity; null: unchanged)"},
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
