"""Generate golden fixtures by running the REFERENCE's own MoE modules on CPU.

Usage (in a container where the reference source tree is available):

    PRISM_REFERENCE=/path/to/prism-infer python tests/golden/make_golden.py [rmsnorm]

(``rmsnorm`` writes only the RMSNorm fixtures.)

Writes ``tests/golden/*.npz``. Inputs are regenerated from seeds by
``prism_infer_b200.synthetic`` (numpy PCG64, platform independent); the reference modules
(``prism_infer.layers.moe.MoE``, ``prism_infer.engine.parallel.expert_parallel``) are loaded
with those weights and run in fp32 or bf16 on CPU. EP cases run W=2 / W=4 gloo ranks in
spawned processes, as the reference's own EP path does under torchrun.

The fixtures pin the numpy oracle (``oracle/moe_oracle.py``) to the reference; the GPU path
is then checked against the oracle.
"""
from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")  # SiluAndMul's torch.compile cannot build on CPU here

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from prism_infer_b200 import synthetic  # noqa: E402


def _ref_path() -> str:
    p = os.environ.get("PRISM_REFERENCE")
    if not p or not Path(p, "prism_infer").is_dir():
        raise SystemExit("set PRISM_REFERENCE to the reference source tree")
    return p


def _import_reference():
    sys.path.insert(0, _ref_path())
    import torch  # noqa: F401
    from prism_infer.layers.moe import MoE
    from prism_infer.engine.parallel import expert_parallel as ep
    return MoE, ep


def _load_single(moe, wts, dtype):
    import torch
    with torch.no_grad():
        moe.gate.weight.copy_(torch.from_numpy(wts.w_gate))
        for e, ex in enumerate(moe.experts):
            ex.gate_up_proj.weight.copy_(torch.from_numpy(wts.w_gate_up[e]))
            ex.down_proj.weight.copy_(torch.from_numpy(wts.w_down[e]))
    return moe.to(dtype)


# (name, H, E, k, I, T or shape, renorm, dtype, seed, skew)
SINGLE_CASES = [
    ("moe_fp32_small", 64, 16, 4, 32, 37, True, "float32", 11, False),
    ("moe_fp32_norenorm", 64, 16, 4, 32, 37, False, "float32", 12, False),
    ("moe_fp32_refshape", 16, 8, 2, 8, 6, True, "float32", 13, False),
    ("moe_fp32_empty_experts", 16, 32, 2, 8, 2, True, "float32", 14, False),
    ("moe_fp32_single_token", 16, 8, 2, 8, 1, True, "float32", 15, False),
    ("moe_fp32_multidim", 16, 8, 2, 8, (2, 3), True, "float32", 16, False),
    ("moe_fp32_k6", 64, 24, 6, 32, 20, True, "float32", 17, False),
    ("moe_fp32_skew", 64, 32, 4, 32, 64, True, "float32", 18, True),
    ("moe_bf16_small", 64, 16, 4, 32, 37, True, "bfloat16", 21, False),
    ("moe_bf16_k8", 128, 32, 8, 64, 48, True, "bfloat16", 22, False),
]


def run_single(MoE, name, H, E, k, I, T, renorm, dtype, seed, skew):
    import torch
    tdt = torch.float32 if dtype == "float32" else torch.bfloat16
    wts = synthetic.make_weights_np(H, E, I, seed, skew=skew, k=k)
    shape = T if isinstance(T, tuple) else (T,)
    ntok = int(np.prod(shape))
    x = synthetic.make_hidden_np(ntok, H, seed, skew=skew).reshape(*shape, H)
    moe = _load_single(MoE(H, I, E, k, norm_topk_prob=renorm), wts, tdt).eval()
    xt = torch.from_numpy(x).to(tdt)
    captured = {}

    def hook(_m, _inp, out):
        captured["logits"] = out.detach().float().numpy()
    h = moe.gate.register_forward_hook(hook)
    with torch.no_grad():
        out = moe(xt)
        logits = torch.from_numpy(captured["logits"]).to(tdt)
        rw = torch.softmax(logits, dim=-1, dtype=torch.float)
        w, ids = torch.topk(rw, k, dim=-1)
        if renorm:
            w = w / w.sum(dim=-1, keepdim=True)
        w = w.to(tdt)
    h.remove()
    rec = dict(H=H, E=E, k=k, I=I, shape=np.array(shape), renorm=renorm, dtype=dtype, seed=seed,
               skew=skew, logits=captured["logits"], topk_ids=ids.numpy().astype(np.int64),
               topk_weights=w.float().numpy(), out=out.float().numpy())
    if H * E * I <= 64 * 64 * 64:   # small cases keep their inputs for independent checks
        rec["x"] = x
    return rec


def run_cfg0(MoE):
    """Benchmark config 0 (T=256, H=2048, E=128, k=8, I=768, fp32) through the reference."""
    import torch
    c = synthetic.CONFIGS[0]
    seed = synthetic.config_seed(0)
    wts = synthetic.make_weights_np(c["H"], c["E"], c["I"], seed)
    x = synthetic.make_hidden_np(c["T"], c["H"], seed)
    moe = _load_single(MoE(c["H"], c["I"], c["E"], c["k"], True), wts, torch.float32).eval()
    captured = {}
    def hook(_m, _inp, out):
        captured["logits"] = out.detach().numpy()
    h = moe.gate.register_forward_hook(hook)
    with torch.no_grad():
        out = moe(torch.from_numpy(x)).numpy()
        rw = torch.softmax(torch.from_numpy(captured["logits"]), dim=-1, dtype=torch.float)
        w, ids = torch.topk(rw, c["k"], dim=-1)
        w = w / w.sum(dim=-1, keepdim=True)
    h.remove()
    return dict(H=c["H"], E=c["E"], k=c["k"], I=c["I"], shape=np.array([c["T"]]), renorm=True,
                dtype="float32", seed=seed, skew=False, topk_ids=ids.numpy().astype(np.int64),
                topk_weights=w.numpy(), out_rows=out[:16].copy(), out_row_sums=out.sum(axis=1),
                out_abs_sums=np.abs(out).sum(axis=1))


# ---------------------------------------------------------------- EP cases (gloo ranks)

EP_CASES = [
    # name, W, H, E, k, I, T per rank (list), dtype, seed
    ("ep2_fp32", 2, 64, 16, 4, 32, [10, 13], "float32", 31),
    ("ep4_fp32", 4, 64, 16, 4, 32, [10, 7, 12, 9], "float32", 32),
    ("ep4_tiny", 4, 32, 8, 2, 16, [1, 1, 2, 1], "float32", 33),
    ("ep2_bf16", 2, 64, 16, 4, 32, [24, 24], "bfloat16", 34),
]


def _ep_worker(rank, W, port, case, qdir):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=W)
    MoE, ep = _import_reference()
    name, W_, H, E, k, I, Ts, dtype, seed = case
    tdt = torch.float32 if dtype == "float32" else torch.bfloat16
    ep.set_expert_parallel_size(W)
    wts = synthetic.make_weights_np(H, E, I, seed)
    moe = MoE(H, I, E, k, norm_topk_prob=True)
    El = E // W
    with torch.no_grad():
        moe.gate.weight.copy_(torch.from_numpy(wts.w_gate))
        for le, ex in enumerate(moe.ep_moe.local_experts):
            ex.gate_up_proj.weight.copy_(torch.from_numpy(wts.w_gate_up[rank * El + le]))
            ex.down_proj.weight.copy_(torch.from_numpy(wts.w_down[rank * El + le]))
    moe = moe.to(tdt).eval()
    x = synthetic.make_hidden_np(Ts[rank], H, seed + 100 * (rank + 1))
    rec = {}
    orig_a2a = moe.ep_moe._all_to_all
    calls = []

    def spy(t, out_splits, in_splits):
        r = orig_a2a(t, out_splits, in_splits)
        calls.append((r.detach().float().numpy().copy(), list(out_splits)))
        return r
    moe.ep_moe._all_to_all = spy
    cap = {}
    def hook(_m, _inp, out):
        cap["logits"] = out.detach().float().numpy()
    moe.gate.register_forward_hook(hook)
    with torch.no_grad():
        out = moe(torch.from_numpy(x).to(tdt))
        logits = torch.from_numpy(cap["logits"]).to(tdt)
        rw = torch.softmax(logits, dim=-1, dtype=torch.float)
        w, ids = torch.topk(rw, k, dim=-1)
        w = (w / w.sum(dim=-1, keepdim=True)).to(tdt)
        perm, splits, sleid = ep.build_dispatch_plan(ids, El, W)
    rec.update(x=x, logits=cap["logits"], topk_ids=ids.numpy().astype(np.int64),
               topk_weights=w.float().numpy(), perm=perm.numpy().astype(np.int64),
               input_splits=splits.numpy().astype(np.int64),
               sorted_local_eid=sleid.numpy().astype(np.int64),
               output_splits=np.array(calls[0][1], np.int64),
               recv_eid=calls[1][0].astype(np.int64), out=out.float().numpy())
    np.savez(Path(qdir) / f"rank{rank}.npz", **rec)
    dist.barrier()
    dist.destroy_process_group()


def run_ep(case):
    import tempfile
    import torch.multiprocessing as mp
    W = case[1]
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as qdir:
        mp.start_processes(_ep_worker, args=(W, port, case, qdir), nprocs=W, join=True,
                           start_method="spawn")
        per_rank = [dict(np.load(Path(qdir) / f"rank{r}.npz")) for r in range(W)]
    name, W, H, E, k, I, Ts, dtype, seed = case
    rec = dict(W=W, H=H, E=E, k=k, I=I, Ts=np.array(Ts), dtype=dtype, seed=seed)
    for r, d in enumerate(per_rank):
        for key, v in d.items():
            rec[f"r{r}_{key}"] = v
    return rec


# (name, T, H, dtype, eps, seed): the decoder layer's RMSNorm (prism_infer/layers/layernorm.py),
# run eagerly (its torch.compile is disabled here, as above)
NORM_CASES = [
    ("rmsnorm_fp32", 33, 256, "float32", 1e-6, 41),
    ("rmsnorm_bf16", 8, 2048, "bfloat16", 1e-6, 42),
    ("rmsnorm_bf16_eps", 5, 64, "bfloat16", 1e-2, 43),
]


def run_rmsnorm(name, T, H, dtype, eps, seed):
    sys.path.insert(0, _ref_path())
    import torch
    from prism_infer.layers.layernorm import RMSNorm
    tdt = torch.float32 if dtype == "float32" else torch.bfloat16
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((T, H), dtype=np.float32) * 2).astype(np.float32)
    res = rng.standard_normal((T, H), dtype=np.float32)
    w = (1 + 0.25 * rng.standard_normal(H, dtype=np.float32)).astype(np.float32)
    norm = RMSNorm(H, eps=eps)
    with torch.no_grad():
        norm.weight.copy_(torch.from_numpy(w))
    norm = norm.to(tdt)
    xt, rt = torch.from_numpy(x).to(tdt), torch.from_numpy(res).to(tdt)
    with torch.no_grad():
        rms = norm(xt.clone())
        add, add_res = norm(xt.clone(), rt.clone())
    f = lambda t: t.detach().float().numpy()
    return dict(x=f(xt), residual=f(rt), weight=f(norm.weight), eps=np.float32(eps),
                dtype=dtype, rms_out=f(rms), add_out=f(add), add_residual=f(add_res))


def main():
    only = sys.argv[1:]
    if only == ["rmsnorm"]:
        for case in NORM_CASES:
            np.savez_compressed(HERE / f"{case[0]}.npz", **run_rmsnorm(*case))
            print("wrote", case[0])
        return
    MoE, _ = _import_reference()
    import torch
    torch.manual_seed(0)
    for case in NORM_CASES:
        np.savez_compressed(HERE / f"{case[0]}.npz", **run_rmsnorm(*case))
        print("wrote", case[0])
    for case in SINGLE_CASES:
        rec = run_single(MoE, *case)
        np.savez_compressed(HERE / f"{case[0]}.npz", **rec)
        print("wrote", case[0])
    np.savez_compressed(HERE / "cfg0.npz", **run_cfg0(MoE))
    print("wrote cfg0")
    for case in EP_CASES:
        np.savez_compressed(HERE / f"{case[0]}.npz", **run_ep(case))
        print("wrote", case[0])


if __name__ == "__main__":
    main()
