"""Expert-parallel host logic on CPU: W=2 and W=4 gloo ranks (no GPU).

``ExpertParallelMoE.forward`` orchestrates plan -> permute -> counts exchange -> all-to-all ->
grouped experts -> reverse all-to-all -> combine. Here its kernel calls are served by
oracle-backed stand-ins on CPU tensors, so the distributed logic — split sizes, segment table,
receive layout, un-permutation — is checked against the outputs the REFERENCE's own
ExpertParallelMoE produced under gloo (tests/golden/ep*_fp32.npz).
"""
import os
import socket
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import load_golden

REPO = Path(__file__).resolve().parent.parent


class OracleKernels:
    """CPU stand-ins with the signatures of prism_infer_b200.capi used by the EP module."""

    @staticmethod
    def dispatch_plan(topk_ids, num_experts, ep_size, want_perm=True):
        from oracle import moe_oracle as O
        ids = topk_ids.numpy()
        order = O.expert_major_order(ids, num_experts)
        entry_row = np.empty_like(order)
        entry_row[order] = np.arange(order.size)
        counts = O.expert_counts(ids, num_experts)
        out = dict(entry_row=torch.from_numpy(entry_row.astype(np.int32)),
                   expert_counts=torch.from_numpy(counts.astype(np.int32)),
                   expert_offsets=torch.from_numpy(
                       np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)))
        if want_perm:
            perm, splits, sleid = O.build_dispatch_plan(ids, num_experts // ep_size, ep_size)
            out.update(perm=torch.from_numpy(perm), input_splits=torch.from_numpy(splits),
                       sorted_local_eid=torch.from_numpy(sleid))
        return out

    @staticmethod
    def permute_rows(x, top_k, entry_row, out=None):
        order = torch.empty_like(entry_row.long())
        order[entry_row.long()] = torch.arange(entry_row.numel())
        return x[order // top_k].contiguous()

    @staticmethod
    def expert_swiglu(x_sorted, seg_offsets, w_gate_up, w_down, seg_expert=None, y=None,
                      device_error=None):
        from oracle import moe_oracle as O
        dt = "float32" if x_sorted.dtype == torch.float32 else "bfloat16"
        out = torch.zeros_like(x_sorted)
        off = seg_offsets.tolist()
        for s in range(len(off) - 1):
            a, b = off[s], off[s + 1]
            if a == b:
                continue
            e = int(seg_expert[s]) if seg_expert is not None else s
            out[a:b] = torch.from_numpy(O.expert_mlp(x_sorted[a:b].float().numpy(),
                                                     w_gate_up[e].float().numpy(),
                                                     w_down[e].float().numpy(), dt))
        return out

    @staticmethod
    def combine(expert_out, topk_weights, entry_row=None, out=None):
        from oracle import moe_oracle as O
        T, k = topk_weights.shape
        rows = entry_row.long() if entry_row is not None else torch.arange(T * k)
        dt = "float32" if expert_out.dtype == torch.float32 else "bfloat16"
        res = O.combine_weighted_sum(expert_out[rows].float().numpy(),
                                     topk_weights.float().numpy(), T, k, dt)
        return torch.from_numpy(res).to(expert_out.dtype)


def _worker(rank, W, port, name, outdir):
    import sys
    sys.path.insert(0, str(REPO))
    sys.path.insert(0, str(REPO / "tests"))
    import torch.distributed as dist

    from prism_infer_b200 import synthetic
    from prism_infer_b200.engine.parallel import expert_parallel as ep
    from test_ep_host import OracleKernels
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=W, timeout=timedelta(seconds=60))
    g = load_golden(name)
    H, E, k, I = (int(g[n]) for n in ("H", "E", "k", "I"))
    wts = synthetic.make_weights_np(H, E, I, int(g["seed"]))
    ep._KERNELS = OracleKernels
    El = E // W
    m = ep.ExpertParallelMoE(H, I, E, W, rank)
    with torch.no_grad():
        m.w_gate_up.copy_(torch.from_numpy(wts.w_gate_up[rank * El:(rank + 1) * El]))
        m.w_down.copy_(torch.from_numpy(wts.w_down[rank * El:(rank + 1) * El]))
    x = torch.from_numpy(g[f"r{rank}_x"])
    ids = torch.from_numpy(g[f"r{rank}_topk_ids"])
    w = torch.from_numpy(g[f"r{rank}_topk_weights"])
    out = m(x, ids, w)
    recv_counts, in_splits, out_splits = m.exchange_plan(
        OracleKernels.dispatch_plan(ids, E, W, want_perm=False)["expert_counts"])
    np.savez(Path(outdir) / f"r{rank}.npz", out=out.numpy(), out_splits=np.array(out_splits),
             in_splits=np.array(in_splits), recv_counts=recv_counts.numpy())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("name", ["ep2_fp32", "ep4_fp32", "ep4_tiny"])
def test_ep_host_logic_reproduces_reference_ep(name):
    import torch.multiprocessing as mp
    g = load_golden(name)
    W = int(g["W"])
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_worker, args=(W, port, name, d), nprocs=W, join=True,
                           start_method="spawn")
        res = [dict(np.load(Path(d) / f"r{r}.npz")) for r in range(W)]
    for r in range(W):
        # split sizes equal the reference's (output_splits of its counts exchange)
        assert res[r]["out_splits"].tolist() == g[f"r{r}_output_splits"].tolist()
        assert res[r]["in_splits"].tolist() == g[f"r{r}_input_splits"].tolist()
        # received rows per local expert equal the reference's received expert ids
        ref_recv = np.bincount(g[f"r{r}_recv_eid"], minlength=res[r]["recv_counts"].shape[1])
        assert (res[r]["recv_counts"].sum(0) == ref_recv).all()
        np.testing.assert_allclose(res[r]["out"], g[f"r{r}_out"], atol=1e-5, rtol=1e-4)
