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


def _receive_layout_model(ids_per_rank, E, W, k):
    """The receive buffers the NVLink transport builds, restated on the host from the index
    arithmetic of ep_counts_kernel (segment offsets, source rows of each segment, tokens and copy
    chunks per slot) and of the fused launch's copy warps (own rows by plan row, other sources'
    rows pulled token by token). Returns, per rank, an array mapping each receive row to the
    (source rank, token) whose row it holds (-1: never written), plus the rows each rank pulls."""
    from oracle import moe_oracle as O
    El = E // W
    counts = [O.expert_counts(ids, E) for ids in ids_per_rank]           # C[s][e]
    tokens = [ids.shape[0] for ids in ids_per_rank]
    entry_rows = []
    for ids in ids_per_rank:                     # the source's plan: expert-major row of entry f
        order = O.expert_major_order(ids, E)
        er = np.empty(order.size, np.int64)
        er[order] = np.arange(order.size)
        entry_rows.append(er)
    offsets = [np.concatenate([[0], np.cumsum(c)]) for c in counts]
    layouts, pulled = [], []
    for me in range(W):
        seg_rows = [counts[(me - j) % W][me * El + le] for j in range(W) for le in range(El)]
        seg_off = np.concatenate([[0], np.cumsum(seg_rows)])
        seg_src_row = [offsets[(me - j) % W][me * El + le] for j in range(W) for le in range(El)]
        recv = np.full(int(seg_off[-1]), -1, np.int64)
        src_of = np.full(int(seg_off[-1]), -1, np.int64)
        tpc = 32 // k
        chunk_base = [0, -(-int(sum(counts[me][me * El:(me + 1) * El])) // 32)]
        for j in range(1, W):
            chunk_base.append(chunk_base[-1] - (-tokens[(me - j) % W] // tpc))
        # slot 0: own rows, by expert-major plan row
        ids, er = ids_per_rank[me], entry_rows[me]
        for q in range(offsets[me][me * El], offsets[me][(me + 1) * El]):
            f = int(np.nonzero(er == q)[0][0])
            e = int(ids.reshape(-1)[f])
            dst = seg_off[e - me * El] + (q - offsets[me][e])
            assert recv[dst] == -1
            recv[dst], src_of[dst] = f // k, me
        # slots j >= 1: pulled token by token, chunks of 32 // k tokens
        n_pulled = 0
        for j in range(1, W):
            s = (me - j) % W
            n_chunks = chunk_base[j + 1] - chunk_base[j]
            for c in range(n_chunks):
                for t in range(c * tpc, min((c + 1) * tpc, tokens[s])):
                    hit = False
                    for jj in range(k):
                        f = t * k + jj
                        e = int(ids_per_rank[s].reshape(-1)[f])
                        if me * El <= e < (me + 1) * El:
                            seg = j * El + e - me * El
                            dst = seg_off[seg] + (entry_rows[s][f] - seg_src_row[seg])
                            assert recv[dst] == -1
                            recv[dst], src_of[dst] = t, s
                            hit = True
                    n_pulled += hit
        layouts.append((recv, src_of, seg_off))
        pulled.append(n_pulled)
    return layouts, pulled


@pytest.mark.parametrize("W,k,T", [(2, 8, 67), (3, 8, 50), (4, 6, 41), (8, 8, 37), (8, 2, 9)])
def test_pulled_receive_layout_matches_reference_order(W, k, T):
    """The receive layout of the NVLink transport, from the kernels' index arithmetic, holds in
    segment (slot j, local expert le) exactly the rows the reference's all_to_all delivers to
    rank me from source (me - j) mod W for expert me*El + le, in the reference's order (flat
    order inside an expert, expert_parallel.py:37-39), every row written once; and a token row
    is pulled once per owner rank however many of its experts that owner holds."""
    E = 8 * W
    rng = np.random.default_rng(W * 100 + k)
    ids_per_rank = [np.stack([rng.choice(E, k, replace=False) for _ in range(T + r)])
                    for r in range(W)]
    layouts, pulled = _receive_layout_model(ids_per_rank, E, W, k)
    El = E // W
    for me in range(W):
        recv, src_of, seg_off = layouts[me]
        assert (recv >= 0).all()
        for j in range(W):
            s = (me - j) % W
            flat = ids_per_rank[s].reshape(-1)
            for le in range(El):
                e = me * El + le
                want = np.nonzero(flat == e)[0] // k          # tokens, flat order
                a, b = seg_off[j * El + le], seg_off[j * El + le + 1]
                assert np.array_equal(recv[a:b], want)
                assert (src_of[a:b] == s).all()
        want_pulled = sum(int(np.any((ids_per_rank[(me - j) % W] >= me * El) &
                                     (ids_per_rank[(me - j) % W] < (me + 1) * El), axis=1).sum())
                          for j in range(1, W))
        assert pulled[me] == want_pulled
