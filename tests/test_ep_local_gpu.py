"""The expert-parallel step on ONE GPU: ``prism_moe_ep_forward`` with ep_size 1 (the same kernels
as at EP>1 — counts exchange, fused expert launch with its copy warps, return wait, combine —
against this rank's own landing zone), and what only needs one GPU to check:

* parity with the oracle (routing bit-exact, outputs within the bf16 tolerance);
* the step captured once in a CUDA graph and replayed (the epoch is counted on the device;
  the reference's decode capture, prism_infer/engine/model_runner.py:281-318);
* caller-given expert ids outside [0, E): nothing is sent for them, their slots add nothing and
  the step reports PRISM_MOE_ERR_ARG (the reference raises on such ids:
  prism_infer/engine/parallel/expert_parallel.py:37-40 bincount / all_to_all);
* a peer that never arrives: two landing zones on this GPU stand for a group of two ranks whose
  second rank never runs; with a 20 ms bound the counts exchange gives up, the step reports
  PRISM_MOE_ERR_TIMEOUT, its later kernels do nothing, and the GPU stays usable;
* the step statistics (dispatch window, rows sent / received).
"""
import numpy as np
import pytest
import torch

from oracle import moe_oracle as O
from prism_infer_b200 import capi, synthetic
from prism_infer_b200.engine.parallel.expert_parallel import ExpertParallelMoE

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_MAX_ABS, BF16_MEAN_REL = 2e-2, 1e-2


def _np(t):
    return t.detach().float().cpu().numpy()


def make_bank(H, E, I, seed):
    wts = synthetic.make_weights_np(H, E, I, seed)
    bank = ExpertParallelMoE(H, I, E, 1, 0, transport="p2p")
    with torch.no_grad():
        bank.w_gate_up.copy_(torch.from_numpy(wts.w_gate_up))
        bank.w_down.copy_(torch.from_numpy(wts.w_down))
    bank = bank.to(DEV, torch.bfloat16)
    w_gate = torch.from_numpy(wts.w_gate).to(DEV, torch.bfloat16)
    return bank, w_gate, wts


def check_close(got, ref):
    d = np.abs(got - ref)
    assert d.max() <= BF16_MAX_ABS, d.max()
    assert d.mean() / max(np.abs(ref).mean(), 1e-12) <= BF16_MEAN_REL


@pytest.mark.parametrize("H,E,k,I,T", [(256, 32, 8, 128, 300), (2048, 128, 8, 768, 1024)])
def test_ep1_step_matches_oracle(H, E, k, I, T):
    bank, w_gate, wts = make_bank(H, E, I, seed=H + T)
    x = synthetic.make_hidden_np(T, H, seed=H + T)
    xt = torch.from_numpy(x).to(DEV, torch.bfloat16)
    with torch.inference_mode():
        logits = torch.nn.functional.linear(xt, w_gate)
        out = bank.forward_p2p(xt, router_logits=logits, top_k=k)
        out2 = bank.forward_p2p(xt, router_logits=logits, top_k=k)   # the other parity
    bank.check_device_error()
    assert torch.equal(out, out2)
    ref = O.ep_forward_all_ranks([x], wts.w_gate, wts.w_gate_up, wts.w_down, k, True,
                                 "bfloat16", logits=[_np(logits)])[0]
    check_close(_np(out), ref["out"])
    st = bank.step_stats()
    assert st["epoch"] == st["counter"] == 2
    assert st["send_rows"] == 0 and st["recv_rows"] == 0          # one rank: nothing crosses
    assert 0 < st["dispatch_t0_ns"] <= st["dispatch_t1_ns"]
    assert 0 < st["fused_t0_ns"] < st["fused_t1_ns"]
    bank.release()


def test_ep1_step_replays_from_cuda_graph():
    H, E, k, I, T = 512, 64, 8, 256, 256
    bank, w_gate, _ = make_bank(H, E, I, seed=5)
    xs = [torch.randn(T, H, device=DEV).to(torch.bfloat16) for _ in range(3)]
    x_in = xs[0].clone()
    with torch.inference_mode():
        eager = []
        for x in xs:                              # first call reserves the landing zone
            eager.append(bank.forward_p2p(x, router_logits=torch.nn.functional.linear(x, w_gate),
                                          top_k=k))
        torch.cuda.synchronize()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            bank.forward_p2p(x_in, router_logits=torch.nn.functional.linear(x_in, w_gate), top_k=k)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            y = bank.forward_p2p(x_in, router_logits=torch.nn.functional.linear(x_in, w_gate),
                                 top_k=k)
        before = bank.step_stats()["counter"]
        for rep in range(2):
            for x, ref in zip(xs, eager):
                x_in.copy_(x)
                graph.replay()
                torch.cuda.synchronize()
                assert torch.equal(y, ref), rep
    bank.check_device_error()
    assert bank.step_stats()["counter"] == before + 6      # every replay took a new epoch
    del graph
    bank.release()


def test_ep1_out_of_range_ids_send_nothing_and_report():
    H, E, k, I, T = 256, 32, 4, 128, 200
    bank, w_gate, _ = make_bank(H, E, I, seed=9)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    logits = torch.nn.functional.linear(x, w_gate)
    ids, w, _ = capi.route_topk(logits.contiguous(), k, True)
    bad = ids.clone()
    bad[3, 1] = -1
    bad[17, 0] = E
    bad[150, 3] = 1 << 40
    with torch.inference_mode():
        got = bank.forward_p2p(x, topk_ids=bad, topk_weights=w)
    with pytest.raises(RuntimeError, match="status 1"):
        bank.check_device_error()
    # the same step with those slots pointed at a valid expert with weight 0
    ok_ids, ok_w = bad.clone(), w.clone()
    for t, j in ((3, 1), (17, 0), (150, 3)):
        ok_ids[t, j] = 0
        ok_w[t, j] = 0
    with torch.inference_mode():
        ref = bank.forward_p2p(x, topk_ids=ok_ids, topk_weights=ok_w)
    bank.check_device_error()
    assert torch.equal(got, ref)
    bank.release()


def test_dispatch_plan_reports_out_of_range_ids():
    ids = torch.tensor([[0, 3], [5, -2], [1, 7]], dtype=torch.int64, device=DEV)
    lib = capi.load()
    ws_bytes = lib.prism_moe_dispatch_workspace_size(3, 2, 8, 2)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=DEV)
    plan = capi.dispatch_plan(ids.clamp(0, 7), 8, 2)         # valid ids: no error
    entry_row = torch.full((6,), 99, dtype=torch.int32, device=DEV)
    counts = torch.empty(8, dtype=torch.int32, device=DEV)
    capi.check(lib.prism_moe_build_dispatch_plan(
        ids.data_ptr(), 3, 2, 8, 2, None, None, None, counts.data_ptr(), None,
        entry_row.data_ptr(), ws.data_ptr(), ws_bytes, capi.stream_of(ids.device)), "plan")
    assert capi.read_device_error(ws[:4].view(torch.int32)) == capi.ERR_ARG
    assert capi.read_device_error(ws[:4].view(torch.int32)) == capi.OK     # read clears it
    assert entry_row[3].item() == -1
    assert counts.sum().item() == 5
    assert plan["expert_counts"].sum().item() == 6


def test_peer_that_never_arrives_times_out_and_the_gpu_stays_usable():
    lib = capi.load()
    H, E, k, I, T, W = 256, 16, 4, 128, 64, 2
    El = E // W
    max_tokens = 256
    land_bytes = lib.prism_moe_ep_landing_bytes(W, max_tokens, k, H, E, capi.BF16)
    ws_bytes = lib.prism_moe_ep_workspace_size(max_tokens, H, I, E, k, W, capi.BF16)
    assert land_bytes > 0 and ws_bytes > 0
    zones = [capi.ep_alloc_landing(land_bytes)[0] for _ in range(W)]   # rank 1 never runs
    try:
        table = torch.tensor(zones, dtype=torch.int64, device=DEV)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=DEV)
        x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
        logits = torch.randn(T, E, device=DEV).to(torch.bfloat16)
        wgu = (torch.randn(El, 2 * I, H, device=DEV) / 16).to(torch.bfloat16)
        wd = (torch.randn(El, H, I, device=DEV) / 11).to(torch.bfloat16)
        out = torch.zeros_like(x)
        capi.set_wait_limits(0, 20_000_000)                   # 20 ms for waits on other ranks
        try:
            st = lib.prism_moe_ep_forward(
                x.data_ptr(), logits.data_ptr(), None, None, capi.BF16, T, max_tokens, H, I, E,
                k, 1, W, 0, wgu.data_ptr(), wd.data_ptr(), zones[0], table.data_ptr(), 0,
                out.data_ptr(), ws.data_ptr(), ws_bytes, capi.stream_of(x.device))
            capi.check(st, "prism_moe_ep_forward")
            err = capi.read_device_error(ws[:4].view(torch.int32))
        finally:
            capi.set_wait_limits(0, 0)
        assert err == capi.ERR_TIMEOUT
        stats = capi.ep_read_stats(ws)
        assert stats["epoch"] == 1 and stats["fused_t1_ns"] == 0     # the experts never ran
    finally:
        torch.cuda.synchronize()
        for z in zones:
            capi.check(lib.prism_moe_ep_free_landing(z), "free landing")
    # the context is intact: a normal one-rank step still gives the right answer
    test_ep1_step_matches_oracle(256, 32, 8, 128, 300)
