"""The ``torch.ops.prism_moe.*`` custom operators: registered, with fake implementations that
give the right shapes and dtypes without a GPU (what torch.compile / torch.export trace
through), and a ``MoE`` module that traces in one graph. Nothing here launches a kernel."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from prism_infer_b200 import ops  # noqa: F401  (registers the ops)

OPS = ("route_topk", "dispatch_plan", "permute_rows", "combine", "expert_swiglu",
       "block_forward", "ep_forward", "rmsnorm", "add_rmsnorm", "block_forward_norm",
       "ep_forward_norm")


def test_ops_are_registered():
    for name in OPS:
        assert hasattr(torch.ops.prism_moe, name), name


def test_fake_shapes():
    T, H, E, k, I, W = 37, 64, 16, 4, 32, 4
    with FakeTensorMode():
        dev = "cuda"
        x = torch.empty(T, H, device=dev, dtype=torch.bfloat16)
        logits = torch.empty(T, E, device=dev, dtype=torch.bfloat16)
        ids, w = torch.ops.prism_moe.route_topk(logits, k, True)
        assert ids.shape == (T, k) and ids.dtype == torch.int64
        assert w.shape == (T, k) and w.dtype == torch.bfloat16
        perm, splits, sleid, counts, offsets, entry_row = torch.ops.prism_moe.dispatch_plan(
            ids, E, W)
        assert perm.shape == (T * k,) and perm.dtype == torch.int64
        assert splits.shape == (W,) and sleid.shape == (T * k,)
        assert counts.shape == (E,) and counts.dtype == torch.int32
        assert offsets.shape == (E + 1,) and entry_row.shape == (T * k,)
        xs = torch.ops.prism_moe.permute_rows(x, k, entry_row)
        assert xs.shape == (T * k, H) and xs.dtype == x.dtype
        wgu = torch.empty(E, 2 * I, H, device=dev, dtype=torch.bfloat16)
        wd = torch.empty(E, H, I, device=dev, dtype=torch.bfloat16)
        y = torch.ops.prism_moe.expert_swiglu(xs, offsets, wgu, wd, None)
        assert y.shape == xs.shape
        out = torch.ops.prism_moe.combine(y, w, entry_row)
        assert out.shape == (T, H) and out.dtype == x.dtype
        blk = torch.ops.prism_moe.block_forward(x, logits, wgu, wd, k, True)
        assert blk.shape == x.shape and blk.dtype == x.dtype
        nw = torch.empty(H, device=dev, dtype=torch.bfloat16)
        assert torch.ops.prism_moe.rmsnorm(x, nw, 1e-6).shape == x.shape
        o, r = torch.ops.prism_moe.add_rmsnorm(x, x, nw, 1e-6)
        assert o.shape == r.shape == x.shape
        o, r = torch.ops.prism_moe.block_forward_norm(x, logits, wgu, wd, k, True, x, nw, 1e-6)
        assert o.shape == r.shape == x.shape and o.dtype == x.dtype


def test_moe_exports_as_one_graph():
    """torch.export (strict tracing through the fake implementations) of the drop-in ``MoE`` on
    meta tensors: one graph with the router GEMM and the block op."""
    from prism_infer_b200.engine.parallel import set_expert_parallel_size
    from prism_infer_b200.layers.moe import MoE
    set_expert_parallel_size(1)
    H, E, k, I = 64, 16, 4, 32
    moe = MoE(H, I, E, k).to("meta", torch.bfloat16)
    x = torch.empty(2, 5, H, device="meta", dtype=torch.bfloat16)
    y = moe(x)
    assert y.shape == x.shape and y.dtype == x.dtype
    ep = torch.export.export(moe, (x,))
    called = [str(n.target) for n in ep.graph.nodes if n.op == "call_function"]
    assert "aten.linear.default" in called
    assert "prism_moe.block_forward.default" in called


def test_cpu_tensors_raise():
    x = torch.zeros(4, 8, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        torch.ops.prism_moe.route_topk(x, 2, True)


def test_decoder_layer_fusion_exports_as_one_graph():
    """post_attention_layernorm (the drop-in RMSNorm) -> MoE with the next layer's
    input_layernorm fused into its combine, exported on meta tensors."""
    from torch import nn

    from prism_infer_b200.engine.parallel import set_expert_parallel_size
    from prism_infer_b200.layers.layernorm import RMSNorm
    from prism_infer_b200.layers.moe import MoE
    set_expert_parallel_size(1)
    H, E, k, I = 64, 16, 4, 32

    class Tail(nn.Module):
        def __init__(self):
            super().__init__()
            self.post_attention_layernorm = RMSNorm(H)
            self.mlp = MoE(H, I, E, k)
            self.next_input_layernorm = RMSNorm(H)

        def forward(self, hidden, residual):
            hidden, residual = self.post_attention_layernorm(hidden, residual)
            return self.mlp(hidden, residual=residual, norm=self.next_input_layernorm)

    tail = Tail().to("meta", torch.bfloat16)
    x = torch.empty(7, H, device="meta", dtype=torch.bfloat16)
    out, res = tail(x, x)
    assert out.shape == res.shape == x.shape
    ep = torch.export.export(tail, (x, x))
    called = [str(n.target) for n in ep.graph.nodes if n.op == "call_function"]
    assert "prism_moe.add_rmsnorm.default" in called
    assert "prism_moe.block_forward_norm.default" in called
