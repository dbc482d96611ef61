"""Host-side checks of the drop-in modules (no GPU): parameter names and the checkpoint-loading
contract that prism_infer/utils/loader.py:63-88 relies on (``param.weight_loader(param, w)`` or
``param.weight_loader(param, w, shard_id)`` for packed modules)."""
import torch

from prism_infer_b200.layers.mlp import Qwen3MLP
from prism_infer_b200.layers.moe import MoE


def test_dense_mlp_parameter_names_and_loaders():
    H, I = 64, 48
    m = Qwen3MLP(H, I, "silu")
    assert set(dict(m.named_parameters())) == {"gate_up_proj.weight", "down_proj.weight"}
    gate = torch.randn(I, H)
    up = torch.randn(I, H)
    down = torch.randn(H, I)
    p = m.gate_up_proj.weight
    p.weight_loader(p, gate, 0)      # packed_modules_mapping: gate_proj -> shard 0
    p.weight_loader(p, up, 1)        #                        up_proj   -> shard 1
    q = m.down_proj.weight
    q.weight_loader(q, down)
    assert torch.equal(m.gate_up_proj.weight[:I], gate)
    assert torch.equal(m.gate_up_proj.weight[I:], up)
    assert torch.equal(m.down_proj.weight, down)


def test_dense_mlp_rejects_other_activations():
    try:
        Qwen3MLP(64, 48, "gelu")
    except AssertionError:
        return
    raise AssertionError("hidden_act other than silu must be rejected, as in the reference")


def test_moe_expert_views_write_stacked_storage():
    H, I, E, k = 32, 16, 4, 2
    moe = MoE(H, I, E, k)
    names = set(dict(moe.named_parameters()))
    assert "gate.weight" in names
    assert {f"experts.{e}.gate_up_proj.weight" for e in range(E)} <= names
    assert {f"experts.{e}.down_proj.weight" for e in range(E)} <= names
    w = torch.randn(I, H)
    p = moe.experts[2].gate_up_proj.weight
    p.weight_loader(p, w, 1)
    assert torch.equal(moe.w_gate_up[2, I:], w)
    d = torch.randn(H, I)
    q = moe.experts[3].down_proj.weight
    q.weight_loader(q, d)
    assert torch.equal(moe.w_down[3], d)
