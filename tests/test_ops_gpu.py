"""``torch.compile(fullgraph=True)`` over a module that contains the drop-in ``MoE``: the custom
ops (``torch.ops.prism_moe.*``) trace as single graph nodes and run the CUDA kernels; the
compiled module matches the oracle (routing bit-exact on the logits the compiled graph
computed, outputs within the bf16 tolerance) and the eager module."""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import moe_oracle as O
from prism_infer_b200 import synthetic
from prism_infer_b200.engine.parallel import set_expert_parallel_size
from prism_infer_b200.layers.moe import MoE

pytestmark = pytest.mark.gpu
BF16_MAX_ABS, BF16_MEAN_REL = 2e-2, 1e-2


class ScaledMoE(nn.Module):
    """Some ordinary torch work around the block, so the compiled graph holds more than the op."""

    def __init__(self, moe):
        super().__init__()
        self.moe = moe

    def forward(self, x):
        h = x * 0.5 + 0.25
        return self.moe(h), self.moe.gate(h)


@pytest.mark.parametrize("backend", ["aot_eager", "inductor"])
def test_compiled_block_matches_oracle(backend):
    torch._dynamo.reset()
    set_expert_parallel_size(1)
    H, E, k, I, T = 512, 64, 8, 256, 300
    wts = synthetic.make_weights_np(H, E, I, seed=31)
    moe = MoE(H, I, E, k)
    with torch.no_grad():
        moe.gate.weight.copy_(torch.from_numpy(wts.w_gate))
        moe.w_gate_up.copy_(torch.from_numpy(wts.w_gate_up))
        moe.w_down.copy_(torch.from_numpy(wts.w_down))
    mod = ScaledMoE(moe.to("cuda", torch.bfloat16))
    x = torch.randn(T, H, device="cuda").to(torch.bfloat16)
    compiled = torch.compile(mod, fullgraph=True, backend=backend)
    with torch.inference_mode():
        out, logits = compiled(x)
        out2, _ = compiled(x)
        eager, _ = mod(x)
    moe.check_device_error()
    assert torch.equal(out, out2)
    h = ((x * 0.5 + 0.25).float().cpu().numpy())
    res = O.moe_forward(h, wts.w_gate, wts.w_gate_up, wts.w_down, k, True, "bfloat16",
                        logits=logits.float().cpu().numpy())
    ids, _ = torch.ops.prism_moe.route_topk(logits.contiguous(), k, True)
    assert (ids.cpu().numpy() == res["topk_ids"]).all()
    got = out.float().cpu().numpy()
    d = np.abs(got - res["out"])
    assert d.max() <= BF16_MAX_ABS, d.max()
    assert d.mean() / np.abs(res["out"]).mean() <= BF16_MEAN_REL
    d2 = (out.float() - eager.float()).abs()
    assert d2.max().item() <= BF16_MAX_ABS
