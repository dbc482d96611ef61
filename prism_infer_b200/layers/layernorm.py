"""Drop-in for prism_infer/layers/layernorm.py: ``RMSNorm`` on the library's norm kernel.

Same constructor (``RMSNorm(hidden_size, eps=1e-6)``, weight initialised to ones) and the same
``forward(x, residual=None)``: without a residual it returns the normalised ``x``
(rms_forward, layernorm.py:16-26); with one it returns ``(normalised x + residual,
x + residual)`` (add_rms_forward, :28-40). Arithmetic: fp32 sum and sum of squares, the
reference's two roundings to the input dtype (see include/prism_moe.h, prism_moe_rmsnorm).

In a Qwen3 decoder layer the ``post_attention_layernorm`` in front of the MoE block is this
module (prism_infer/models/qwen3.py:184), and the next layer's ``input_layernorm(hidden,
residual)`` on the block's output can run inside the block's combine instead:
``MoE.forward(hidden, residual=residual, norm=next_layer.input_layernorm)``.
"""
from __future__ import annotations

import torch
from torch import nn

from prism_infer_b200 import ops  # noqa: F401  (registers torch.ops.prism_moe)


class RMSNorm(nn.Module):

    def __init__(self, hidden_size: int, eps: float = 1e-6) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(hidden_size))

    def rms_forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        out = torch.ops.prism_moe.rmsnorm(x.reshape(-1, shape[-1]).contiguous(), self.weight,
                                          float(self.eps))
        return out.view(shape)

    def add_rms_forward(self, x: torch.Tensor,
                        residual: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        shape = x.shape
        out, res = torch.ops.prism_moe.add_rmsnorm(
            x.reshape(-1, shape[-1]).contiguous(),
            residual.reshape(-1, shape[-1]).contiguous(), self.weight, float(self.eps))
        return out.view(shape), res.view(shape)

    def forward(self, x: torch.Tensor, residual: torch.Tensor | None = None):
        if residual is None:
            return self.rms_forward(x)
        return self.add_rms_forward(x, residual)
