"""Dense SwiGLU MLP on the grouped expert kernels — the one-expert case of the MoE block.

Drop-in for the reference's ``Qwen3MLP`` (prism_infer/models/qwen3.py:96-122), which the dense
layers of Qwen3 models use: ``gate_up_proj`` is a ``MergedColumnParallelLinear`` of two
``intermediate_size`` halves (gate rows first, prism_infer/layers/linear.py:102-119),
``act_fn`` is ``SiluAndMul`` (prism_infer/layers/activation.py:8-11) and ``down_proj`` a
``RowParallelLinear`` (linear.py:157-182). Here the three run as one segment of the grouped
SwiGLU GEMMs: gate_up and SwiGLU in one tcgen05 launch (bf16; CUDA cores for fp32), down in
the next. Parameter names and ``weight_loader`` signatures match the reference, so its
``load_model`` fills them unchanged. Tensor parallelism is not supported (world size 1 only).
"""
from __future__ import annotations

import torch
from torch import nn

from prism_infer_b200 import ops  # noqa: F401  (registers torch.ops.prism_moe)


class MergedGateUp(nn.Module):
    """``weight`` [sum(output_sizes), input_size]; checkpoint shard i fills rows
    [sum(output_sizes[:i]), +output_sizes[i]) (MergedColumnParallelLinear.weight_loader,
    linear.py:113-119, at tensor-parallel size 1)."""

    def __init__(self, input_size: int, output_sizes: list[int]):
        super().__init__()
        self.output_sizes = list(output_sizes)
        self.weight = nn.Parameter(torch.empty(sum(output_sizes), input_size),
                                   requires_grad=False)
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor,
                      loaded_shard_id: int) -> None:
        off = sum(self.output_sizes[:loaded_shard_id])
        param.data.narrow(0, off, self.output_sizes[loaded_shard_id]).copy_(loaded_weight)


class DownProj(nn.Module):
    """``weight`` [output_size, input_size] (RowParallelLinear.weight_loader, linear.py:168-176,
    at tensor-parallel size 1)."""

    def __init__(self, input_size: int, output_size: int):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(output_size, input_size), requires_grad=False)
        self.weight.weight_loader = self.weight_loader

    def weight_loader(self, param: nn.Parameter, loaded_weight: torch.Tensor) -> None:
        param.data.copy_(loaded_weight)


_segments: dict = {}


def _one_segment(rows: int, device: torch.device) -> torch.Tensor:
    """Device int32 [0, rows], built on the device (no host copy) and cached per shape."""
    key = (device.index, rows)
    seg = _segments.get(key)
    if seg is None:
        seg = torch.arange(2, dtype=torch.int32, device=device) * rows
        _segments[key] = seg
    return seg


class Qwen3MLP(nn.Module):
    """``Qwen3MLP(hidden_size, intermediate_size, hidden_act)``; ``forward(x[..., H])`` returns
    the same shape and dtype. ``hidden_act`` must be ``"silu"``, as the reference asserts."""

    def __init__(self, hidden_size: int, intermediate_size: int, hidden_act: str = "silu"):
        super().__init__()
        assert hidden_act == "silu"
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.gate_up_proj = MergedGateUp(hidden_size, [intermediate_size] * 2)
        self.down_proj = DownProj(intermediate_size, hidden_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        if x2.shape[0] == 0:
            return torch.empty_like(x)
        wgu = self.gate_up_proj.weight
        wd = self.down_proj.weight
        if x2.dtype != wgu.dtype:
            raise RuntimeError(f"input dtype {x2.dtype} != MLP weight dtype {wgu.dtype}")
        y = torch.ops.prism_moe.expert_swiglu(x2, _one_segment(x2.shape[0], x2.device),
                                              wgu.unsqueeze(0), wd.unsqueeze(0), None)
        return y.view(shape)
