"""Drop-in for prism_infer/layers/moe.py: the Qwen3-MoE sparse block on B200 kernels.

Same constructor (``MoE(hidden_size, intermediate_size, num_experts, top_k,
norm_topk_prob=True)``, moe.py:40-67), same parameter names (``gate.weight``,
``experts.{e}.gate_up_proj.weight``, ``experts.{e}.down_proj.weight``; under expert parallelism
``ep_moe.local_experts.{le}.*``) and same ``forward(hidden_states) -> Tensor`` of the input's
shape and dtype (moe.py:69-100). The expert-parallel size is read from the process-global
``set_expert_parallel_size`` before construction, as in the reference (moe.py:57-61).

Forward, single GPU (EP=1):
  1. ``router_logits = F.linear(x, gate.weight)`` — the reference's own call (moe.py:74), so the
     logits are bit-identical to the reference's on the same device;
  2. ``torch.ops.prism_moe.block_forward`` (``prism_moe_block_forward`` in the C ABI): route
     (softmax/top-k/renorm, bit-exact with torch on CUDA), dispatch plan, row permutation,
     grouped SwiGLU experts on tcgen05, weighted combine. Under expert parallelism,
     ``torch.ops.prism_moe.ep_forward`` runs the step over NVLink peer memory.
No host synchronisation happens inside ``forward``; it can be captured in a CUDA graph (under
expert parallelism after the first call, which reserves the landing zones), and it traces
through ``torch.compile(fullgraph=True)`` (the ops have fake implementations).
Only bfloat16 and float32 on an sm_100 device are supported; anything else raises.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from prism_infer_b200 import capi, ops  # noqa: F401  (ops registers torch.ops.prism_moe)
from prism_infer_b200.engine.parallel.expert_parallel import (
    ExpertParallelMoE,
    get_expert_parallel_size,
)
from prism_infer_b200.layers.experts import ExpertBank


class ReplicatedGate(nn.Module):
    """Router weight [E, H] replicated on every rank (reference ReplicatedLinear,
    prism_infer/layers/linear.py:63-77)."""

    def __init__(self, hidden_size: int, num_experts: int):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(num_experts, hidden_size), requires_grad=False)
        self.weight.weight_loader = lambda param, loaded: param.data.copy_(loaded)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x, self.weight)


class MoE(ExpertBank):
    """Token-choice MoE, Qwen/Mixtral routing: softmax -> top-k -> re-norm (moe.py:31-38)."""

    _expert_list_name = "experts"

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int, top_k: int,
                 norm_topk_prob: bool = True) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_experts = num_experts
        self.top_k = top_k
        self.norm_topk_prob = norm_topk_prob
        self.gate = ReplicatedGate(hidden_size, num_experts)
        self.ep_size = get_expert_parallel_size()
        if self.ep_size > 1:
            import torch.distributed as dist
            ep_rank = dist.get_rank() if dist.is_initialized() else 0
            self.ep_moe = ExpertParallelMoE(hidden_size, intermediate_size, num_experts,
                                            self.ep_size, ep_rank)
            self.experts = None
        else:
            self.ep_moe = None
            self._init_bank(num_experts, hidden_size, intermediate_size)

    # ExpertBank hooks are inert when the experts live in ep_moe
    def _views(self):
        return self.experts if self.experts is not None else []

    def _apply(self, fn, recurse=True):
        if self.experts is None:
            return nn.Module._apply(self, fn, recurse)
        return super()._apply(fn, recurse)

    def route(self, hidden_states: torch.Tensor):
        """(router_logits, topk_ids, topk_weights) exactly as moe.py:74-81 computes them."""
        x = hidden_states.reshape(-1, hidden_states.shape[-1])
        logits = self.gate(x)
        ids, w, _ = capi.route_topk(logits.contiguous(), self.top_k, self.norm_topk_prob)
        return logits, ids, w

    def forward(self, hidden_states: torch.Tensor, residual: torch.Tensor | None = None,
                norm: nn.Module | None = None):
        """``forward(hidden_states)`` -> the block output, as moe.py:69-100.

        Decoder-layer fusion (optional): with ``residual`` (the layer's residual stream, shaped
        like ``hidden_states``) and ``norm`` (the next layer's ``RMSNorm``: its ``weight`` and
        ``eps`` are used), the combine kernel also applies ``norm(output, residual)`` and the call
        returns ``(normalised, output + residual)`` — what prism_infer/models/qwen3.py:179-186
        computes with the next layer's input_layernorm — without writing the block output.
        """
        orig_shape = hidden_states.shape
        x = hidden_states.reshape(-1, orig_shape[-1])
        if not x.is_contiguous():
            x = x.contiguous()
        if x.dtype != self.gate.weight.dtype:
            raise RuntimeError(f"hidden_states dtype {x.dtype} != MoE weight dtype "
                               f"{self.gate.weight.dtype}")
        fuse = norm is not None
        if fuse and residual is None:
            raise RuntimeError("MoE.forward: norm= needs residual=")
        logits = self.gate(x)                     # moe.py:74 — cuBLAS, as in the reference
        renorm = bool(self.norm_topk_prob)
        if self.ep_size > 1:
            bank = self.ep_moe
            if bank.use_p2p(x):
                if fuse:
                    out, res = torch.ops.prism_moe.ep_forward_norm(
                        x, logits, bank.w_gate_up, bank.w_down, self.top_k, renorm, bank.op_id,
                        residual.reshape(x.shape), norm.weight, float(norm.eps))
                    return out.view(orig_shape), res.view(orig_shape)
                out = torch.ops.prism_moe.ep_forward(x, logits, bank.w_gate_up, bank.w_down,
                                                     self.top_k, renorm, bank.op_id)
                return out.view(orig_shape)
            ids, w = torch.ops.prism_moe.route_topk(logits, self.top_k, renorm)
            out = bank(x, ids, w)
            if fuse:
                out, res = norm(out, residual.reshape(x.shape))
                return out.view(orig_shape), res.view(orig_shape)
            return out.view(orig_shape)
        if fuse:
            out, res = torch.ops.prism_moe.block_forward_norm(
                x, logits, self.w_gate_up, self.w_down, self.top_k, renorm,
                residual.reshape(x.shape), norm.weight, float(norm.eps))
            return out.view(orig_shape), res.view(orig_shape)
        out = torch.ops.prism_moe.block_forward(x, logits, self.w_gate_up, self.w_down,
                                                self.top_k, renorm)
        return out.view(orig_shape)

    def check_device_error(self, device=None) -> None:
        """Synchronise and raise if a kernel of the last forward recorded an error."""
        if self.ep_moe is not None:
            self.ep_moe.check_device_error()
            return
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
        word = capi.block_error_word(dev)
        if word is not None:
            capi.check(capi.read_device_error(word, dev), "MoE kernels")
