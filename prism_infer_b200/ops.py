"""``torch.ops.prism_moe.*``: the library's kernels as torch custom operators.

Every op calls one entry point of ``libprism_moe.so`` through ``capi`` (which checks device,
dtype and contiguity and turns a non-zero status into ``RuntimeError``; there is no CPU
fallback) and has a fake implementation giving its output shapes, so a module that calls them
can be traced by ``torch.compile(fullgraph=True)`` or ``torch.export`` without running a kernel.
The reference compiles the layers around the block the same way (prism_infer/layers/
layernorm.py:16,28 and activation.py:8 are ``@torch.compile``'d).

Ops (shapes: T tokens, H hidden, E experts, k top-k, W expert-parallel ranks):

* ``route_topk(logits[T,E], top_k, renorm) -> (topk_ids[T,k] int64, topk_weights[T,k])`` —
  prism_infer/layers/moe.py:77-81.
* ``dispatch_plan(topk_ids[T,k], num_experts, ep_size) -> (perm[T*k], input_splits[W],
  sorted_local_eid[T*k]`` (int64, expert_parallel.py:23-42) ``, expert_counts[E],
  expert_offsets[E+1], entry_row[T*k]`` (int32, the expert-major layout)``)``.
* ``permute_rows(x[T,H], top_k, entry_row) -> x_sorted[T*k,H]`` — expert_parallel.py:154-156.
* ``expert_swiglu(x_sorted[R,H], seg_offsets, w_gate_up[El,2I,H], w_down[El,H,I],
  seg_expert) -> y[R,H]`` — moe.py:27-28 with activation.py:8-11 over a segment table.
* ``combine(expert_out, topk_weights[T,k], entry_row) -> out[T,H]`` — expert_parallel.py:45-57.
* ``block_forward(x[T,H], router_logits[T,E], w_gate_up[E,2I,H], w_down[E,H,I], top_k, renorm)
  -> out[T,H]`` — moe.py:77-100 after the router GEMM.
* ``ep_forward(x, router_logits, w_gate_up[El,2I,H], w_down[El,H,I], top_k, renorm, bank)
  -> out[T,H]`` — moe.py:77-85 + expert_parallel.py:140-176 over NVLink peer memory; ``bank``
  names the ``ExpertParallelMoE`` whose landing zones the step uses (``ep_bank_id``).
* ``rmsnorm(x[T,H], weight[H], eps) -> out`` and ``add_rmsnorm(x, residual, weight, eps) ->
  (out, residual_out)`` — prism_infer/layers/layernorm.py:16-40.
* ``block_forward_norm`` / ``ep_forward_norm``: the two block ops with the decoder layer's next
  residual add + RMSNorm fused into the combine; extra arguments ``residual[T,H],
  norm_weight[H], eps``; they return ``(out, residual_out)``.
"""
from __future__ import annotations

import weakref

import torch
from torch import Tensor
from torch.library import custom_op

from prism_infer_b200 import capi

_EP_BANKS: "weakref.WeakValueDictionary[int, object]" = weakref.WeakValueDictionary()


def ep_bank_id(bank) -> int:
    """Register an ``ExpertParallelMoE`` for ``ep_forward`` and return its id."""
    key = id(bank)
    _EP_BANKS[key] = bank
    return key


# ---------------------------------------------------------------------------------- routing

@custom_op("prism_moe::route_topk", mutates_args=())
def route_topk(logits: Tensor, top_k: int, renorm: bool) -> tuple[Tensor, Tensor]:
    ids, w, _ = capi.route_topk(logits, top_k, renorm)
    return ids, w


@route_topk.register_fake
def _(logits, top_k, renorm):
    T = logits.shape[0]
    return (logits.new_empty((T, top_k), dtype=torch.int64),
            logits.new_empty((T, top_k)))


@custom_op("prism_moe::dispatch_plan", mutates_args=())
def dispatch_plan(topk_ids: Tensor, num_experts: int,
                  ep_size: int) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor, Tensor]:
    p = capi.dispatch_plan(topk_ids, num_experts, ep_size, want_perm=True)
    return (p["perm"], p["input_splits"], p["sorted_local_eid"], p["expert_counts"],
            p["expert_offsets"], p["entry_row"])


@dispatch_plan.register_fake
def _(topk_ids, num_experts, ep_size):
    N = topk_ids.numel()
    i64, i32 = torch.int64, torch.int32
    return (topk_ids.new_empty((N,), dtype=i64), topk_ids.new_empty((ep_size,), dtype=i64),
            topk_ids.new_empty((N,), dtype=i64), topk_ids.new_empty((num_experts,), dtype=i32),
            topk_ids.new_empty((num_experts + 1,), dtype=i32),
            topk_ids.new_empty((N,), dtype=i32))


# ---------------------------------------------------------------------------------- data movement

@custom_op("prism_moe::permute_rows", mutates_args=())
def permute_rows(x: Tensor, top_k: int, entry_row: Tensor) -> Tensor:
    return capi.permute_rows(x, top_k, entry_row)


@permute_rows.register_fake
def _(x, top_k, entry_row):
    return x.new_empty((x.shape[0] * top_k, x.shape[1]))


@custom_op("prism_moe::combine", mutates_args=())
def combine(expert_out: Tensor, topk_weights: Tensor, entry_row: Tensor | None) -> Tensor:
    return capi.combine(expert_out, topk_weights, entry_row=entry_row)


@combine.register_fake
def _(expert_out, topk_weights, entry_row):
    return expert_out.new_empty((topk_weights.shape[0], expert_out.shape[-1]))


# ---------------------------------------------------------------------------------- experts

@custom_op("prism_moe::expert_swiglu", mutates_args=())
def expert_swiglu(x_sorted: Tensor, seg_offsets: Tensor, w_gate_up: Tensor, w_down: Tensor,
                  seg_expert: Tensor | None) -> Tensor:
    return capi.expert_swiglu(x_sorted, seg_offsets, w_gate_up, w_down, seg_expert=seg_expert)


@expert_swiglu.register_fake
def _(x_sorted, seg_offsets, w_gate_up, w_down, seg_expert):
    return torch.empty_like(x_sorted)


# ---------------------------------------------------------------------------------- whole block

@custom_op("prism_moe::block_forward", mutates_args=())
def block_forward(x: Tensor, router_logits: Tensor, w_gate_up: Tensor, w_down: Tensor,
                  top_k: int, renorm: bool) -> Tensor:
    return capi.block_forward(x, router_logits, w_gate_up, w_down, top_k, renorm)


@block_forward.register_fake
def _(x, router_logits, w_gate_up, w_down, top_k, renorm):
    return torch.empty_like(x)


@custom_op("prism_moe::ep_forward", mutates_args=())
def ep_forward(x: Tensor, router_logits: Tensor, w_gate_up: Tensor, w_down: Tensor, top_k: int,
               renorm: bool, bank: int) -> Tensor:
    owner = _EP_BANKS.get(bank)
    if owner is None:
        raise RuntimeError("prism_moe::ep_forward: unknown expert-parallel bank id")
    if owner.w_gate_up.data_ptr() != w_gate_up.data_ptr() or \
            owner.w_down.data_ptr() != w_down.data_ptr():
        raise RuntimeError("prism_moe::ep_forward: weights are not the bank's")
    return owner.forward_p2p(x, router_logits=router_logits, top_k=top_k, renorm=renorm)


@ep_forward.register_fake
def _(x, router_logits, w_gate_up, w_down, top_k, renorm, bank):
    return torch.empty_like(x)


# ---------------------------------------------------------------------------------- norms

@custom_op("prism_moe::rmsnorm", mutates_args=())
def rmsnorm(x: Tensor, weight: Tensor, eps: float) -> Tensor:
    return capi.rmsnorm(x, weight, eps)


@rmsnorm.register_fake
def _(x, weight, eps):
    return torch.empty_like(x)


@custom_op("prism_moe::add_rmsnorm", mutates_args=())
def add_rmsnorm(x: Tensor, residual: Tensor, weight: Tensor, eps: float) -> tuple[Tensor, Tensor]:
    return capi.rmsnorm(x, weight, eps, residual=residual)


@add_rmsnorm.register_fake
def _(x, residual, weight, eps):
    return torch.empty_like(x), torch.empty_like(x)


@custom_op("prism_moe::block_forward_norm", mutates_args=())
def block_forward_norm(x: Tensor, router_logits: Tensor, w_gate_up: Tensor, w_down: Tensor,
                       top_k: int, renorm: bool, residual: Tensor, norm_weight: Tensor,
                       eps: float) -> tuple[Tensor, Tensor]:
    residual = residual.contiguous()
    res_out = torch.empty_like(x)
    epi = capi.norm_epilogue(residual, norm_weight, eps, res_out)
    out = capi.block_forward(x, router_logits, w_gate_up, w_down, top_k, renorm, epilogue=epi)
    return out, res_out


@block_forward_norm.register_fake
def _(x, router_logits, w_gate_up, w_down, top_k, renorm, residual, norm_weight, eps):
    return torch.empty_like(x), torch.empty_like(x)


@custom_op("prism_moe::ep_forward_norm", mutates_args=())
def ep_forward_norm(x: Tensor, router_logits: Tensor, w_gate_up: Tensor, w_down: Tensor,
                    top_k: int, renorm: bool, bank: int, residual: Tensor, norm_weight: Tensor,
                    eps: float) -> tuple[Tensor, Tensor]:
    owner = _EP_BANKS.get(bank)
    if owner is None:
        raise RuntimeError("prism_moe::ep_forward_norm: unknown expert-parallel bank id")
    return owner.forward_p2p(x, router_logits=router_logits, top_k=top_k, renorm=renorm,
                             residual=residual, norm_weight=norm_weight, eps=eps)


@ep_forward_norm.register_fake
def _(x, router_logits, w_gate_up, w_down, top_k, renorm, bank, residual, norm_weight, eps):
    return torch.empty_like(x), torch.empty_like(x)
