"""Stacked expert weights with per-expert, reference-named views.

The reference keeps one ``MoEExpert`` module per expert (prism_infer/layers/moe.py:18-28,
prism_infer/engine/parallel/expert_parallel.py:60-88) with parameters
``gate_up_proj.weight`` [2I, H] (gate rows first) and ``down_proj.weight`` [H, I]. The grouped
GEMM wants all experts of a rank in two contiguous tensors, ``w_gate_up`` [E, 2I, H] and
``w_down`` [E, H, I]. ``ExpertBank`` owns those stacked tensors (non-persistent buffers) and
exposes each expert's slice as a Parameter *view* under the reference's name, so that
``state_dict()`` / ``load_state_dict()`` and the reference's ``load_model`` (which calls
``param.weight_loader(param, w[, shard_id])``, prism_infer/utils/loader.py:63-88) read and write
the stacked storage directly. Views are re-tied after ``.to()`` / ``.cuda()``.
"""
from __future__ import annotations

import weakref

import torch
from torch import nn

from prism_infer_b200 import capi


class _WeightView(nn.Module):
    """Holds one ``weight`` Parameter that is a view into a stacked tensor."""


class ExpertView(nn.Module):
    """One expert: ``gate_up_proj.weight`` [2I, H] and ``down_proj.weight`` [H, I] views.

    ``forward(x)`` runs this single expert through the grouped SwiGLU kernel, the equivalent of
    the reference's ``MoEExpert.forward`` (moe.py:27-28).
    """

    def __init__(self, bank: "ExpertBank", index: int):
        super().__init__()
        self.gate_up_proj = _WeightView()
        self.down_proj = _WeightView()
        object.__setattr__(self, "_bank", weakref.ref(bank))
        object.__setattr__(self, "_index", index)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        bank = self._bank()
        e = self._index
        seg = torch.tensor([0, x.shape[0]], dtype=torch.int32, device=x.device)
        return capi.expert_swiglu(x.contiguous(), seg, bank.w_gate_up[e:e + 1],
                                  bank.w_down[e:e + 1])


class ExpertBank(nn.Module):
    """Mixin owning ``w_gate_up`` / ``w_down`` and a ModuleList of ``ExpertView`` under the
    attribute name ``_expert_list_name``."""

    _expert_list_name = "experts"

    def _init_bank(self, num: int, hidden: int, inter: int) -> None:
        self.register_buffer("w_gate_up", torch.empty(num, 2 * inter, hidden), persistent=False)
        self.register_buffer("w_down", torch.empty(num, hidden, inter), persistent=False)
        setattr(self, self._expert_list_name, nn.ModuleList(ExpertView(self, e) for e in range(num)))
        self._tie()

    def _views(self):
        return getattr(self, self._expert_list_name)

    def _tie(self) -> None:
        me = weakref.ref(self)
        for e, ex in enumerate(self._views()):
            gu = nn.Parameter(self.w_gate_up[e], requires_grad=False)
            dn = nn.Parameter(self.w_down[e], requires_grad=False)

            def gu_loader(param, loaded, shard_id=None, _e=e):
                # packed checkpoint shards: 0 = gate_proj, 1 = up_proj (qwen3.py:214-220)
                dst = me().w_gate_up[_e]
                half = dst.shape[0] // 2
                if shard_id is None:
                    dst.copy_(loaded)
                elif int(shard_id) == 0:
                    dst[:half].copy_(loaded)
                else:
                    dst[half:].copy_(loaded)

            def dn_loader(param, loaded, _e=e):
                me().w_down[_e].copy_(loaded)

            gu.weight_loader = gu_loader
            dn.weight_loader = dn_loader
            ex.gate_up_proj._parameters["weight"] = gu
            ex.down_proj._parameters["weight"] = dn

    def _apply(self, fn, recurse=True):
        for ex in self._views():
            ex.gate_up_proj._parameters.pop("weight", None)
            ex.down_proj._parameters.pop("weight", None)
        super()._apply(fn, recurse)
        self._tie()
        return self
