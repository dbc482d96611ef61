"""Expert parallelism for the MoE block — names and behaviour of
prism_infer/engine/parallel/expert_parallel.py, on B200 kernels.

* ``set_expert_parallel_size`` / ``get_expert_parallel_size`` — process-global EP size
  (expert_parallel.py:7-16).
* ``expert_rank`` — contiguous expert ownership ``e // E_l`` (expert_parallel.py:19-20).
* ``build_dispatch_plan`` — (perm, input_splits, sorted_local_eid), bit-identical to the
  reference's (expert_parallel.py:23-42), computed by the dispatch-plan kernel.
* ``combine_weighted_sum`` — the weighted sum over k (expert_parallel.py:45-57) by the combine
  kernel.
* ``ExpertParallelMoE`` — experts sharded by rank, tokens exchanged with all-to-all
  (expert_parallel.py:91-176).

Transports. ``p2p`` (the default for bf16 on CUDA) runs the whole step in the library's
``prism_moe_ep_forward``: a device-side counts all-gather, then one fused expert launch whose
copy warps fill this rank's receive buffer — pulling the rows other ranks routed here from their
CUDA-IPC-mapped landing zones, one row per (token, rank) — and whose down epilogue writes the
outputs back into the sources' buffers — no host synchronisation. ``nccl``
keeps the reference's structure (all_to_all_single with a host read of the split sizes) around
the library's kernels, with the layout below.

Exchange layout (nccl). The reference sends rows in perm order (grouped by destination rank, flat
order inside) and the receiver regroups them per local expert with boolean masks
(:165-169). Here rows are sent in expert-major order — destination rank, then local expert, then
flat order — which is the same rank grouping refined by expert (experts are owned in contiguous
blocks), so the receiver's buffer is already a list of (source rank, local expert) segments that
the grouped GEMM consumes directly. The per-expert row sequences are the reference's.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from prism_infer_b200 import capi
from prism_infer_b200.layers.experts import ExpertBank

_EXPERT_PARALLEL_SIZE = 1

# Kernel entry points used by ExpertParallelMoE. Tests of the distributed host logic on CPU
# (gloo) substitute an oracle-backed object; the product always uses the CUDA library.
_KERNELS = capi


def set_expert_parallel_size(n: int) -> None:
    global _EXPERT_PARALLEL_SIZE
    _EXPERT_PARALLEL_SIZE = n


def get_expert_parallel_size() -> int:
    return _EXPERT_PARALLEL_SIZE


def expert_rank(expert_id: int, num_local_experts: int) -> int:
    return expert_id // num_local_experts


def build_dispatch_plan(topk_ids: torch.Tensor, num_local_experts: int, ep_size: int):
    """(perm [T*k] int64, input_splits [W] int64, sorted_local_eid [T*k] int64) — the
    reference's plan (expert_parallel.py:23-42), from a deterministic counting sort on the GPU."""
    plan = _KERNELS.dispatch_plan(topk_ids.contiguous(), num_local_experts * ep_size, ep_size,
                                  want_perm=True)
    return plan["perm"], plan["input_splits"], plan["sorted_local_eid"]


def combine_weighted_sum(unpermuted: torch.Tensor, topk_weights: torch.Tensor,
                         num_tokens: int, top_k: int) -> torch.Tensor:
    """out[t] = sum_k w[t,k] * unpermuted[t*k + k] (expert_parallel.py:45-57)."""
    assert unpermuted.shape[0] == num_tokens * top_k
    w = topk_weights.to(unpermuted.dtype).reshape(num_tokens, top_k).contiguous()
    return _KERNELS.combine(unpermuted.contiguous(), w)


class ExpertParallelMoE(ExpertBank):
    """MoE layer with expert parallelism: experts sharded by rank, tokens routed via
    all-to-all (dispatch -> local experts -> combine); expert_parallel.py:91-111."""

    _expert_list_name = "local_experts"

    def __init__(self, hidden_size: int, intermediate_size: int, num_experts: int,
                 ep_size: int, ep_rank: int, group=None, transport: str | None = None):
        super().__init__()
        assert num_experts % ep_size == 0, "num_experts must be divisible by ep_size"
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.num_experts = num_experts
        self.ep_size = ep_size
        self.ep_rank = ep_rank
        self.num_local_experts = num_experts // ep_size
        self.local_expert_base = ep_rank * self.num_local_experts
        self.group = group
        # "p2p": rows written straight into the owners' memory over NVLink (CUDA IPC mappings,
        # device-side counts exchange, no host synchronisation); "nccl": all_to_all_single with
        # a host read of the split sizes, like the reference. None picks p2p for bf16 on CUDA.
        self.transport = transport
        self._p2p = None
        self._init_bank(self.num_local_experts, hidden_size, intermediate_size)
        from prism_infer_b200 import ops
        self.op_id = ops.ep_bank_id(self)   # names this bank to torch.ops.prism_moe.ep_forward

    # ------------------------------------------------------------------ NVLink peer transport

    def use_p2p(self, x: torch.Tensor) -> bool:
        if self.transport == "nccl" or _KERNELS is not capi:
            return False
        if self.transport == "p2p":
            return True
        return x.is_cuda and x.dtype == torch.bfloat16 and (
            self.ep_size == 1 or dist.get_backend(self.group) == "nccl")

    def reserve(self, max_tokens: int, top_k: int) -> None:
        """Collective: allocate this rank's landing zone for up to ``max_tokens`` tokens per rank
        (the maximum over ranks is used) and map every peer's. Called by the first forward."""
        W, me = self.ep_size, self.ep_rank
        dev = self.w_gate_up.device
        cap = torch.tensor([max_tokens], dtype=torch.int64, device=dev)
        if W > 1:
            dist.all_reduce(cap, op=dist.ReduceOp.MAX, group=self.group)
        max_tokens = max(256, -(-int(cap.item()) // 256) * 256)
        lib = capi.load()
        H, I, E = self.hidden_size, self.intermediate_size, self.num_experts
        nbytes = lib.prism_moe_ep_landing_bytes(W, max_tokens, top_k, H, E, capi.BF16)
        ws_bytes = lib.prism_moe_ep_workspace_size(max_tokens, H, I, E, top_k, W, capi.BF16)
        if nbytes == 0 or ws_bytes == 0:
            raise RuntimeError("expert-parallel landing zone: invalid shape")
        self.release()
        ptr, handle = capi.ep_alloc_landing(nbytes)
        handles = [None] * W
        if W > 1:
            dist.all_gather_object(handles, handle, group=self.group)
        else:
            handles[0] = handle
        peers = [ptr if d == me else capi.ep_open_peer(handles[d]) for d in range(W)]
        self._p2p = dict(max_tokens=max_tokens, top_k=top_k, ptr=ptr, peers=peers,
                         table=torch.tensor(peers, dtype=torch.int64, device=dev),
                         ws=torch.zeros(ws_bytes, dtype=torch.uint8, device=dev))
        if W > 1:
            dist.barrier(group=self.group)

    def release(self) -> None:
        """Unmap peers and free the landing zone (collective when W > 1)."""
        st = self._p2p
        if st is None:
            return
        torch.cuda.synchronize()
        if self.ep_size > 1 and dist.is_initialized():
            dist.barrier(group=self.group)
        lib = capi.load()
        for d, p in enumerate(st["peers"]):
            if d != self.ep_rank:
                lib.prism_moe_ep_close_peer(p)
        lib.prism_moe_ep_free_landing(st["ptr"])
        self._p2p = None

    def forward_p2p(self, x: torch.Tensor, router_logits=None, topk_ids=None, topk_weights=None,
                    top_k: int | None = None, renorm: bool = True, residual=None,
                    norm_weight=None, eps: float = 1e-6):
        """One step over NVLink peer memory: route (from logits, or given ids/weights), rows
        pulled by their experts' owners (one per token and owner), grouped experts, outputs
        stored back into the sources' landing zones by the down GEMM, combine. Collective over
        the EP group.

        The step's epoch is counted on the device (epoch argument 0), so after the first call
        (which reserves the landing zones, a collective that allocates) a step can be captured in
        a CUDA graph and replayed; every rank must replay it the same number of times.

        With ``residual`` and ``norm_weight`` the final combine also applies the decoder layer's
        next residual add + RMSNorm and the call returns (normalised, residual_out)."""
        T = x.shape[0]
        k = top_k if top_k is not None else topk_ids.shape[1]
        if self._p2p is None or self._p2p["top_k"] != k:
            self.reserve(T, k)
        st = self._p2p
        if T > st["max_tokens"]:
            raise RuntimeError(f"{T} tokens exceed the expert-parallel landing capacity "
                               f"{st['max_tokens']}; call reserve() with a larger max_tokens")
        x = x.contiguous()
        out = torch.empty_like(x)
        ids = None if topk_ids is None else topk_ids.contiguous()
        w = None if topk_weights is None else topk_weights.to(x.dtype).contiguous()
        lg = None if router_logits is None else router_logits.contiguous()
        res_out = torch.empty_like(x) if norm_weight is not None else None
        epi = capi.norm_epilogue(None if residual is None else residual.contiguous(),
                                 norm_weight, eps, res_out)
        lib = capi.load()
        capi.check(lib.prism_moe_ep_forward_norm(
            x.data_ptr(), capi.ptr(lg), capi.ptr(ids), capi.ptr(w), capi.BF16, T,
            st["max_tokens"], self.hidden_size, self.intermediate_size, self.num_experts, k,
            int(bool(renorm)), self.ep_size, self.ep_rank, self.w_gate_up.data_ptr(),
            self.w_down.data_ptr(), st["ptr"], st["table"].data_ptr(), 0,
            out.data_ptr(), st["ws"].data_ptr(), st["ws"].numel(), capi.stream_of(x.device),
            None if epi is None else ctypes.byref(epi)), "prism_moe_ep_forward")
        return out if epi is None else (out, res_out)

    def step_stats(self) -> dict:
        """Timing and row counts of the last step (``capi.ep_read_stats``; synchronises)."""
        if self._p2p is None:
            raise RuntimeError("no expert-parallel step has run")
        return capi.ep_read_stats(self._p2p["ws"])

    def landing_bytes(self) -> int:
        """Bytes of this rank's landing zone (0 before the first step)."""
        if self._p2p is None:
            return 0
        st = self._p2p
        return int(capi.load().prism_moe_ep_landing_bytes(
            self.ep_size, st["max_tokens"], st["top_k"], self.hidden_size, self.num_experts,
            capi.BF16))

    def check_device_error(self) -> None:
        """Synchronise and raise if a kernel of the last step recorded an error (a peer wait
        that ran out shows up here as PRISM_MOE_ERR_TIMEOUT)."""
        if self._p2p is not None:
            ws = self._p2p["ws"]
            capi.check(capi.read_device_error(ws[:4].view(torch.int32)), "expert-parallel step")

    def exchange_plan(self, expert_counts: torch.Tensor):
        """Counts exchange (expert_parallel.py:113-127), per local expert instead of per rank:
        recv_counts[s, le] = rows source rank s sends for local expert le. Returns
        (recv_counts [W, E_l] int32 device, in_splits list, out_splits list)."""
        W, El = self.ep_size, self.num_local_experts
        send = expert_counts.to(torch.int32).contiguous()
        if W == 1:
            recv = send.clone()
        else:
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=self.group)
        recv = recv.view(W, El)
        splits = torch.cat([send.view(W, El).sum(1), recv.sum(1)]).tolist()   # one host sync
        return recv, splits[:W], splits[W:]

    def _all_to_all(self, x: torch.Tensor, out_splits, in_splits) -> torch.Tensor:
        if self.ep_size == 1:
            return x.clone()
        out = x.new_empty((sum(out_splits),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), out_splits, in_splits, group=self.group)
        return out

    def forward(self, x: torch.Tensor, topk_ids: torch.Tensor,
                topk_weights: torch.Tensor) -> torch.Tensor:
        """x [T, H], topk_ids [T, k] global expert ids, topk_weights [T, k] -> [T, H]
        (expert_parallel.py:140-176)."""
        if self.use_p2p(x):
            return self.forward_p2p(x, topk_ids=topk_ids, topk_weights=topk_weights)
        K = _KERNELS
        T, k = topk_ids.shape
        W, El = self.ep_size, self.num_local_experts
        plan = K.dispatch_plan(topk_ids.contiguous(), self.num_experts, W, want_perm=False)
        entry_row = plan["entry_row"]
        send_x = K.permute_rows(x.contiguous(), k, entry_row)
        recv_counts, in_splits, out_splits = self.exchange_plan(plan["expert_counts"])
        recv_x = self._all_to_all(send_x, out_splits, in_splits)
        seg_offsets = torch.zeros(W * El + 1, dtype=torch.int32, device=x.device)
        seg_offsets[1:] = torch.cumsum(recv_counts.reshape(-1), 0)
        seg_expert = (torch.arange(W * El, dtype=torch.int32, device=x.device) % El).contiguous()
        recv_y = K.expert_swiglu(recv_x, seg_offsets, self.w_gate_up, self.w_down,
                                 seg_expert=seg_expert)
        back = self._all_to_all(recv_y, in_splits, out_splits)
        w = topk_weights.to(x.dtype).contiguous()
        return K.combine(back, w, entry_row=entry_row)
