"""CPU oracle for the Qwen3-MoE sparse block — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of the reference's MoE hot path:

* ``MoE.forward``                 prism_infer/layers/moe.py:69-100
* ``MoEExpert.forward``           prism_infer/layers/moe.py:27-28
* ``SiluAndMul.forward``          prism_infer/layers/activation.py:8-11
* ``build_dispatch_plan``         prism_infer/engine/parallel/expert_parallel.py:23-42
* ``combine_weighted_sum``        prism_infer/engine/parallel/expert_parallel.py:45-57
* ``ExpertParallelMoE.forward``   prism_infer/engine/parallel/expert_parallel.py:140-176
* ``RMSNorm.rms_forward`` / ``add_rms_forward``   prism_infer/layers/layernorm.py:16-40 (the
  decoder layer's norms at the block's edges, prism_infer/models/qwen3.py:179-186)

It is the checker, never the thing measured or shipped: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it. The product
path (``prism_infer_b200``) never calls into this file.

Parity pins (what ties this restatement to the reference):

* golden fixtures in ``tests/golden/`` produced by running the reference's own modules on
  CPU (``tests/golden/make_golden.py``), including W=2 and W=4 gloo EP runs;
* the reference's known-answer tests ``tests/test_expert_parallel.py:15-22`` (dispatch plan)
  and ``:34-43`` (weighted combine);
* on a CUDA host, the torch CUDA ops the reference calls on GPU (``F.softmax`` / ``torch.topk``
  / ``sum`` / cast) for the tie order of ``torch.topk`` (``tests/test_kernels_gpu.py``).

Numerics modelled:

* ``dtype="bfloat16"``: values are carried as float32 arrays holding bf16-representable
  numbers; every point where the reference materialises a bf16 tensor is rounded with
  round-to-nearest-even (``bf16_round``). GEMMs accumulate in float32 (the reference's cuBLAS
  / CPU BLAS also accumulate in fp32; the order differs, hence a tolerance on outputs).
* ``torch.topk`` on CUDA (the reference's production device) selects every value strictly
  greater than the k-th value, then values equal to it in ascending index order, and sorts the
  k gathered pairs with a 32-wide bitonic network (invalid slots sort last). ``topk_torch_cuda``
  emulates exactly that, so tied router probabilities resolve as they do on the GPU.
* the renormalisation sum over k follows torch's CUDA reduction tree (decreasing offsets).
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "bf16_round", "router_logits", "softmax_fp32", "topk_torch_cuda", "renorm_weights", "route",
    "expert_mlp", "moe_forward", "build_dispatch_plan", "combine_weighted_sum",
    "ep_forward_all_ranks", "expert_major_order", "expert_counts", "rms_norm",
]


# ----------------------------------------------------------------------------------------
# bf16 helpers
# ----------------------------------------------------------------------------------------

def bf16_round(a) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even), returned as float32.

    Mirrors every ``.to(torch.bfloat16)`` / bf16-output op of the reference. NaN stays NaN.
    """
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    out = rounded.astype(np.uint32).view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.float32("nan")
    return out


def _cast(a: np.ndarray, dtype: str) -> np.ndarray:
    a = np.asarray(a, dtype=np.float32)
    return bf16_round(a) if dtype == "bfloat16" else a


# ----------------------------------------------------------------------------------------
# Router: logits -> softmax -> top-k -> renorm -> cast        (moe.py:74-81)
# ----------------------------------------------------------------------------------------

def router_logits(x: np.ndarray, w_gate: np.ndarray, dtype: str) -> np.ndarray:
    """``self.gate(hidden_states)`` = ``F.linear(x, W_g)`` (moe.py:74, linear.py:76-77).

    float32 accumulation; output materialised in the input dtype.
    """
    return _cast(np.asarray(x, np.float32) @ np.asarray(w_gate, np.float32).T, dtype)


def softmax_fp32(logits: np.ndarray) -> np.ndarray:
    """``F.softmax(router_logits, dim=-1, dtype=torch.float)`` (moe.py:77).

    The sum of exponentials follows the order of torch's warp softmax on CUDA (a per-lane
    serial sum over elements ``lane + 32*it`` followed by an xor-butterfly over the lanes),
    so the result differs from the GPU only by the last-ulp behaviour of ``exp``.
    """
    x = np.asarray(logits, np.float32)
    T, E = x.shape
    if T == 0:
        return np.zeros((0, E), np.float32)
    p2 = 1
    while p2 < E:
        p2 *= 2
    width = min(p2, 32)
    iters = p2 // width
    pad = np.full((T, p2), -np.inf, np.float32)
    pad[:, :E] = x
    lanes = pad.reshape(T, iters, width)                       # [T, it, lane]
    m = lanes.max(axis=(1, 2)).astype(np.float32)
    ex = np.exp((lanes - m[:, None, None]).astype(np.float32)).astype(np.float32)
    acc = np.zeros((T, width), np.float32)
    for it in range(iters):
        acc = (acc + ex[:, it, :]).astype(np.float32)
    off = width // 2
    lane = np.arange(width)
    while off > 0:
        acc = (acc + acc[:, lane ^ off]).astype(np.float32)
        off //= 2
    s = acc[:, 0]
    probs = (ex.reshape(T, p2)[:, :E] / s[:, None]).astype(np.float32)
    return probs


def _bitonic32_desc(keys: np.ndarray, vals: np.ndarray, valid: np.ndarray):
    """Sort rows of 32 (key, value, valid) triples descending with the compare-exchange network
    torch uses for top-k outputs of size <= 32 (ATen/native/cuda/SortUtils.cuh bitonicSort,
    16 threads x 2 items). Invalid entries sink to the end. Vectorised over rows."""
    keys, vals, valid = keys.copy(), vals.copy(), valid.copy()
    n = 32
    t = np.arange(n // 2)

    def stage(size_flag_bits: int | None, stride: int):
        pos = 2 * t - (t & (stride - 1))
        a, b = pos, pos + stride
        if size_flag_bits is None:
            flag = np.zeros_like(t, dtype=bool)
        else:
            flag = (t & size_flag_bits) != 0
        ka, kb = keys[:, a], keys[:, b]
        va_ok, vb_ok = valid[:, a], valid[:, b]
        gt = (ka > kb) | (np.isnan(ka) & ~np.isnan(kb))
        swap = (gt & va_ok) | ~vb_ok
        do = swap == flag[None, :]
        for arr in (keys, vals, valid):
            xa, xb = arr[:, a].copy(), arr[:, b].copy()
            arr[:, a] = np.where(do, xb, xa)
            arr[:, b] = np.where(do, xa, xb)

    size = 2
    while size < n:
        stride = size // 2
        while stride > 0:
            stage(size // 2, stride)
            stride //= 2
        size *= 2
    stride = n // 2
    while stride > 0:
        stage(None, stride)
        stride //= 2
    return keys, vals, valid


def topk_torch_cuda(probs: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """``torch.topk(routing_weights, k, dim=-1)`` as executed on CUDA (moe.py:78).

    Selection: all values strictly greater than the k-th largest, then values equal to it in
    ascending expert index. Order: the gathered k pairs (greater ones in index order, then the
    equal ones) pass through the 32-wide bitonic network of ``_bitonic32_desc``.
    Returns (values float32 [T,k], indices int64 [T,k]).
    """
    p = np.asarray(probs, np.float32)
    T, E = p.shape
    assert 1 <= k <= min(E, 32)
    if T == 0:
        return np.zeros((0, k), np.float32), np.zeros((0, k), np.int64)
    kth = -np.sort(-p, axis=1)[:, k - 1]
    cls = np.where(p > kth[:, None], 0, np.where(p == kth[:, None], 1, 2))
    order = np.argsort(cls, axis=1, kind="stable")[:, :k]     # gather order
    keys = np.zeros((T, 32), np.float32)
    vals = np.zeros((T, 32), np.int64)
    valid = np.zeros((T, 32), bool)
    keys[:, :k] = np.take_along_axis(p, order, axis=1)
    vals[:, :k] = order
    valid[:, :k] = True
    keys, vals, valid = _bitonic32_desc(keys, vals, valid)
    return keys[:, :k].copy(), vals[:, :k].copy()


def renorm_weights(w: np.ndarray) -> np.ndarray:
    """``routing_weights / routing_weights.sum(dim=-1, keepdim=True)`` (moe.py:79-80).

    The sum over k follows torch's CUDA reduction of a short contiguous row
    (ATen/native/cuda/Reduce.cuh, torch 2.11): lane ``j`` of a ``last_pow2(k)``-wide group sums
    elements ``j, j+width, ...`` serially, then lanes combine by shuffle-down with decreasing
    offsets ``width/2, ..., 2, 1``; for k=8 that is ``((w0+w4)+(w2+w6)) + ((w1+w5)+(w3+w7))``.
    """
    w = np.asarray(w, np.float32)
    T, k = w.shape
    width = 1
    while width * 2 <= min(k, 32):
        width *= 2
    lanes = np.zeros((T, width), np.float32)
    for j in range(k):
        lanes[:, j % width] = (lanes[:, j % width] + w[:, j]).astype(np.float32)
    off = width // 2
    while off > 0:
        nxt = lanes.copy()
        for l in range(width):
            if l + off < width:
                nxt[:, l] = (lanes[:, l] + lanes[:, l + off]).astype(np.float32)
        lanes = nxt
        off //= 2
    s = lanes[:, 0]
    return (w / s[:, None]).astype(np.float32)


def route(logits: np.ndarray, k: int, renorm: bool, dtype: str):
    """Routing of moe.py:77-81: softmax(fp32) -> top-k -> optional renorm -> cast to dtype.

    Returns (topk_ids int64 [T,k], topk_weights float32 [T,k] holding ``dtype`` values).
    """
    probs = softmax_fp32(logits)
    w, ids = topk_torch_cuda(probs, k)
    if renorm:
        w = renorm_weights(w)
    return ids, _cast(w, dtype)


def expert_counts(topk_ids: np.ndarray, E: int) -> np.ndarray:
    """Rows routed to each expert: ``token_idx.numel()`` per expert in moe.py:93-94."""
    return np.bincount(np.asarray(topk_ids).reshape(-1), minlength=E).astype(np.int64)


def expert_major_order(topk_ids: np.ndarray, E: int) -> np.ndarray:
    """Routed entries (flat index ``t*k + j``) grouped by expert, flat order kept inside each
    expert: the row layout in which this build runs the expert GEMMs. It groups the same rows
    per expert as moe.py:92-96 (which lists them slot-major) and, because experts are owned in
    contiguous blocks (expert_parallel.py:19-20), also groups them by destination rank as
    expert_parallel.py:37-39 does."""
    return np.argsort(np.asarray(topk_ids).reshape(-1), kind="stable").astype(np.int64)


# ----------------------------------------------------------------------------------------
# Experts (moe.py:18-28, activation.py:6-11)
# ----------------------------------------------------------------------------------------

def _silu(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, np.float32)
    with np.errstate(over="ignore"):
        return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def expert_mlp(x: np.ndarray, w_gate_up: np.ndarray, w_down: np.ndarray, dtype: str) -> np.ndarray:
    """``down_proj(SiluAndMul(gate_up_proj(x)))`` for one expert (moe.py:27-28).

    gate_up output [n, 2I] is materialised in dtype; SiluAndMul (compiled; one rounding) computes
    ``silu(g) * u`` in fp32 and materialises in dtype; down_proj output is materialised in dtype.
    """
    I = w_down.shape[1]
    gu = _cast(np.asarray(x, np.float32) @ np.asarray(w_gate_up, np.float32).T, dtype)
    a = _cast(_silu(gu[:, :I]) * gu[:, I:], dtype)
    return _cast(a @ np.asarray(w_down, np.float32).T, dtype)


def moe_forward(x: np.ndarray, w_gate: np.ndarray, w_gate_up: np.ndarray, w_down: np.ndarray,
                k: int, renorm: bool, dtype: str, logits: np.ndarray | None = None):
    """Single-GPU ``MoE.forward`` (moe.py:69-100).

    ``x`` [..., H]; returns a dict with logits, topk_ids, topk_weights, counts, out [..., H].
    ``logits`` may be given to route on exactly the logits a GPU run produced.
    """
    x = _cast(x, dtype)
    shape = x.shape
    x2 = x.reshape(-1, shape[-1])
    T, H = x2.shape
    E = w_gate.shape[0]
    if logits is None:
        logits = router_logits(x2, _cast(w_gate, dtype), dtype)
    ids, w = route(logits, k, renorm, dtype)
    final = np.zeros((T, H), np.float32)
    counts = np.zeros(E, np.int64)
    for e in range(E):
        # torch.where(one_hot(ids).permute(2,1,0)[e]) -> (slot, token), slot-major (moe.py:91-93)
        slot_idx, token_idx = np.nonzero((ids == e).T)
        counts[e] = token_idx.size
        if token_idx.size == 0:
            continue
        y = expert_mlp(x2[token_idx], _cast(w_gate_up[e], dtype), _cast(w_down[e], dtype), dtype)
        contrib = _cast(y * w[token_idx, slot_idx][:, None], dtype)
        # index_add_ in x's dtype (moe.py:98): each token occurs once per expert
        final[token_idx] = _cast(final[token_idx] + contrib, dtype)
    return dict(logits=logits, topk_ids=ids, topk_weights=w, counts=counts,
                out=final.reshape(shape))


# ----------------------------------------------------------------------------------------
# Expert parallelism (expert_parallel.py)
# ----------------------------------------------------------------------------------------

def build_dispatch_plan(topk_ids: np.ndarray, num_local_experts: int, ep_size: int):
    """expert_parallel.py:23-42: dst = id // E_l; perm = stable argsort(dst);
    splits = bincount(dst, W); sorted_local_eid = (id % E_l)[perm]. All int64."""
    flat = np.asarray(topk_ids, np.int64).reshape(-1)
    dst = flat // num_local_experts
    perm = np.argsort(dst, kind="stable").astype(np.int64)
    splits = np.bincount(dst, minlength=ep_size).astype(np.int64)
    sorted_local_eid = (flat % num_local_experts)[perm].astype(np.int64)
    return perm, splits, sorted_local_eid


def combine_weighted_sum(unpermuted: np.ndarray, topk_weights: np.ndarray, num_tokens: int,
                         top_k: int, dtype: str) -> np.ndarray:
    """expert_parallel.py:45-57: ``(unperm.view(T,k,H) * w.to(dtype)[...,None]).sum(1)``.

    The product is materialised in dtype; the sum accumulates in fp32 and is cast once.
    """
    H = unpermuted.shape[-1]
    g = np.asarray(unpermuted, np.float32).reshape(num_tokens, top_k, H)
    wt = _cast(topk_weights, dtype).reshape(num_tokens, top_k, 1)
    prod = _cast(g * wt, dtype)
    acc = np.zeros((num_tokens, H), np.float32)
    for j in range(top_k):
        acc = (acc + prod[:, j, :]).astype(np.float32)
    return _cast(acc, dtype)


def ep_forward_all_ranks(xs: list, w_gate: np.ndarray, w_gate_up: np.ndarray,
                         w_down: np.ndarray, k: int, renorm: bool, dtype: str,
                         logits: list | None = None):
    """``MoE.forward`` with ``ExpertParallelMoE`` on W ranks (moe.py:83-85,
    expert_parallel.py:140-176), all ranks emulated in one process.

    ``xs[r]`` is rank r's [T_r, H] tokens; ``w_gate_up``/``w_down`` hold all E experts (rank r owns
    experts ``[r*E_l, (r+1)*E_l)``, expert_parallel.py:19-20). Returns per-rank dicts with the
    routing, the dispatch plan, the received local expert ids, the output splits and ``out``.
    """
    W = len(xs)
    E = w_gate.shape[0]
    assert E % W == 0, "num_experts must be divisible by ep_size"
    El = E // W
    ranks = []
    for r in range(W):
        x = _cast(xs[r], dtype).reshape(-1, xs[r].shape[-1])
        lg = router_logits(x, _cast(w_gate, dtype), dtype) if logits is None else logits[r]
        ids, w = route(lg, k, renorm, dtype)
        perm, splits, sleid = build_dispatch_plan(ids, El, W)
        flat_x = np.repeat(x, k, axis=0)                      # repeat_interleave (:154)
        ranks.append(dict(x=x, logits=lg, topk_ids=ids, topk_weights=w, perm=perm,
                          input_splits=splits, sorted_local_eid=sleid, sorted_x=flat_x[perm]))
    # counts exchange (:113-127): recv[i] = rank_i.input_splits[this_rank]
    for r in range(W):
        ranks[r]["output_splits"] = np.array([ranks[s]["input_splits"][r] for s in range(W)],
                                             np.int64)

    def _segment(s, r):
        off = int(ranks[s]["input_splits"][:r].sum())
        n = int(ranks[s]["input_splits"][r])
        return off, n

    # dispatch a2a (:161-162): rank r receives, in source-rank order, the rows sent to it
    for r in range(W):
        rx, re = [], []
        for s in range(W):
            off, n = _segment(s, r)
            rx.append(ranks[s]["sorted_x"][off:off + n])
            re.append(ranks[s]["sorted_local_eid"][off:off + n])
        H = xs[0].shape[-1]
        recv_x = np.concatenate(rx) if rx else np.zeros((0, H), np.float32)
        recv_eid = np.concatenate(re) if re else np.zeros(0, np.int64)
        out = np.zeros_like(recv_x)
        for le in range(El):                                  # (:165-169)
            sel = recv_eid == le
            if sel.any():
                e = r * El + le
                out[sel] = expert_mlp(recv_x[sel], _cast(w_gate_up[e], dtype),
                                      _cast(w_down[e], dtype), dtype)
        ranks[r]["recv_eid"] = recv_eid
        ranks[r]["expert_out"] = out
    # combine a2a (:172): reverse splits, then unperm[perm] = recv_out and weighted sum
    for r in range(W):
        pieces = []
        for d in range(W):
            # rows rank d computed for rank r sit in d's receive order after the rows from ranks < r
            before = int(sum(ranks[s]["input_splits"][d] for s in range(r)))
            n = int(ranks[r]["input_splits"][d])
            pieces.append(ranks[d]["expert_out"][before:before + n])
        recv_out = np.concatenate(pieces)
        unperm = np.empty_like(recv_out)
        unperm[ranks[r]["perm"]] = recv_out
        T = ranks[r]["x"].shape[0]
        ranks[r]["out"] = combine_weighted_sum(unperm, ranks[r]["topk_weights"], T, k, dtype)
    return ranks


# ----------------------------------------------------------------------------------------
# Decoder-layer norms at the block's edges (layernorm.py:16-40)
# ----------------------------------------------------------------------------------------

def rms_norm(x: np.ndarray, weight: np.ndarray, eps: float, dtype: str,
             residual: np.ndarray | None = None):
    """``RMSNorm.rms_forward(x)`` (layernorm.py:16-26) or, with ``residual``,
    ``add_rms_forward(x, residual)`` (:28-40), which returns ``(out, residual_out)``.

    xf = float(x) (+ float(residual)); residual_out = dtype(xf); var = mean(xf^2);
    out = dtype(dtype(xf * rsqrt(var + eps)) * weight) — the product with the weight is a
    ``dtype`` multiply (one rounding). The mean's summation order is numpy's, so the result
    agrees with the reference to rounding, not bit for bit.
    """
    xf = _cast(x, dtype).astype(np.float32)
    if residual is not None:
        xf = (xf + _cast(residual, dtype).astype(np.float32)).astype(np.float32)
    res_out = _cast(xf, dtype)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=np.float32)
    rs = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    n = _cast((xf * rs).astype(np.float32), dtype)
    out = _cast((n * _cast(weight, dtype)).astype(np.float32), dtype)
    return out if residual is None else (out, res_out)
