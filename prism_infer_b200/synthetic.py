"""Seeded synthetic workloads for the Qwen3-MoE sparse block.

The reference publishes no dataset for this path; its benchmark configurations are
synthetic shapes with stated value distributions:

* hidden ~ N(0, 1)
* router weight W_g[E, H] ~ N(0, 0.02)
* expert gate/up weight W_gu[E, 2I, H] ~ N(0, 1/sqrt(H))   (rows 0..I-1 gate, I..2I-1 up,
  the fused layout of MergedColumnParallelLinear, prism_infer/layers/linear.py:102-119)
* expert down weight W_d[E, H, I] ~ N(0, 1/sqrt(I))

Two generators are provided:

* ``numpy`` (PCG64 via ``np.random.default_rng``) — platform independent, used for parity
  tests and golden fixtures so that the same seed gives the same bits on every host;
* ``torch`` on a CUDA device — fast generation of the full-size benchmark tensors, where
  only size-independent properties are checked.

Skewed routing (benchmark config 3) needs an additive per-expert logit bias. The
reference router is ``F.linear(x, W_g)`` with no bias term (prism_infer/layers/moe.py:55,74),
so the bias is carried through the inputs themselves: hidden feature 0 of every token is
set to 1.0 and column 0 of the router weight holds the bias, giving
``logit[t, e] = b[e] + sum_{h>=1} W_g[e, h] x[t, h]`` through the reference's own forward.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

# Benchmark configurations (shapes only; the dtype is the compute dtype).
CONFIGS = {
    0: dict(name="cfg0-cpu-fp32", T=256, H=2048, E=128, k=8, I=768, dtype="float32", skew=False),
    1: dict(name="cfg1-decode-bf16", T=64, H=2048, E=128, k=8, I=768, dtype="bfloat16", skew=False),
    2: dict(name="cfg2-prefill-bf16", T=8192, H=2048, E=128, k=8, I=768, dtype="bfloat16", skew=False),
    3: dict(name="cfg3-skew-bf16", T=4096, H=2048, E=128, k=8, I=768, dtype="bfloat16", skew=True),
    4: dict(name="cfg4-235b-bf16", T=16384, H=4096, E=128, k=8, I=1536, dtype="bfloat16", skew=False),
}


def config_seed(cfg: int, rank: int = 0) -> int:
    """Seed of benchmark config ``cfg`` on EP rank ``rank`` (weights use rank 0's seed)."""
    return 1000 * cfg + rank


@dataclass
class BlockWeights:
    """Full (all-expert) weights of one MoE block, as float32 numpy arrays."""
    w_gate: np.ndarray        # [E, H]
    w_gate_up: np.ndarray     # [E, 2I, H]
    w_down: np.ndarray        # [E, H, I]
    bias: np.ndarray | None = field(default=None)   # [E] logit bias folded into w_gate[:, 0]


def zipf_bias(E: int, k: int, rng: np.random.Generator, s: float = 1.2,
              top_load_ratio: float = 8.0, H_probe: int = 256, T_probe: int = 4096) -> np.ndarray:
    """Per-expert additive logit bias: Zipf(s) over a seeded expert permutation.

    ``b[perm[r]] = alpha * log(1 / (r+1)^s)``; ``alpha`` is found by bisection so that, for
    near-uniform router logits (N(0,1) hidden, N(0,0.02) router weight), the most loaded
    expert receives ``top_load_ratio`` times the mean load ``T*k/E``.
    """
    perm = rng.permutation(E)
    base = -s * np.log(np.arange(1, E + 1, dtype=np.float64))
    shape = np.empty(E)
    shape[perm] = base
    probe_rng = np.random.default_rng(12345)
    logits0 = (probe_rng.standard_normal((T_probe, H_probe)) @
               (probe_rng.standard_normal((H_probe, E)) * 0.02)) * math.sqrt(2048 / H_probe)

    def top_ratio(alpha: float) -> float:
        lg = logits0 + alpha * shape[None, :]
        top = np.argpartition(-lg, k - 1, axis=1)[:, :k]
        load = np.bincount(top.ravel(), minlength=E)
        return load.max() / (T_probe * k / E)

    lo, hi = 0.0, 4.0
    for _ in range(40):
        mid = 0.5 * (lo + hi)
        if top_ratio(mid) < top_load_ratio:
            lo = mid
        else:
            hi = mid
    return (0.5 * (lo + hi) * shape).astype(np.float32)


def make_weights_np(H: int, E: int, I: int, seed: int, skew: bool = False, k: int = 8,
                    experts: slice | None = None) -> BlockWeights:
    """Seeded block weights (float32 numpy). ``experts`` restricts the expert weights generated
    (the full stream is still drawn in the same order, so the values do not depend on it)."""
    rng = np.random.default_rng(seed)
    w_gate = (rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.02))
    bias = None
    if skew:
        bias = zipf_bias(E, k, np.random.default_rng(seed + 7))
        w_gate[:, 0] = bias
    sel = range(E) if experts is None else range(E)[experts]
    gu = np.empty((len(sel), 2 * I, H), dtype=np.float32)
    dn = np.empty((len(sel), H, I), dtype=np.float32)
    sg = np.float32(1.0 / math.sqrt(H))
    sd = np.float32(1.0 / math.sqrt(I))
    j = 0
    for e in range(E):
        a = rng.standard_normal((2 * I, H), dtype=np.float32)
        b = rng.standard_normal((H, I), dtype=np.float32)
        if e in sel:
            gu[j] = a * sg
            dn[j] = b * sd
            j += 1
    return BlockWeights(w_gate, gu, dn, bias)


def make_hidden_np(T: int, H: int, seed: int, skew: bool = False) -> np.ndarray:
    """Seeded hidden states [T, H] ~ N(0,1) (float32 numpy)."""
    rng = np.random.default_rng(seed + 500_000)
    x = rng.standard_normal((T, H), dtype=np.float32)
    if skew:
        x[:, 0] = 1.0
    return x


def make_weights_torch(H: int, E: int, I: int, seed: int, dtype, device, skew: bool = False,
                       k: int = 8, expert_range: tuple[int, int] | None = None):
    """Full-size block weights generated on ``device`` with a seeded torch generator.

    Returns (w_gate [E,H], w_gate_up [E_sel,2I,H], w_down [E_sel,H,I]) in ``dtype``. Expert
    ``e`` is drawn from its own generator seeded with ``seed*1009 + e`` so that an EP rank can
    generate only its local experts and still hold the same values as a single GPU.
    """
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    w_gate = torch.randn(E, H, generator=g, device=device) * 0.02
    if skew:
        bias = torch.from_numpy(zipf_bias(E, k, np.random.default_rng(seed + 7))).to(device)
        w_gate[:, 0] = bias
    lo, hi = expert_range if expert_range is not None else (0, E)
    gu = torch.empty(hi - lo, 2 * I, H, device=device, dtype=dtype)
    dn = torch.empty(hi - lo, H, I, device=device, dtype=dtype)
    for e in range(lo, hi):
        gu[e - lo], dn[e - lo] = expert_weights_torch(H, I, seed, e, dtype, device)
    return w_gate.to(dtype), gu, dn


def expert_weights_torch(H: int, I: int, seed: int, e: int, dtype, device):
    """Expert ``e``'s (w_gate_up [2I,H], w_down [H,I]) exactly as ``make_weights_torch`` draws
    them (its own generator, seeded ``seed*1009 + e``)."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed * 1009 + e)
    gu = (torch.randn(2 * I, H, generator=g, device=device) / math.sqrt(H)).to(dtype)
    dn = (torch.randn(H, I, generator=g, device=device) / math.sqrt(I)).to(dtype)
    return gu, dn


def make_hidden_torch(T: int, H: int, seed: int, dtype, device, skew: bool = False):
    """Hidden states [T, H] ~ N(0,1) generated on ``device``."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed + 500_000)
    x = torch.randn(T, H, generator=g, device=device)
    if skew:
        x[:, 0] = 1.0
    return x.to(dtype)
