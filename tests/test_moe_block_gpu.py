"""Block-level parity on the GPU: ``prism_infer_b200.layers.moe.MoE`` (the drop-in) against the
oracle and against the reference's own golden outputs.

Routing (ids, per-expert counts) is compared bit-exact; outputs within max-abs 2e-2 and mean
relative 1e-2 (bf16) or the reference suite's atol 1e-5 / rtol 1e-4 (fp32,
prism_infer tests/test_moe.py:64).
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import moe_oracle as O
from prism_infer_b200 import synthetic
from prism_infer_b200.layers.moe import MoE

pytestmark = pytest.mark.gpu

DEV = "cuda"
BF16_MAX_ABS, BF16_MEAN_REL = 2e-2, 1e-2
FP32_ATOL, FP32_RTOL = 1e-5, 1e-4


def build_moe(H, E, k, I, dtype, wts, renorm=True):
    moe = MoE(H, I, E, k, norm_topk_prob=renorm)
    with torch.no_grad():
        moe.gate.weight.copy_(torch.from_numpy(wts.w_gate))
        moe.w_gate_up.copy_(torch.from_numpy(wts.w_gate_up))
        moe.w_down.copy_(torch.from_numpy(wts.w_down))
    return moe.to(device=DEV, dtype=dtype).eval()


def _np(t):
    return t.detach().float().cpu().numpy()


def check_close(out, ref, dtype):
    if dtype == torch.float32:
        np.testing.assert_allclose(out, ref, atol=FP32_ATOL, rtol=FP32_RTOL)
    else:
        d = np.abs(out - ref)
        assert d.max() <= BF16_MAX_ABS, d.max()
        assert d.mean() / max(np.abs(ref).mean(), 1e-12) <= BF16_MEAN_REL


def run_vs_oracle(H, E, k, I, T, dtype, seed, renorm=True, skew=False, shape=None):
    wts = synthetic.make_weights_np(H, E, I, seed, skew=skew, k=k)
    x = synthetic.make_hidden_np(T, H, seed, skew=skew)
    if shape is not None:
        x = x.reshape(*shape, H)
    moe = build_moe(H, E, k, I, dtype, wts, renorm)
    xt = torch.from_numpy(x).to(DEV, dtype)
    with torch.inference_mode():
        logits, ids, w = moe.route(xt)
        out = moe(xt)
    moe.check_device_error()
    assert out.shape == xt.shape and out.dtype == xt.dtype
    dt = "bfloat16" if dtype == torch.bfloat16 else "float32"
    res = O.moe_forward(x, wts.w_gate, wts.w_gate_up, wts.w_down, k, renorm, dt,
                        logits=_np(logits))
    # logits: the reference's F.linear on this device; the oracle's own are within bf16 rounding
    own = O.router_logits(O._cast(x.reshape(-1, H), dt), O._cast(wts.w_gate, dt), dt)
    g = _np(logits)
    ulp = 2.0 ** (-22 if dtype == torch.float32 else -7)   # ~2 ulps of the logits' type
    assert (np.abs(own - g) <= np.abs(g) * ulp + 1e-6).all()
    assert (ids.cpu().numpy() == res["topk_ids"]).all()
    counts = np.bincount(ids.cpu().numpy().ravel(), minlength=E)
    assert (counts == res["counts"]).all()
    check_close(_np(out), res["out"], dtype)
    return moe, out


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("H,E,k,I,T", [(64, 16, 4, 32, 37), (16, 8, 2, 8, 6), (16, 32, 2, 8, 2),
                                       (16, 8, 2, 8, 1), (128, 32, 8, 64, 300),
                                       (64, 24, 6, 32, 20), (256, 64, 8, 128, 1000)])
def test_block_matches_oracle(dtype, H, E, k, I, T):
    run_vs_oracle(H, E, k, I, T, dtype, seed=H + E + k + I + T)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_block_no_renorm_and_multidim(dtype):
    run_vs_oracle(64, 16, 4, 32, 6, dtype, seed=5, renorm=False, shape=(2, 3))


def test_block_skewed_routing():
    run_vs_oracle(256, 64, 8, 128, 512, torch.bfloat16, seed=9, skew=True)


def test_block_config1_full_shape():
    """Benchmark config 1: T=64, H=2048, E=128, k=8, I=768, bf16, all experts local."""
    c = synthetic.CONFIGS[1]
    run_vs_oracle(c["H"], c["E"], c["k"], c["I"], c["T"], torch.bfloat16, synthetic.config_seed(1))


SINGLE_FP32 = ["moe_fp32_small", "moe_fp32_norenorm", "moe_fp32_refshape",
               "moe_fp32_empty_experts", "moe_fp32_single_token", "moe_fp32_multidim",
               "moe_fp32_k6", "moe_fp32_skew"]


@pytest.mark.parametrize("name", SINGLE_FP32)
def test_block_matches_reference_goldens(name):
    """Outputs the reference's own MoE produced (tests/golden/make_golden.py) — fp32, same
    tolerance as prism_infer tests/test_moe.py."""
    g = load_golden(name)
    H, E, k, I = int(g["H"]), int(g["E"]), int(g["k"]), int(g["I"])
    shape = tuple(int(s) for s in g["shape"])
    wts = synthetic.make_weights_np(H, E, I, int(g["seed"]), skew=bool(g["skew"]), k=k)
    x = g["x"]
    moe = build_moe(H, E, k, I, torch.float32, wts, bool(g["renorm"]))
    with torch.inference_mode():
        xt = torch.from_numpy(x).to(DEV)
        _, ids, _ = moe.route(xt)
        out = moe(xt)
    assert (ids.cpu().numpy() == g["topk_ids"].reshape(-1, k)).all()
    np.testing.assert_allclose(_np(out), g["out"], atol=FP32_ATOL, rtol=FP32_RTOL)


def test_block_config0_matches_reference_golden():
    """Benchmark config 0 (T=256, H=2048, E=128, k=8, I=768, fp32) against the reference's
    output recorded on CPU."""
    g = load_golden("cfg0")
    H, E, k, I = int(g["H"]), int(g["E"]), int(g["k"]), int(g["I"])
    seed = int(g["seed"])
    wts = synthetic.make_weights_np(H, E, I, seed)
    x = synthetic.make_hidden_np(int(g["shape"][0]), H, seed)
    moe = build_moe(H, E, k, I, torch.float32, wts)
    with torch.inference_mode():
        xt = torch.from_numpy(x).to(DEV)
        _, ids, w = moe.route(xt)
        out = _np(moe(xt))
    assert (ids.cpu().numpy() == g["topk_ids"]).all()
    np.testing.assert_allclose(_np(w), g["topk_weights"], rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(out[:16], g["out_rows"], atol=FP32_ATOL, rtol=FP32_RTOL)
    np.testing.assert_allclose(out.sum(1), g["out_row_sums"], atol=1e-3, rtol=1e-4)


@pytest.mark.parametrize("cfg", [2, 4])
def test_block_full_size_sampled_tokens(cfg):
    """Configs 2 and 4 at full size on one GPU: routing of every token is checked against the
    oracle on the same logits; outputs of a sample of tokens against the oracle (each token's
    output depends only on its own row)."""
    c = synthetic.CONFIGS[cfg]
    H, E, k, I, T = c["H"], c["E"], c["k"], c["I"], c["T"]
    seed = synthetic.config_seed(cfg)
    wg, wgu, wd = synthetic.make_weights_torch(H, E, I, seed, torch.bfloat16, DEV)
    x = synthetic.make_hidden_torch(T, H, seed, torch.bfloat16, DEV)
    moe = MoE(H, I, E, k).to(DEV, torch.bfloat16)
    with torch.no_grad():
        moe.gate.weight.copy_(wg)
        moe.w_gate_up.copy_(wgu)
        moe.w_down.copy_(wd)
    with torch.inference_mode():
        logits, ids, w = moe.route(x)
        out = moe(x)
    moe.check_device_error()
    r_ids, r_w = O.route(_np(logits), k, True, "bfloat16")
    assert (ids.cpu().numpy() == r_ids).all()
    rng = np.random.default_rng(cfg)
    sample = np.sort(rng.choice(T, 48, replace=False))
    xs = _np(x[torch.from_numpy(sample).to(DEV)])
    prods = np.zeros((len(sample), k, H), np.float32)
    for e in np.unique(r_ids[sample]):
        gu_e, dn_e = _np(wgu[int(e)]), _np(wd[int(e)])
        for i, t in enumerate(sample):
            for j in np.nonzero(r_ids[t] == e)[0]:
                y = O.expert_mlp(xs[i:i + 1], gu_e, dn_e, "bfloat16")
                prods[i, j] = O._cast(y[0] * r_w[t, j], "bfloat16")
    res_out = np.zeros((len(sample), H), np.float32)
    for j in range(k):                     # fp32 sum in slot order, as the combine does
        res_out += prods[:, j]
    check_close(_np(out[torch.from_numpy(sample).to(DEV)]), O._cast(res_out, "bfloat16"),
                torch.bfloat16)
    assert torch.isfinite(out).all()
