"""The decoder layer's norms at the block's edges on the GPU (prism_infer/layers/layernorm.py:16-40
around the MoE block, prism_infer/models/qwen3.py:179-186):

* ``prism_moe_rmsnorm`` (the drop-in ``RMSNorm``) against the reference's own module outputs
  (golden fixtures) and against the oracle at the block's shapes: the residual sum bit for bit,
  the normalised rows within two bf16 units in the last place (the reference's sum of squares is
  Inductor's, in another order) and the fp32 suite tolerance;
* the block with the next layer's residual add + RMSNorm fused into its combine: bit for bit the
  unfused sequence (block, then ``prism_moe_rmsnorm``), for the single-GPU block and for the
  expert-parallel step at ep_size 1, and within tolerance of the oracle.
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import moe_oracle as O
from prism_infer_b200 import capi, synthetic
from prism_infer_b200.engine.parallel import set_expert_parallel_size
from prism_infer_b200.engine.parallel.expert_parallel import ExpertParallelMoE
from prism_infer_b200.layers.layernorm import RMSNorm
from prism_infer_b200.layers.moe import MoE

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_MAX_ABS, BF16_MEAN_REL = 2e-2, 1e-2


def _np(t):
    return t.detach().float().cpu().numpy()


def _ulps_bf16(a, b):
    ia = a.astype(np.float32).view(np.int32) >> 16
    ib = b.astype(np.float32).view(np.int32) >> 16
    ia = np.where(ia < 0, -(ia & 0x7FFF), ia)
    ib = np.where(ib < 0, -(ib & 0x7FFF), ib)
    return np.abs(ia.astype(np.int64) - ib.astype(np.int64))


def check_norm(got, ref, dtype):
    if dtype == torch.float32:
        np.testing.assert_allclose(got, ref, atol=1e-5, rtol=1e-4)
    else:
        # the sum of squares runs in another order (and rsqrt may differ in its last bit): a
        # normalised value near a rounding boundary can land one bf16 step away, and the
        # product with the weight can widen that to two
        u = _ulps_bf16(got, ref)
        assert u.max() <= 2 and (u > 0).mean() < 0.01, (u.max(), (u > 0).mean())


@pytest.mark.parametrize("name", ["rmsnorm_fp32", "rmsnorm_bf16", "rmsnorm_bf16_eps"])
def test_rmsnorm_matches_reference_module(name):
    g = load_golden(name)
    dtype = torch.float32 if str(g["dtype"]) == "float32" else torch.bfloat16
    eps = float(g["eps"])
    x = torch.from_numpy(g["x"]).to(DEV, dtype)
    r = torch.from_numpy(g["residual"]).to(DEV, dtype)
    w = torch.from_numpy(g["weight"]).to(DEV, dtype)
    rms = capi.rmsnorm(x, w, eps)
    add, add_res = capi.rmsnorm(x, w, eps, residual=r)
    torch.cuda.synchronize()
    check_norm(_np(rms), g["rms_out"], dtype)
    check_norm(_np(add), g["add_out"], dtype)
    if dtype == torch.bfloat16:
        assert np.array_equal(_np(add_res), g["add_residual"])
    else:   # the reference's fp32 residual aliases its output (see the oracle test)
        assert torch.equal(add_res, x + r)


@pytest.mark.parametrize("T,H", [(4096, 2048), (257, 4096), (3, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rmsnorm_matches_oracle(T, H, dtype):
    x = (torch.randn(T, H, device=DEV) * 3).to(dtype)
    r = torch.randn(T, H, device=DEV).to(dtype)
    w = (1 + 0.1 * torch.randn(H, device=DEV)).to(dtype)
    norm = RMSNorm(H, eps=1e-6).to(DEV, dtype)
    with torch.no_grad():
        norm.weight.copy_(w)
    rms = norm(x.view(1, T, H)).view(T, H)
    add, add_res = norm(x, r)
    dt = "bfloat16" if dtype == torch.bfloat16 else "float32"
    check_norm(_np(rms), O.rms_norm(_np(x), _np(w), 1e-6, dt), dtype)
    ref, ref_res = O.rms_norm(_np(x), _np(w), 1e-6, dt, residual=_np(r))
    check_norm(_np(add), ref, dtype)
    assert np.array_equal(_np(add_res), ref_res)


def _moe(H, E, k, I, seed):
    set_expert_parallel_size(1)
    wts = synthetic.make_weights_np(H, E, I, seed)
    moe = MoE(H, I, E, k)
    with torch.no_grad():
        moe.gate.weight.copy_(torch.from_numpy(wts.w_gate))
        moe.w_gate_up.copy_(torch.from_numpy(wts.w_gate_up))
        moe.w_down.copy_(torch.from_numpy(wts.w_down))
    return moe.to(DEV, torch.bfloat16), wts


@pytest.mark.parametrize("H,E,k,I,T", [(2048, 128, 8, 768, 512), (256, 32, 4, 128, 37)])
def test_block_with_fused_norm_equals_unfused(H, E, k, I, T):
    moe, wts = _moe(H, E, k, I, seed=H + T)
    norm = RMSNorm(H, eps=1e-6).to(DEV, torch.bfloat16)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(H, device=DEV))
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    res = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    with torch.inference_mode():
        fused, fused_res = moe(x, residual=res, norm=norm)
        y = moe(x)
        ref, ref_res = norm(y, res)
        logits, _, _ = moe.route(x)
    moe.check_device_error()
    assert torch.equal(fused_res, ref_res)
    assert torch.equal(fused, ref)
    # and against the oracle: the block, then the next layer's add_rms_forward
    blk = O.moe_forward(_np(x), wts.w_gate, wts.w_gate_up, wts.w_down, k, True, "bfloat16",
                        logits=_np(logits))["out"]
    o_out, o_res = O.rms_norm(blk, _np(norm.weight), 1e-6, "bfloat16", residual=_np(res))
    for got, want in ((_np(fused), o_out), (_np(fused_res), o_res)):
        d = np.abs(got - want)
        assert d.max() <= 4 * BF16_MAX_ABS, d.max()   # normalised rows: values up to ~4
        assert d.mean() / np.abs(want).mean() <= BF16_MEAN_REL


def test_ep_step_with_fused_norm_equals_unfused():
    H, E, k, I, T = 512, 64, 8, 256, 300
    wts = synthetic.make_weights_np(H, E, I, 3)
    bank = ExpertParallelMoE(H, I, E, 1, 0, transport="p2p")
    with torch.no_grad():
        bank.w_gate_up.copy_(torch.from_numpy(wts.w_gate_up))
        bank.w_down.copy_(torch.from_numpy(wts.w_down))
    bank = bank.to(DEV, torch.bfloat16)
    w_gate = torch.from_numpy(wts.w_gate).to(DEV, torch.bfloat16)
    norm_w = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    res = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    with torch.inference_mode():
        logits = torch.nn.functional.linear(x, w_gate)
        fused, fused_res = bank.forward_p2p(x, router_logits=logits, top_k=k, residual=res,
                                            norm_weight=norm_w, eps=1e-6)
        y = bank.forward_p2p(x, router_logits=logits, top_k=k)
        ref, ref_res = capi.rmsnorm(y, norm_w, 1e-6, residual=res)
    bank.check_device_error()
    assert torch.equal(fused_res, ref_res)
    assert torch.equal(fused, ref)
    bank.release()
