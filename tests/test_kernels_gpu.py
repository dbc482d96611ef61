"""Per-kernel parity on the GPU: the CUDA path (through the C ABI) against the oracle.

Integer outputs (top-k ids, counts, plans, permutations) must be bit-exact. Floating outputs
carry the tolerance written in each test. The oracle's tie rule for torch.topk is pinned here
against torch's own CUDA ops (the reference calls F.softmax / torch.topk / sum / cast,
prism_infer/layers/moe.py:77-81).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import moe_oracle as O
from prism_infer_b200 import capi

pytestmark = pytest.mark.gpu

DEV = "cuda"
BF16_MAX_ABS, BF16_MEAN_REL = 2e-2, 1e-2


def _np(t):
    return t.detach().float().cpu().numpy()


def torch_route(logits, k, renorm):
    """The reference's routing ops (moe.py:77-81) run by torch on CUDA."""
    rw = F.softmax(logits, dim=-1, dtype=torch.float)
    w, ids = torch.topk(rw, k, dim=-1)
    if renorm:
        w = w / w.sum(dim=-1, keepdim=True)
    return ids, w.to(logits.dtype), rw


def tied_logits(T, E, dtype, levels, gen):
    """Logits drawn from a few values so that ties at and inside the top-k are common."""
    q = torch.randint(0, levels, (T, E), generator=gen, device=DEV)
    return (q.float() * 0.25 - 1.0).to(dtype)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("E,k", [(128, 8), (8, 2), (16, 4), (24, 6), (256, 8), (60, 1), (32, 32)])
@pytest.mark.parametrize("kind", ["normal", "tied"])
def test_route_matches_torch_cuda_and_oracle(dtype, E, k, kind):
    gen = torch.Generator(device=DEV).manual_seed(E * 100 + k)
    T = 777
    if kind == "normal":
        logits = (torch.randn(T, E, generator=gen, device=DEV) * 0.9).to(dtype)
    else:
        logits = tied_logits(T, E, dtype, 5, gen)
    for renorm in (True, False):
        ids, w, counts = capi.route_topk(logits, k, renorm, with_counts=True)
        t_ids, t_w, t_probs = torch_route(logits, k, renorm)
        # bit-exact with torch on CUDA: ids and weights
        assert torch.equal(ids, t_ids), "top-k ids differ from torch.topk on CUDA"
        if k & (k - 1) == 0:
            assert torch.equal(w.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                               t_w.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))
        else:
            torch.testing.assert_close(w, t_w, rtol=1e-6 if dtype == torch.float32 else 8e-3,
                                       atol=1e-7)
        # the oracle's tie rule reproduces torch.topk on CUDA (pins the oracle)
        o_vals, o_ids = O.topk_torch_cuda(_np(t_probs), k)
        assert (o_ids == t_ids.cpu().numpy()).all()
        # the oracle end to end on the same logits
        r_ids, r_w = O.route(_np(logits), k, renorm, "bfloat16" if dtype == torch.bfloat16 else "float32")
        assert (r_ids == ids.cpu().numpy()).all()
        np.testing.assert_allclose(r_w, _np(w), rtol=8e-3 if dtype == torch.bfloat16 else 2e-6,
                                   atol=1e-6)
        assert torch.equal(counts.long().cpu(), torch.bincount(ids.flatten().cpu(), minlength=E))


def test_route_empty_and_single_token():
    for T in (0, 1):
        logits = torch.randn(T, 128, device=DEV).to(torch.bfloat16)
        ids, w, _ = capi.route_topk(logits, 8, True)
        assert ids.shape == (T, 8)
        if T:
            assert torch.equal(ids, torch_route(logits, 8, True)[0])


# ------------------------------------------------------------------------- dispatch plan

def test_dispatch_plan_reference_golden_vector():
    # prism_infer tests/test_expert_parallel.py:15-22
    ids = torch.tensor([[0, 5], [2, 3]], dtype=torch.int64, device=DEV)
    plan = capi.dispatch_plan(ids, 8, 4)
    assert plan["input_splits"].tolist() == [1, 2, 1, 0]
    assert plan["perm"].tolist() == [0, 2, 3, 1]
    assert plan["sorted_local_eid"].tolist() == [0, 0, 1, 1]


@pytest.mark.parametrize("T,k,E,W", [(8192, 8, 128, 8), (8192, 8, 128, 1), (4097, 8, 128, 2),
                                     (7, 3, 8, 4), (1, 2, 8, 4), (300, 4, 64, 4),
                                     (2000, 8, 1024, 8), (513, 6, 24, 3)])
def test_dispatch_plan_matches_oracle(T, k, E, W):
    gen = torch.Generator(device=DEV).manual_seed(T + k + E + W)
    # skewed ids: many entries on few experts, some experts empty
    logits = torch.randn(T, E, generator=gen, device=DEV) + torch.linspace(0, 3, E, device=DEV)
    ids = torch.topk(logits, k, dim=-1).indices.contiguous()
    plan = capi.dispatch_plan(ids, E, W)
    ids_np = ids.cpu().numpy()
    perm, splits, sleid = O.build_dispatch_plan(ids_np, E // W, W)
    assert (plan["perm"].cpu().numpy() == perm).all()
    assert (plan["input_splits"].cpu().numpy() == splits).all()
    assert (plan["sorted_local_eid"].cpu().numpy() == sleid).all()
    counts = O.expert_counts(ids_np, E)
    assert (plan["expert_counts"].cpu().numpy() == counts).all()
    assert (plan["expert_offsets"].cpu().numpy() == np.concatenate([[0], np.cumsum(counts)])).all()
    order = O.expert_major_order(ids_np, E)            # order[row] = flat entry
    entry_row = plan["entry_row"].cpu().numpy()
    assert (entry_row[order] == np.arange(T * k)).all()


def test_dispatch_plan_empty():
    ids = torch.empty(0, 8, dtype=torch.int64, device=DEV)
    plan = capi.dispatch_plan(ids, 128, 8)
    assert plan["input_splits"].tolist() == [0] * 8
    assert plan["expert_offsets"].tolist() == [0] * 129


# ------------------------------------------------------------------------- permute / combine

@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T,H,k", [(513, 2048, 8), (37, 64, 4), (1, 4096, 8), (100, 16, 2)])
def test_permute_rows_exact(dtype, T, H, k):
    E = 32
    x = torch.randn(T, H, device=DEV).to(dtype)
    ids = torch.stack([torch.randperm(E, device=DEV)[:k] for _ in range(T)]).contiguous()
    plan = capi.dispatch_plan(ids, E, 1, want_perm=False)
    xs = capi.permute_rows(x, k, plan["entry_row"])
    order = O.expert_major_order(ids.cpu().numpy(), E)
    ref = x.cpu()[torch.from_numpy(order // k)]
    assert torch.equal(xs.cpu(), ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("T,H,k", [(513, 2048, 8), (37, 64, 4), (5, 4096, 8), (2, 8, 2)])
def test_combine_matches_reference_numerics(dtype, T, H, k):
    y = torch.randn(T * k, H, device=DEV).to(dtype)
    w = torch.rand(T, k, device=DEV)
    w = (w / w.sum(-1, keepdim=True)).to(dtype)
    perm = torch.randperm(T * k, device=DEV)
    entry_row = perm.to(torch.int32)
    out = capi.combine(y, w, entry_row=entry_row)
    unperm = y[perm.long()]
    ref = O.combine_weighted_sum(_np(unperm), _np(w), T, k,
                                 "bfloat16" if dtype == torch.bfloat16 else "float32")
    if dtype == torch.bfloat16:
        assert (ref == _np(out)).all(), "bf16 combine must equal combine_weighted_sum bit for bit"
    else:
        np.testing.assert_allclose(_np(out), ref, rtol=1e-6, atol=1e-6)
    # identity entry_row == reference combine_weighted_sum on unpermuted rows
    out2 = capi.combine(unperm.contiguous(), w)
    assert torch.equal(out, out2)


# ------------------------------------------------------------------------- grouped experts

def _segments(counts, device=DEV):
    off = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    return torch.from_numpy(off).to(device)


@pytest.mark.parametrize("H,I,counts", [
    (256, 128, [130, 0, 1, 255, 128, 3]),          # ragged, empty, one-row segments
    (2048, 768, [512, 37, 0, 200]),                # Qwen3-30B-A3B expert shape
    (64, 32, [5, 9, 1]),                           # K and N smaller than one tile
    (320, 200, [129, 64]),                         # K, N not multiples of the tile
    (4096, 1536, [300]),                           # Qwen3-235B-A22B expert shape
    (1024, 512, [2000, 1500, 0, 2100, 1999, 2001, 1]),   # more m-tiles than the fused lag
])
@pytest.mark.parametrize("dtype,engine", [(torch.bfloat16, "fused"), (torch.bfloat16, "single"),
                                          (torch.bfloat16, "pair"), (torch.float32, "simt")])
def test_expert_swiglu_matches_oracle(H, I, counts, dtype, engine, expert_engine):
    """``engine``: bf16 tcgen05 with both GEMMs in one persistent launch (128-row tiles), two
    launches of single-CTA tiles (128 rows), or two launches of CTA-pair tiles (256 rows,
    cta_group::2); fp32 runs on CUDA cores."""
    if dtype == torch.float32 and H * I > 2048 * 768:
        pytest.skip("fp32 CUDA-core path is exercised at the smaller shapes")
    if dtype == torch.float32 and sum(counts) > 5000:
        pytest.skip("fp32 CUDA-core path is exercised at the smaller row counts")
    if dtype == torch.bfloat16:
        expert_engine(engine)
    gen = torch.Generator(device=DEV).manual_seed(H + I + len(counts))
    E = len(counts)
    R = int(sum(counts))
    x = torch.randn(R, H, generator=gen, device=DEV).to(dtype)
    wgu = (torch.randn(E, 2 * I, H, generator=gen, device=DEV) / H ** 0.5).to(dtype)
    wd = (torch.randn(E, H, I, generator=gen, device=DEV) / I ** 0.5).to(dtype)
    seg = _segments(counts)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    y = torch.full((R, H), float("nan"), device=DEV).to(dtype)
    capi.expert_swiglu(x, seg, wgu, wd, y=y, device_error=err)
    assert capi.read_device_error(err) == 0
    dt = "bfloat16" if dtype == torch.bfloat16 else "float32"
    xn, gun, dnn, yn = _np(x), _np(wgu), _np(wd), _np(y)
    off = seg.cpu().numpy()
    for e in range(E):
        a, b = off[e], off[e + 1]
        if a == b:
            continue
        ref = O.expert_mlp(xn[a:b], gun[e], dnn[e], dt)
        got = yn[a:b]
        assert np.isfinite(got).all()
        if dtype == torch.bfloat16:
            d = np.abs(got - ref)
            assert d.max() <= BF16_MAX_ABS, (e, d.max())
            assert d.mean() / np.abs(ref).mean() <= BF16_MEAN_REL
        else:
            np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("engine", ["fused", "single", "pair"])
def test_expert_swiglu_segment_expert_map(engine, expert_engine):
    """Segments may name any local expert (EP receiver layout: (source rank, local expert))."""
    expert_engine(engine)
    H, I, El = 256, 128, 3
    x = torch.randn(300, H, device=DEV).to(torch.bfloat16)
    wgu = (torch.randn(El, 2 * I, H, device=DEV) / 16).to(torch.bfloat16)
    wd = (torch.randn(El, H, I, device=DEV) / 11).to(torch.bfloat16)
    counts = [50, 0, 70, 30, 100, 50]
    seg = _segments(counts)
    seg_expert = torch.tensor([0, 1, 2, 0, 1, 2], dtype=torch.int32, device=DEV)
    y = capi.expert_swiglu(x, seg, wgu, wd, seg_expert=seg_expert)
    off = seg.cpu().numpy()
    for s, e in enumerate(seg_expert.tolist()):
        a, b = off[s], off[s + 1]
        if a < b:
            ref = O.expert_mlp(_np(x[a:b]), _np(wgu[e]), _np(wd[e]), "bfloat16")
            assert np.abs(_np(y[a:b]) - ref).max() <= BF16_MAX_ABS
