"""The allocation-free dispatch plan (``prism_moe_build_dispatch_plan_static``).

Some callers of this library cannot allocate device memory where they call it — a plugin
running inside a host framework's execute callback that only receives the buffers that
framework owns, or an embedded runtime whose device memory all belongs to its own pool. The
static-scratch entry point serves them: it takes no workspace and keeps its scratch in a fixed
array inside the library.

This test calls it through the C ABI and checks that its outputs equal those of the
workspace entry point ``prism_moe_build_dispatch_plan`` bit for bit (integer outputs: the
tolerance is zero), on two different calls in a row — the second must not see anything left in
the shared array by the first. It lives in its own file, collected last, and needs no other
test to have run first.
"""
import ctypes

import pytest
import torch

from prism_infer_b200 import capi

pytestmark = pytest.mark.gpu


def static_plan(ids, E, W):
    T, k = ids.shape
    dev = ids.device
    N = T * k
    out = dict(perm=torch.full((N,), -7, dtype=torch.int64, device=dev),
               input_splits=torch.full((W,), -7, dtype=torch.int64, device=dev),
               sorted_local_eid=torch.full((N,), -7, dtype=torch.int64, device=dev),
               expert_counts=torch.full((E,), -7, dtype=torch.int32, device=dev),
               expert_offsets=torch.full((E + 1,), -7, dtype=torch.int32, device=dev),
               entry_row=torch.full((N,), -7, dtype=torch.int32, device=dev))
    lib = capi.load()
    st = lib.prism_moe_build_dispatch_plan_static(
        ids.data_ptr(), T, k, E, W, out["perm"].data_ptr(), out["input_splits"].data_ptr(),
        out["sorted_local_eid"].data_ptr(), out["expert_counts"].data_ptr(),
        out["expert_offsets"].data_ptr(), out["entry_row"].data_ptr(),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    capi.check(st, "prism_moe_build_dispatch_plan_static")
    return out


def routed_ids(T, k, E, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    logits = torch.randn(T, E, generator=gen, device="cuda")
    logits += torch.linspace(0, 2, E, device="cuda")      # uneven loads, some heavy experts
    return torch.topk(logits, k, dim=-1).indices.contiguous()


@pytest.mark.parametrize("order", ["large_then_small", "small_then_large"])
def test_static_plan_equals_workspace_plan_twice_in_a_row(order):
    cases = [(8192, 8, 128, 8, 1), (300, 6, 24, 3, 2)]     # (T, k, E, W, seed); 8192*8 = limit
    if order == "small_then_large":
        cases = cases[::-1]
    for T, k, E, W in [c[:4] for c in cases]:
        ids = routed_ids(T, k, E, seed=T + E)
        got = static_plan(ids, E, W)
        ref = capi.dispatch_plan(ids, E, W)
        torch.cuda.synchronize()
        for key in ("perm", "input_splits", "sorted_local_eid", "expert_counts",
                    "expert_offsets", "entry_row"):
            assert torch.equal(got[key], ref[key]), f"{key} differs (T={T}, E={E}, W={W})"


def test_static_plan_rejects_sizes_beyond_its_limits():
    lib = capi.load()
    ids = torch.zeros(8193, 8, dtype=torch.int64, device="cuda")   # 65,544 entries > 65,536
    st = lib.prism_moe_build_dispatch_plan_static(ids.data_ptr(), 8193, 8, 128, 8, None, None,
                                                  None, None, None, None, None)
    assert st == capi.ERR_ARG and "static limit" in capi.last_error()
    st = lib.prism_moe_build_dispatch_plan_static(ids.data_ptr(), 4, 8, 512, 8, None, None,
                                                  None, None, None, None, None)
    assert st == capi.ERR_ARG and "num_experts" in capi.last_error()
