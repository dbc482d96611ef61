"""ctypes binding of ``libprism_moe.so`` (the C ABI declared in ``include/prism_moe.h``).

The library is loaded on first use. There is no fallback: if the library is missing, or the
current device is not an sm_100 GPU, calls raise ``RuntimeError``.

The torch-facing helpers below validate dtype / device / contiguity, pass raw pointers and the
current CUDA stream, and raise ``RuntimeError`` with the library's message on a non-zero
status (the reference surfaces torch ``RuntimeError`` the same way, prism_infer
layers/moe.py:69-100).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libprism_moe.so"
HEADER = Path(__file__).resolve().parent.parent / "include" / "prism_moe.h"

OK, ERR_ARG, ERR_CUDA, ERR_TIMEOUT, ERR_UNSUPPORTED, ERR_DEVICE = range(6)
F32, BF16 = 0, 1
ENGINES = {"auto": 0, "fused": 1, "single": 2, "pair": 3}
EP_STATS_FIELDS = ("epoch", "counter", "dispatch_t0_ns", "dispatch_t1_ns", "fused_t0_ns",
                   "fused_t1_ns", "send_rows", "recv_rows")

_vp, _i32, _i64, _sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t


class NormEpilogue(ctypes.Structure):
    """``prism_moe_norm_epilogue``: the decoder layer's residual add + RMSNorm fused into the
    block's combine."""
    _fields_ = [("residual", ctypes.c_void_p), ("norm_weight", ctypes.c_void_p),
                ("eps", ctypes.c_float), ("residual_out", ctypes.c_void_p)]


_ep = ctypes.POINTER(NormEpilogue)
_SIGNATURES = {
    "prism_moe_version": (ctypes.c_int, []),
    "prism_moe_last_error": (ctypes.c_char_p, []),
    "prism_moe_route_topk": (ctypes.c_int, [_vp, ctypes.c_int, _i64, _i32, _i32, _i32, _vp, _vp,
                                            _vp, _vp]),
    "prism_moe_dispatch_workspace_size": (_sz, [_i64, _i32, _i32, _i32]),
    "prism_moe_build_dispatch_plan": (ctypes.c_int, [_vp, _i64, _i32, _i32, _i32, _vp, _vp, _vp,
                                                     _vp, _vp, _vp, _vp, _sz, _vp]),
    "prism_moe_build_dispatch_plan_static": (ctypes.c_int, [_vp, _i64, _i32, _i32, _i32, _vp,
                                                            _vp, _vp, _vp, _vp, _vp, _vp]),
    "prism_moe_permute_rows": (ctypes.c_int, [_vp, ctypes.c_int, _i64, _i64, _i32, _vp, _vp,
                                              _vp]),
    "prism_moe_expert_workspace_size": (_sz, [_i64, _i64, _i64, ctypes.c_int]),
    "prism_moe_expert_swiglu": (ctypes.c_int, [_vp, ctypes.c_int, _i64, _i64, _i64, _vp, _vp,
                                               _i32, _i32, _vp, _vp, _vp, _vp, _sz, _vp, _vp]),
    "prism_moe_combine": (ctypes.c_int, [_vp, ctypes.c_int, _vp, _vp, _i64, _i32, _i64, _vp,
                                         _vp]),
    "prism_moe_block_workspace_size": (_sz, [_i64, _i64, _i64, _i32, _i32, ctypes.c_int]),
    "prism_moe_block_forward": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _i64, _i64, _i64, _i32,
                                               _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                                               _vp]),
    "prism_moe_ep_landing_bytes": (_sz, [_i32, _i64, _i32, _i64, _i32, ctypes.c_int]),
    "prism_moe_ep_alloc_landing": (ctypes.c_int, [_sz, ctypes.POINTER(_vp), _vp]),
    "prism_moe_ep_free_landing": (ctypes.c_int, [_vp]),
    "prism_moe_ep_ipc_handle_bytes": (ctypes.c_int, []),
    "prism_moe_ep_open_peer": (ctypes.c_int, [_vp, ctypes.POINTER(_vp)]),
    "prism_moe_ep_close_peer": (ctypes.c_int, [_vp]),
    "prism_moe_ep_workspace_size": (_sz, [_i64, _i64, _i64, _i32, _i32, _i32, ctypes.c_int]),
    "prism_moe_ep_forward": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, _i64, _i64, _i64,
                                            _i64, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp,
                                            _vp, ctypes.c_uint64, _vp, _vp, _sz, _vp]),
    "prism_moe_ep_read_stats": (ctypes.c_int, [_vp, ctypes.POINTER(ctypes.c_uint64), _vp]),
    "prism_moe_set_expert_engine": (ctypes.c_int, [ctypes.c_int]),
    "prism_moe_set_wait_limits": (ctypes.c_int, [_i64, _i64]),
    "prism_moe_rmsnorm": (ctypes.c_int, [_vp, _vp, _vp, ctypes.c_float, ctypes.c_int, _i64, _i64,
                                         _vp, _vp, _vp]),
    "prism_moe_block_forward_norm": (ctypes.c_int, [_vp, _vp, ctypes.c_int, _i64, _i64, _i64, _i32,
                                                    _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                                                    _vp, _ep]),
    "prism_moe_ep_forward_norm": (ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int, _i64, _i64,
                                                 _i64, _i64, _i32, _i32, _i32, _i32, _i32, _vp,
                                                 _vp, _vp, _vp, ctypes.c_uint64, _vp, _vp, _sz,
                                                 _vp, _ep]),
    "prism_moe_profile_events": (ctypes.c_int, [ctypes.POINTER(_vp), _i32]),
    "prism_moe_read_device_error": (ctypes.c_int, [_vp, _vp]),
}

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libprism_moe.so (once) and declare every entry point's signature."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m prism_infer_b200.build` "
                    "(the MoE block has no CPU or eager fallback)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    msg = load().prism_moe_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str) -> None:
    if status != OK:
        raise RuntimeError(f"{what} failed with status {status}: {last_error()}")


# ---------------------------------------------------------------------------------- torch glue

def _torch():
    import torch
    return torch


def dtype_code(dt) -> int:
    torch = _torch()
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float32:
        return F32
    raise RuntimeError(f"prism MoE kernels support bfloat16 and float32, got {dt}")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(device) -> int:
    torch = _torch()
    return torch.cuda.current_stream(device).cuda_stream


def _need_cuda(*ts):
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("prism MoE kernels run on CUDA tensors only (no CPU fallback)")
        if not t.is_contiguous():
            raise RuntimeError("prism MoE kernels need contiguous tensors")


def route_topk(logits, top_k: int, renorm: bool, with_counts: bool = False):
    """Kernel 1 on ``logits`` [T, E]: returns (topk_ids int64 [T,k], topk_weights [T,k],
    expert_counts int32 [E] or None)."""
    torch = _torch()
    _need_cuda(logits)
    T, E = logits.shape
    ids = torch.empty(T, top_k, dtype=torch.int64, device=logits.device)
    w = torch.empty(T, top_k, dtype=logits.dtype, device=logits.device)
    counts = torch.empty(E, dtype=torch.int32, device=logits.device) if with_counts else None
    check(load().prism_moe_route_topk(ptr(logits), dtype_code(logits.dtype), T, E, top_k,
                                      int(bool(renorm)), ptr(ids), ptr(w), ptr(counts),
                                      stream_of(logits.device)), "prism_moe_route_topk")
    return ids, w, counts


def dispatch_plan(topk_ids, num_experts: int, ep_size: int, want_perm: bool = True):
    """Kernel 2 (plan) on ``topk_ids`` [T, k] int64. Returns a dict of int tensors: perm,
    input_splits, sorted_local_eid (int64, reference layout) and expert_counts,
    expert_offsets, entry_row (int32, expert-major layout)."""
    torch = _torch()
    _need_cuda(topk_ids)
    if topk_ids.dtype != torch.int64:
        raise RuntimeError("topk_ids must be int64")
    T, k = topk_ids.shape
    dev = topk_ids.device
    N = T * k
    lib = load()
    ws_bytes = lib.prism_moe_dispatch_workspace_size(T, k, num_experts, ep_size)
    ws = torch.zeros(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    out = dict(
        perm=torch.empty(N, dtype=torch.int64, device=dev) if want_perm else None,
        input_splits=torch.empty(ep_size, dtype=torch.int64, device=dev) if want_perm else None,
        sorted_local_eid=torch.empty(N, dtype=torch.int64, device=dev) if want_perm else None,
        expert_counts=torch.empty(num_experts, dtype=torch.int32, device=dev),
        expert_offsets=torch.empty(num_experts + 1, dtype=torch.int32, device=dev),
        entry_row=torch.empty(N, dtype=torch.int32, device=dev),
    )
    check(lib.prism_moe_build_dispatch_plan(
        ptr(topk_ids), T, k, num_experts, ep_size, ptr(out["perm"]), ptr(out["input_splits"]),
        ptr(out["sorted_local_eid"]), ptr(out["expert_counts"]), ptr(out["expert_offsets"]),
        ptr(out["entry_row"]), ptr(ws), ws_bytes, stream_of(dev)), "prism_moe_build_dispatch_plan")
    return out


def permute_rows(x, top_k: int, entry_row, out=None):
    """x_sorted[entry_row[t*k+j]] = x[t] (rows not named by entry_row are left as they are)."""
    torch = _torch()
    _need_cuda(x, entry_row)
    T, H = x.shape
    if out is None:
        out = torch.empty(T * top_k, H, dtype=x.dtype, device=x.device)
    check(load().prism_moe_permute_rows(ptr(x), dtype_code(x.dtype), T, H, top_k, ptr(entry_row),
                                        ptr(out), stream_of(x.device)), "prism_moe_permute_rows")
    return out


def expert_swiglu(x_sorted, seg_offsets, w_gate_up, w_down, seg_expert=None, y=None,
                  device_error=None):
    """Kernel 4: grouped SwiGLU experts over the segment table (int32 device tensors)."""
    torch = _torch()
    _need_cuda(x_sorted, seg_offsets, w_gate_up, w_down, seg_expert)
    R, H = x_sorted.shape
    El, twoI, H2 = w_gate_up.shape
    I = twoI // 2
    if H2 != H or tuple(w_down.shape) != (El, H, I):
        raise RuntimeError("expert weight shapes do not match x_sorted")
    if w_gate_up.dtype != x_sorted.dtype or w_down.dtype != x_sorted.dtype:
        raise RuntimeError("expert weights must have the activations' dtype")
    lib = load()
    dt = dtype_code(x_sorted.dtype)
    ws_bytes = lib.prism_moe_expert_workspace_size(R, H, I, dt)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x_sorted.device)
    if y is None:
        y = torch.empty_like(x_sorted)
    nseg = seg_offsets.numel() - 1
    check(lib.prism_moe_expert_swiglu(ptr(x_sorted), dt, R, H, I, ptr(seg_offsets),
                                      ptr(seg_expert), nseg, El, ptr(w_gate_up), ptr(w_down),
                                      ptr(y), ptr(ws), ws_bytes, ptr(device_error),
                                      stream_of(x_sorted.device)), "prism_moe_expert_swiglu")
    return y


def combine(expert_out, topk_weights, entry_row=None, out=None):
    """Kernel 5: out[t] = sum_j w[t,j] * expert_out[row(t*k+j)]."""
    torch = _torch()
    _need_cuda(expert_out, topk_weights, entry_row)
    T, k = topk_weights.shape
    H = expert_out.shape[-1]
    if topk_weights.dtype != expert_out.dtype:
        raise RuntimeError("topk_weights must have the expert outputs' dtype")
    if out is None:
        out = torch.empty(T, H, dtype=expert_out.dtype, device=expert_out.device)
    check(load().prism_moe_combine(ptr(expert_out), dtype_code(expert_out.dtype), ptr(entry_row),
                                   ptr(topk_weights), T, k, H, ptr(out),
                                   stream_of(expert_out.device)), "prism_moe_combine")
    return out


_ws_lock = threading.Lock()
_workspaces: dict = {}


def block_workspace(device, nbytes: int):
    """Per-(device, stream) scratch for ``prism_moe_block_forward``; grows on demand. The first
    four bytes are the kernels' device error word (kept zero)."""
    torch = _torch()
    stream = torch.cuda.current_stream(device).cuda_stream
    key = (device.index, stream)
    with _ws_lock:
        ws = _workspaces.get(key)
        if ws is None or ws.numel() < nbytes:
            ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
            _workspaces[key] = ws
    return ws


def block_error_word(device):
    """The device error word of the current stream's block workspace (None before any call)."""
    torch = _torch()
    ws = _workspaces.get((device.index, torch.cuda.current_stream(device).cuda_stream))
    return None if ws is None else ws[:4].view(torch.int32)


def norm_epilogue(residual, norm_weight, eps: float, residual_out):
    """A ``prism_moe_norm_epilogue`` for the *_norm entry points (None when ``norm_weight`` is
    None). The tensors must stay alive for the call."""
    if norm_weight is None:
        return None
    _need_cuda(residual, norm_weight, residual_out)
    return NormEpilogue(residual.data_ptr(), norm_weight.data_ptr(), float(eps),
                        residual_out.data_ptr())


def rmsnorm(x, weight, eps: float, residual=None):
    """RMSNorm of ``x`` [T,H] (prism_moe_rmsnorm); with ``residual``, of ``x + residual``, and
    returns (out, residual_out) as the reference's add_rms_forward does."""
    torch = _torch()
    _need_cuda(x, weight, residual)
    T, H = x.shape
    if weight.shape != (H,) or weight.dtype != x.dtype or (
            residual is not None and (residual.shape != x.shape or residual.dtype != x.dtype)):
        raise RuntimeError("rmsnorm: inconsistent shapes or dtypes")
    out = torch.empty_like(x)
    res_out = torch.empty_like(x) if residual is not None else None
    check(load().prism_moe_rmsnorm(ptr(x), ptr(residual), ptr(weight), float(eps),
                                   dtype_code(x.dtype), T, H, ptr(out), ptr(res_out),
                                   stream_of(x.device)), "prism_moe_rmsnorm")
    return out if residual is None else (out, res_out)


def block_forward(x, router_logits, w_gate_up, w_down, top_k: int, renorm: bool, out=None,
                  epilogue=None):
    """The single-GPU block after the router GEMM (prism_moe_block_forward): route, plan,
    gather, grouped SwiGLU experts, combine. ``x`` [T,H], ``router_logits`` [T,E],
    ``w_gate_up`` [E,2I,H], ``w_down`` [E,H,I]; returns [T,H]. ``epilogue`` (a NormEpilogue)
    fuses the decoder layer's next residual add + RMSNorm into the combine."""
    torch = _torch()
    _need_cuda(x, router_logits, w_gate_up, w_down)
    T, H = x.shape
    E, twoI, H2 = w_gate_up.shape
    I = twoI // 2
    if H2 != H or tuple(w_down.shape) != (E, H, I) or tuple(router_logits.shape) != (T, E):
        raise RuntimeError("block_forward: inconsistent shapes")
    for t in (router_logits, w_gate_up, w_down):
        if t.dtype != x.dtype:
            raise RuntimeError(f"block_forward: dtype {t.dtype} != hidden dtype {x.dtype}")
    if out is None:
        out = torch.empty_like(x)
    if T == 0:
        return out
    lib = load()
    dt = dtype_code(x.dtype)
    nbytes = lib.prism_moe_block_workspace_size(T, H, I, E, top_k, dt)
    ws = block_workspace(x.device, nbytes)
    check(lib.prism_moe_block_forward_norm(
        ptr(x), ptr(router_logits), dt, T, H, I, E, top_k, int(bool(renorm)), ptr(w_gate_up),
        ptr(w_down), ptr(out), None, None, ptr(ws), ws.numel(), stream_of(x.device),
        ctypes.byref(epilogue) if epilogue is not None else None),
        "prism_moe_block_forward")
    return out


def ep_alloc_landing(nbytes: int):
    """Allocate this rank's landing zone; returns (device address, IPC handle bytes)."""
    lib = load()
    buf = ctypes.create_string_buffer(lib.prism_moe_ep_ipc_handle_bytes())
    p = _vp()
    check(lib.prism_moe_ep_alloc_landing(nbytes, ctypes.byref(p), buf),
          "prism_moe_ep_alloc_landing")
    return p.value, buf.raw


def ep_open_peer(handle: bytes) -> int:
    """Map a peer's landing zone from its IPC handle; returns the device address."""
    lib = load()
    p = _vp()
    check(lib.prism_moe_ep_open_peer(ctypes.create_string_buffer(handle, len(handle)),
                                     ctypes.byref(p)), "prism_moe_ep_open_peer")
    return p.value


def set_profile_events(events) -> None:
    """Record ``events`` (torch.cuda.Event, already created) at the kernels' stage boundaries on
    this thread; ``None`` or an empty list turns the hook off."""
    events = list(events or [])
    arr = (_vp * max(len(events), 1))(*[ctypes.c_void_p(e.cuda_event) for e in events])
    check(load().prism_moe_profile_events(arr, len(events)), "prism_moe_profile_events")


def read_device_error(word, device=None) -> int:
    """Synchronise and return (and clear) the status in a device error word."""
    dev = word.device if device is None else device
    return load().prism_moe_read_device_error(ptr(word), stream_of(dev))


def set_expert_engine(name: str) -> None:
    """Expert GEMM engine for calls without an expert-parallel exchange: ``auto`` (default),
    ``fused``, ``single`` or ``pair`` (prism_moe_set_expert_engine)."""
    if name not in ENGINES:
        raise RuntimeError(f"unknown expert engine {name!r}; one of {sorted(ENGINES)}")
    check(load().prism_moe_set_expert_engine(ENGINES[name]), "prism_moe_set_expert_engine")


def set_wait_limits(wait_ns: int = 0, peer_wait_ns: int = 0) -> None:
    """Bounds of the kernels' waits on their own pipeline and on other ranks (0 = default)."""
    check(load().prism_moe_set_wait_limits(int(wait_ns), int(peer_wait_ns)),
          "prism_moe_set_wait_limits")


def ep_read_stats(workspace, device=None) -> dict:
    """Statistics of the last expert-parallel step that used ``workspace`` (synchronises)."""
    dev = workspace.device if device is None else device
    buf = (ctypes.c_uint64 * len(EP_STATS_FIELDS))()
    check(load().prism_moe_ep_read_stats(ptr(workspace), buf, stream_of(dev)),
          "prism_moe_ep_read_stats")
    return dict(zip(EP_STATS_FIELDS, (int(v) for v in buf)))
