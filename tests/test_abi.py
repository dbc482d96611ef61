"""The C-ABI library builds, loads and exports every symbol include/prism_moe.h declares
(no GPU needed: nothing here launches a kernel)."""
import ctypes
import re
from pathlib import Path

import pytest

from prism_infer_b200 import build, capi


def declared_functions():
    text = capi.HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(prism_moe_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return capi.load()


def test_header_declares_entry_points():
    names = declared_functions()
    for must in ("prism_moe_route_topk", "prism_moe_build_dispatch_plan",
                 "prism_moe_permute_rows", "prism_moe_expert_swiglu", "prism_moe_combine",
                 "prism_moe_block_forward"):
        assert must in names


def test_library_exports_every_declared_symbol(lib):
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in prism_moe.h but not exported"
        assert name in capi._SIGNATURES, f"{name} has no ctypes signature"


def test_library_exports_nothing_undeclared():
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(capi.LIB_PATH)],
                         capture_output=True, text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    ours = {s for s in exported if s.startswith("prism_moe_")}
    assert ours == set(declared_functions())


def test_host_side_queries(lib):
    assert lib.prism_moe_version() >= 100
    assert lib.prism_moe_block_workspace_size(64, 2048, 768, 128, 8, capi.BF16) > 64 * 8 * 2048 * 2
    assert lib.prism_moe_dispatch_workspace_size(8192, 8, 128, 8) > 0
    assert lib.prism_moe_block_workspace_size(-1, 2048, 768, 128, 8, capi.BF16) == 0


def test_argument_errors_need_no_gpu(lib):
    # argument checks run before any device call
    st = lib.prism_moe_route_topk(None, 7, 4, 8, 2, 1, None, None, None, None)
    assert st == capi.ERR_ARG and "dtype" in capi.last_error()
    st = lib.prism_moe_build_dispatch_plan(None, 4, 2, 7, 4, None, None, None, None, None, None,
                                           None, 0, None)
    assert st == capi.ERR_ARG and "divisible" in capi.last_error()


def test_controls_and_new_entry_points_check_arguments(lib):
    # process-wide controls (no device call)
    assert lib.prism_moe_set_expert_engine(7) == capi.ERR_ARG and "engine" in capi.last_error()
    assert lib.prism_moe_set_expert_engine(capi.ENGINES["auto"]) == capi.OK
    assert lib.prism_moe_set_wait_limits(-1, 0) == capi.ERR_ARG
    assert lib.prism_moe_set_wait_limits(61_000_000_000, 0) == capi.ERR_ARG
    assert lib.prism_moe_set_wait_limits(0, 0) == capi.OK
    # argument checks that run before any device call
    assert lib.prism_moe_rmsnorm(None, None, None, 1e-6, 9, 4, 64, None, None, None) == capi.ERR_ARG
    assert lib.prism_moe_rmsnorm(None, None, None, -1.0, capi.BF16, 4, 64, None, None,
                                 None) == capi.ERR_ARG
    assert lib.prism_moe_ep_read_stats(None, None, None) == capi.ERR_ARG
    epi = capi.NormEpilogue(0, 0, 1e-6, 0)     # incomplete: no residual / weight / output
    st = lib.prism_moe_block_forward_norm(None, None, capi.BF16, 0, 64, 32, 8, 2, 1, None, None,
                                          None, None, None, None, 1 << 20, None,
                                          ctypes.byref(epi))
    assert st == capi.ERR_ARG
    assert lib.prism_moe_ep_landing_bytes(65, 8, 2, 64, 8, capi.BF16) == 0    # > 64 ranks
    assert lib.prism_moe_ep_workspace_size(8, 64, 32, 9, 2, 2, capi.BF16) == 0   # E % W != 0


def test_c_host_builds_links_and_runs(lib, tmp_path):
    """The header compiles as C99 with every warning as an error, a C program links against the
    library, and the calls that need no GPU behave as from Python."""
    import shutil
    import subprocess
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    src = Path(__file__).resolve().parent / "c_host" / "abi_consumer.c"
    inc = Path(__file__).resolve().parent.parent / "include"
    libdir = capi.LIB_PATH.parent
    exe = tmp_path / "abi_consumer"
    subprocess.run([gcc, "-std=c99", "-Wall", "-Wextra", "-Werror", f"-I{inc}", str(src), "-o",
                    str(exe), f"-L{libdir}", "-lprism_moe", f"-Wl,-rpath,{libdir}"],
                   check=True, capture_output=True, text=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    lines = r.stdout.split("\n")
    assert sum(1 for ln in lines if ln.startswith("ok ")) >= 15, r.stdout
