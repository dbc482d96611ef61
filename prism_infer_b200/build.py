"""Build libprism_moe.so in-tree with nvcc for sm_100a.

    python -m prism_infer_b200.build [--force] [--verbose-ptxas]

Each ``csrc/*.cu`` compiles to an object under ``_build/`` (parallel ``nvcc -c``), then one
``nvcc -shared`` link writes ``prism_infer_b200/_lib/libprism_moe.so`` (cudart linked
statically). A stamp of the sources' and flags' hash skips rebuilding an up-to-date library.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
BUILD = REPO / "_build"
LIBDIR = PKG / "_lib"
LIB = LIBDIR / "libprism_moe.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden", f"-I{INCLUDE}", f"-I{CSRC}",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libprism_moe.so")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _digest(extra: list[str]) -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*")) + list(INCLUDE.glob("*.h"))):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    h.update(" ".join(NVCC_FLAGS + extra).encode())
    return h.hexdigest()


def build(force: bool = False, ptxas_verbose: bool = False, quiet: bool = True) -> Path:
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    stamp = LIBDIR / ".stamp"
    digest = _digest(extra)
    if not force and LIB.exists() and stamp.exists() and stamp.read_text() == digest:
        return LIB
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    exe = nvcc()
    # the library exports exactly the extern "C" symbols of include/prism_moe.h
    vis = ["-Xcompiler", "-fvisibility=default"]

    def compile_one(src: Path):
        obj = BUILD / (src.stem + ".o")
        cmd = [exe, *NVCC_FLAGS, *extra, *(vis if src.stem == "capi" else []), "-c", str(src),
               "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stderr}")
        return obj, r.stderr

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(compile_one, _sources()))
    if not quiet or ptxas_verbose:
        for _, err in results:
            if err.strip():
                print(err, file=sys.stderr)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [exe, *ARCH, "-shared", "-o", str(tmp), *[str(o) for o, _ in results],
           "-cudart", "static", "-Xlinker", "--no-undefined", "-lrt", "-ldl", "-lpthread"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIB)
    stamp.write_text(digest)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, ptxas_verbose=a.verbose_ptxas, quiet=False))


if __name__ == "__main__":
    main()
