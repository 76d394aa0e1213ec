"""Build the sm_100a kernel library in-tree: ``tree_attention/libtree_attn_b200.so``.

Plain ``nvcc -shared`` over ``csrc/*.cu`` and the host-only ``csrc/*.cpp`` (static CUDA runtime, so the library
is self-contained behind its C ABI; streams are passed in as cudaStream_t).
Run ``python build.py`` or call ``build()``; rebuilds only when a source or the
public header is newer than the library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = REPO / "include"
LIB = HERE / "tree_attention" / "libtree_attn_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda) / "bin" / "nvcc"
    if candidate.exists():
        return str(candidate)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME")
    return found


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _stale():
    if not LIB.exists():
        return True
    built = LIB.stat().st_mtime
    deps = list(sources()) + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > built for p in deps)


def build(force=False, verbose=False, extra_flags=()):
    """Compile every kernel for sm_100a and link the shared library."""
    if not force and not _stale():
        return LIB
    objdir = HERE / "_build"
    objdir.mkdir(exist_ok=True)
    nvcc = nvcc_path()
    common = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", str(INCLUDE),
                     "--expt-relaxed-constexpr", *extra_flags]
    objects = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        # host-only planner sources: no FMA contraction, costs must round like the Python statement
        host = ["-Xcompiler", "-ffp-contract=off"] if src.suffix == ".cpp" else []
        cmd = [nvcc, *common, *host, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *objects]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
