"""Build recipe for the sm_100a C-ABI library ``llm_kernels/liblk_b200.so``.

Every ``csrc/*.cu`` file is compiled for ``sm_100a`` only (relocatable device code, so the
device status word is one symbol shared by all kernels), then device-linked and linked into
one shared library with the CUDA runtime linked statically.  The library needs no torch and
exports exactly the functions declared in ``include/llm_kernels_b200.h``.

Usage::

    python build.py            # incremental
    python build.py --force    # rebuild everything
    python build.py --verbose  # also print ptxas register / spill / smem usage
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
BUILD = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "llm_kernels", "liblk_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I" + CSRC,
    "-I" + INCLUDE,
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found: the sm_100a library cannot be built")
    return path


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return obj, (r.stderr if verbose else "")


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    headers = _headers()
    todo = [s for s in srcs if force or verbose or _stale(os.path.join(BUILD, os.path.basename(s)[:-3] + ".o"), [s, *headers])]
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(todo))) as ex:
            for obj, log in ex.map(lambda s: _compile(s, verbose), todo):
                logs.append(log)
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or todo or _stale(OUT, objs):
        cmd = [nvcc(), *ARCH, "-rdc=true", "-shared", "-Xcompiler", "-fPIC", "-o", OUT, *objs, "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        for log in logs:
            sys.stderr.write(log)
    return OUT


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
