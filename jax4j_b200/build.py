"""Builds libjax4j_b200.so (the engine's C-ABI library) for sm_100a with nvcc.

Usage: python -m jax4j_b200.build [--force] [--verbose]

Each .cu under csrc/ is compiled to an object in csrc/_build/, then linked into
jax4j_b200/libjax4j_b200.so next to this file, so the library travels with the source tree.
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(CSRC, "_build")
LIB = os.path.join(HERE, "libjax4j_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", INCLUDE, "-I", BUILD]
# Device headers that are also compiled at run time (NVRTC) are embedded as string literals:
# csrc/<name>.cuh -> _build/<name>.inc
EMBEDDED = ["aad_device.cuh"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the engine is built with the CUDA toolkit's nvcc")


def cuda_lib_dirs() -> list[str]:
    root = os.path.dirname(os.path.dirname(nvcc()))
    return [os.path.join(root, "lib64"), os.path.join(root, "lib64", "stubs")]


def sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def headers() -> list[str]:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool, extra: list[str]) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if _stale(obj, [src] + headers()):
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return obj


def _embed() -> None:
    for name in EMBEDDED:
        text = open(os.path.join(CSRC, name)).read()
        assert ')J4B"' not in text
        body = 'R"J4B(' + text + ')J4B"\n'
        target = os.path.join(BUILD, name.rsplit(".", 1)[0] + ".inc")
        if not os.path.exists(target) or open(target).read() != body:
            with open(target, "w") as f:
                f.write(body)


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    if force:
        for f in os.listdir(BUILD):
            os.remove(os.path.join(BUILD, f))
    _embed()
    srcs = sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, extra or []), srcs))
    if force or _stale(LIB, objs):
        libdirs = sum((["-L", d] for d in cuda_lib_dirs()), [])
        # libcuda is not linked: driver entry points are resolved at run time through the runtime,
        # so the library also loads (for planning and ABI checks) where no driver is installed
        rpath = ["-Xlinker", "-rpath=" + cuda_lib_dirs()[0]]
        # linked to a temporary name and renamed into place: a process that loads (or copies) the
        # library meanwhile sees the old file or the new one, never a partial one
        tmp = LIB + f".tmp{os.getpid()}"
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, *libdirs, *rpath, "-lcudart", "-lnvrtc"]
        try:
            subprocess.run(cmd, check=True)
            os.replace(tmp, LIB)
        finally:
            if os.path.exists(tmp):
                os.remove(tmp)
    return LIB


if __name__ == "__main__":
    p = argparse.ArgumentParser()
    p.add_argument("--force", action="store_true")
    p.add_argument("--verbose", action="store_true")
    args = p.parse_args()
    print(build(force=args.force, verbose=args.verbose))
    sys.exit(0)
