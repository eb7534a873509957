"""Builds libastro_moe.so in-tree with nvcc for sm_100a (no GPU needed)."""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libastro_moe.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "-shared",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def needs_build() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    deps.append(os.path.join(ROOT, "include", "astro_moe.h"))
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles every .cu to an object in parallel, then links the shared library."""
    if not force and not needs_build():
        return LIB
    env = dict(os.environ)
    # nvcc's host compiler: the system gcc (an environment CC may point elsewhere)
    ccbin = ["-ccbin", "/usr/bin/g++"] if os.path.exists("/usr/bin/g++") else []
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    compile_flags = [f for f in NVCC_FLAGS if f != "-shared"]
    jobs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc(), *compile_flags, *ccbin, "-I", os.path.join(ROOT, "include"), "-c", "-o",
               obj, src]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        jobs.append((cmd, obj))
    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        results = list(ex.map(lambda j: subprocess.run(j[0], env=env, capture_output=True,
                                                       text=True), jobs))
    for (cmd, _), r in zip(jobs, results):
        if r.returncode != 0:
            sys.stderr.write(r.stdout + r.stderr)
            raise subprocess.CalledProcessError(r.returncode, cmd)
    tmp = LIB + ".tmp"
    link = [nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared", *ccbin, "-o", tmp,
            *[o for _, o in jobs]]
    if verbose:
        print(" ".join(link), file=sys.stderr)
    subprocess.run(link, check=True, env=env)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
