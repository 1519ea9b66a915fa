"""Build the sm_100a C-ABI library ``qsa_vllm_b200/libqsa_b200.so`` in-tree.

    python -m qsa_vllm_b200.build [--force] [--verbose]

Each ``csrc/*.cu`` translation unit is compiled by nvcc for
``compute_100a/sm_100a`` (cross-compiles on a host without a GPU) into
``_build/`` and linked into one shared library with a static CUDA runtime.
The library exports only the C functions of ``include/qsa_b200.h``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libqsa_b200.so"
SOURCES = ["capi.cu", "topk.cu", "indexer.cu", "indexer_tc.cu", "select_decode.cu", "attention.cu",
           "static_scratch.cu", "prepare.cu", "selftest.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler",
         "-fvisibility=hidden", "--expt-relaxed-constexpr", f"-I{ROOT / 'include'}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _needs_rebuild(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((ROOT / "include").glob("*.h"))
    objs = []
    jobs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if force or _needs_rebuild(o, [s, *headers]):
            cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(s), "-o", str(o)]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 1))) as ex:
        futs = [ex.submit(subprocess.run, j, capture_output=True, text=True) for j in jobs]
        for j, f in zip(jobs, futs):
            r = f.result()
            if verbose or ptxas_verbose or r.returncode:
                sys.stderr.write(" ".join(j) + "\n" + r.stdout + r.stderr)
            if r.returncode:
                raise RuntimeError(f"nvcc failed for {j[-3]}")
    if force or jobs or _needs_rebuild(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
            raise RuntimeError("link failed")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v resource usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas))
