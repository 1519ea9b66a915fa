"""Build the reference top-k (``ops/csrc/topk.cu``) for sm_100a as a GPU-side checker.

TEST INFRASTRUCTURE ONLY.  The reference ships ``topk.cu`` built for sm_80
only (ops/topk.py:10-22), which cannot load on a B200.  This recipe compiles
the unmodified source where it lies under the reference tree with nvcc for
``compute_100a/sm_100a`` into ``oracle/_ref/libqsa_ref_topk.so`` (git-ignored,
carried to the GPU box with the working tree).  The op namespace is renamed on
the command line (``-Dyulan_qsa_kernels=yulan_qsa_ref_kernels``) so the
reference registers ``torch.ops.yulan_qsa_ref_kernels.topk_expand`` and can be
loaded beside this package's own ``torch.ops.yulan_qsa_kernels``.

    python oracle/build_ref.py [REFERENCE_ROOT]

REFERENCE_ROOT is the reference checkout (the directory holding
``yulan_qsa_vllm/``): the argument, else ``$QSA_REFERENCE_ROOT``, else a
checkout named ``reference`` beside this repository.  Nothing here runs unless
that tree is present (development container only); the GPU box uses the
prebuilt library.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref" / "libqsa_ref_topk.so"


def reference_root(explicit: str | None = None) -> Path:
    """The reference checkout: ``explicit``, else ``$QSA_REFERENCE_ROOT``, else
    the directory ``reference`` next to this repository's root."""
    if explicit:
        return Path(explicit)
    env = os.environ.get("QSA_REFERENCE_ROOT")
    if env:
        return Path(env)
    return HERE.parent.parent / "reference"


def build(ref_root: str | None = None, force: bool = False) -> Path | None:
    src = reference_root(ref_root) / "yulan_qsa_vllm" / "ops" / "csrc" / "topk.cu"
    if not src.exists():
        return OUT if OUT.exists() else None
    if OUT.exists() and not force and OUT.stat().st_mtime > src.stat().st_mtime:
        return OUT
    import torch
    from torch.utils import cpp_extension as ce

    OUT.parent.mkdir(parents=True, exist_ok=True)
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{p}" for p in ce.include_paths(device_type="cuda")]
    libdir = Path(torch.__file__).parent / "lib"
    cmd = [
        "nvcc", "-O3", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
        "-gencode", "arch=compute_100a,code=sm_100a",
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_API_INCLUDE_EXTENSION_H",
        "-Dyulan_qsa_kernels=yulan_qsa_ref_kernels",
        *incs, str(src), "-o", str(OUT),
        f"-L{libdir}", "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
        f"-Xlinker", f"-rpath={libdir}",
    ]
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(*sys.argv[1:2], force=True))
