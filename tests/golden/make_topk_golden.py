"""Golden vectors from the reference top-k (ops/csrc/topk.cu) run on a B200.

Run on the GPU box after ``python oracle/build_ref.py`` built
``oracle/_ref/libqsa_ref_topk.so`` (the unmodified reference source compiled
for sm_100a, op namespace renamed to ``yulan_qsa_ref_kernels``):

    python tests/golden/make_topk_golden.py [out.npz]

For every case of ``tests/topk_cases.standard_cases()`` it calls
``torch.ops.yulan_qsa_ref_kernels.topk_expand`` exactly as the reference
wrapper does (ops/topk.py:29-39: dummy tensors for unused table / counts) and
stores inputs and outputs.  Output defaults to ``reference_topk.npz`` in the
current directory; the committed copy lives at ``tests/golden/reference_topk.npz``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "tests"))

from topk_cases import aligned_rows, standard_cases  # noqa: E402


def main(out_path: str | None = None) -> None:
    lib = ROOT / "oracle" / "_ref" / "libqsa_ref_topk.so"
    torch.ops.load_library(str(lib))
    op = torch.ops.yulan_qsa_ref_kernels.topk_expand
    out: dict[str, np.ndarray] = {}
    dev = torch.device("cuda")
    for name, c in standard_cases().items():
        g = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
        g["scores"] = aligned_rows(g["scores"])   # the reference needs 16-byte aligned rows
        rows = c["scores"].shape[0]
        output = torch.full((rows, c["output_width"]), -7, dtype=torch.int32, device=dev)
        counts = torch.full((rows,), -7, dtype=torch.int32, device=dev)
        op(g["scores"], g["lengths"], g["positions"], g["seq_lens"], g["token_to_req"],
           g["table"] if c["physical"] else output, output,
           counts if c["store_counts"] else output,
           c["ratio"], c["page_size"], c["physical"], c["store_counts"])
        torch.cuda.synchronize()
        for k in ("scores", "lengths", "positions", "seq_lens", "token_to_req", "table"):
            out[f"{name}__{k}"] = c[k].numpy()
        out[f"{name}__cfg"] = np.array([c["ratio"], c["page_size"], int(c["physical"]),
                                        int(c["store_counts"])])
        out[f"{name}__output"] = output.cpu().numpy()
        out[f"{name}__counts"] = counts.cpu().numpy()
    path = Path(out_path) if out_path else Path("reference_topk.npz")
    path.parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(path, **out)
    print("wrote", path, len(out), "arrays")


if __name__ == "__main__":
    main(*sys.argv[1:2])
