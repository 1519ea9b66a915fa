"""Golden outputs of the reference's own GPU path (one QSA layer step) on a B200.

The reference's Triton scoring kernels and split-K attention (ops/indexer.py,
ops/qsa.py), compiled by Triton for sm_100, plus its CUDA top-k
(ops/csrc/topk.cu) built for sm_100a by ``oracle/build_ref.py``, run through
``oracle/time_reference.import_reference`` (the reference package imported
from a temporary copy of REFERENCE_ROOT, only ``graph_dispatch`` and the sm_80
top-k loader replaced).  Unlike the Triton-interpreter fixtures, these pin the
hardware results: bf16 rounding of P before P.V and of the gated output.

Run on the GPU box, after ``python oracle/build_ref.py REFERENCE_ROOT``:

    python tests/golden/make_reference_gpu_golden.py REFERENCE_ROOT [out.npz]

Inputs are the seeded synthetic workloads below, built on the CPU (so a test
rebuilds them bit for bit) with the reference's unit head weights; the fixture
stores only the selection, counts and bf16 outputs.  Output defaults to
``reference_gpu.npz`` in the current directory; the committed copy lives at
``tests/golden/reference_gpu.npz``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

# name -> (configuration, seed, overrides): small versions of the benchmark shapes
CASES = {
    "decode": ("cfg2_32k", 11, dict(batch=4, seq_len=4096)),
    "decode_mixed": ("cfg2", 13, dict(batch=3, seq_len=(3000, 6000))),
    "prefill": ("cfg1", 12, dict(batch=1, seq_len=2048, new_tokens=12)),
}


def build(name: str, device):
    from qsa_vllm_b200.indexer import compute_visible_blocks
    from qsa_vllm_b200.synthetic import make_workload
    cfg, seed, ov = CASES[name]
    w = make_workload(cfg, device="cpu", seed=seed, head_weights=False, **ov)
    for f in ("positions", "seq_lens", "token_to_req", "query_start_loc", "q", "gate", "kv",
              "block_table", "index_q", "index_cache", "index_table"):
        v = getattr(w, f, None)
        if isinstance(v, torch.Tensor):
            setattr(w, f, v.to(device))
    w.visible_blocks = compute_visible_blocks(w.positions, w.seq_lens, w.token_to_req, w.ratio)
    return w


def main(reference_root: str, out_path: str | None = None) -> None:
    from oracle.time_reference import import_reference, step_fn
    dev = torch.device("cuda")
    indexer, qsa, _ = import_reference(Path(reference_root))
    out: dict[str, np.ndarray] = {}
    for name in CASES:
        w = build(name, dev)
        width = w.token_topk + w.ratio - 1
        idx = torch.full((w.rows, width), -7, dtype=torch.int32, device=dev)
        cnt = torch.zeros(w.rows, dtype=torch.int32, device=dev)
        o = torch.zeros_like(w.q)
        step_fn((indexer, qsa), w, idx, cnt, o)()
        torch.cuda.synchronize()
        out[f"{name}_indices"] = idx.cpu().numpy()
        out[f"{name}_counts"] = cnt.cpu().numpy()
        out[f"{name}_out_bits"] = o.cpu().view(torch.int16).numpy()
        print(name, w.rows, "rows", flush=True)
    np.savez_compressed(out_path or "reference_gpu.npz", **out)


if __name__ == "__main__":
    main(*sys.argv[1:])
