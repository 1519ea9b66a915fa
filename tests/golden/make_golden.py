"""Generate golden vectors from the reference Triton kernels (CPU interpreter).

Run in the development container, where the reference package is readable:

    python tests/golden/make_golden.py REFERENCE_ROOT   (or set QSA_REFERENCE_ROOT)

It copies the reference package ``yulan_qsa_vllm`` to a temporary directory
(importing it in place would JIT-compile ``ops/csrc/topk.cu`` into the source
tree), stubs the two modules whose imports need a GPU or vLLM 0.30 internals
(``graph_dispatch`` and ``ops.topk``; neither is used by the kernels run here),
sets ``TRITON_INTERPRET=1`` and launches, exactly as the reference launchers do:

* ``_qsa_mqa_paged_uniform_kernel``   (ops/indexer.py:24-114, launch :260-272)
* ``_prefill_logits`` -> ``_qsa_mqa_paged_prefill_kernel`` (ops/indexer.py:117-223, :282-302)
* ``_qsa_sparse_paged_gqa_splitk_kernel`` (ops/qsa.py:109-303, launch :657-678)
* ``expand_qsa_block_indices_cuda`` -> ``_expand_qsa_indices_kernel`` (ops/qsa.py:18-106, :552-591)

The interpreter mishandles bf16 tensors, so every "bf16" tensor is stored as
fp32 holding bf16-representable values.  Consequently the kernel's bf16 casts
(P before P.V, the output before the gate) are no-ops here; the oracle is
compared with ``round_p=False, round_out=False`` against these vectors.
The split-K merge kernel does not run in the interpreter (scalar-bool & vector
at ops/qsa.py:336), so multi-split cases record the per-split partial outputs
and LSE written by the split kernel itself.

Output: ``tests/golden/reference_triton.npz``.
"""

from __future__ import annotations

import os
import shutil
import sys
import tempfile
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent



def _reference_root(explicit: str | None) -> Path:
    """The reference checkout (holding ``yulan_qsa_vllm/``): the command-line
    argument, else ``$QSA_REFERENCE_ROOT``; one of them is required."""
    root = explicit or os.environ.get("QSA_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: pass the reference checkout as the first argument "
                         "or set QSA_REFERENCE_ROOT")
    return Path(root)

def _import_reference(ref_root: Path):
    tmp = Path(tempfile.mkdtemp(prefix="qsa_ref_"))
    shutil.copytree(ref_root / "yulan_qsa_vllm", tmp / "yulan_qsa_vllm")
    sys.path.insert(0, str(tmp))
    gd = types.ModuleType("yulan_qsa_vllm.graph_dispatch")
    gd.decode_logits_columns = lambda *a, **k: 0
    tk = types.ModuleType("yulan_qsa_vllm.ops.topk")
    tk.topk_expand = None
    sys.modules["yulan_qsa_vllm.graph_dispatch"] = gd
    sys.modules["yulan_qsa_vllm.ops.topk"] = tk
    from yulan_qsa_vllm.ops import indexer, qsa  # noqa: E402
    return indexer, qsa, tmp


def bf16ish(*shape, gen, scale=1.0):
    return (torch.randn(*shape, generator=gen) * scale).to(torch.bfloat16).float()


def bits16(x: torch.Tensor) -> np.ndarray:
    return x.to(torch.bfloat16).view(torch.int16).numpy()


def main(ref_root: str | None = None) -> None:
    ref_root = str(_reference_root(ref_root))
    indexer, qsa, tmp = _import_reference(Path(ref_root))
    gen = torch.Generator().manual_seed(1234)
    out: dict[str, np.ndarray] = {}

    # ---------------- A: uniform decode indexer ----------------
    for case, (requests, dql, heads, dim, page, width, nblk) in {
        "idx_dec1": (3, 1, 4, 64, 16, 6, 24),
        "idx_dec2": (2, 2, 8, 64, 16, 4, 12),
    }.items():
        rows = requests * dql
        q = bf16ish(rows, heads, dim, gen=gen)
        kc = bf16ish(nblk, page, 1, dim, gen=gen)
        table = torch.randperm(nblk, generator=gen)[: requests * width].view(requests, width)
        table = table.to(torch.int32).contiguous()
        visible = torch.randint(0, width * page + 1, (rows,), generator=gen).to(torch.int32)
        visible[0] = width * page
        logits = torch.full((rows, width * page), float("nan"))
        ppr = max(16, -(-128 // requests))
        indexer._qsa_mqa_paged_uniform_kernel[(requests, ppr)](
            q, kc, table, visible, logits,
            *q.stride()[:-1], *kc.stride()[:2], *table.stride()[:-1], *logits.stride()[:-1],
            PAGE_SIZE=page, PAGE_TABLE_WIDTH=width, NUM_HEADS=heads, HEAD_DIM=dim,
            DECODE_QUERY_LEN=dql, BLOCK_N=64, PROGRAMS_PER_REQUEST=ppr, STAGES=1,
            num_warps=4, num_stages=1,
        )
        out.update({f"{case}_q": bits16(q), f"{case}_kc": bits16(kc),
                    f"{case}_table": table.numpy(), f"{case}_visible": visible.numpy(),
                    f"{case}_dql": np.array(dql), f"{case}_logits": logits.numpy()})

    # ---------------- B: packed prefill indexer ----------------
    heads, dim, page, width, nblk = 4, 64, 16, 8, 20
    qsl = torch.tensor([0, 40, 70], dtype=torch.int32)
    rows = 70
    q = bf16ish(rows, heads, dim, gen=gen)
    kc = bf16ish(nblk, page, 1, dim, gen=gen)
    table = torch.randperm(nblk, generator=gen)[: 2 * width].view(2, width).to(torch.int32)
    visible = torch.randint(0, width * page + 1, (rows,), generator=gen).to(torch.int32)
    logits_width = 128
    for name, (qoff, nq) in {"full": (0, rows), "chunk": (32, 38)}.items():
        ws = torch.full((nq * logits_width,), float("nan"))
        lg = indexer._prefill_logits(q, kc, table, qsl, visible, ws, 40, logits_width,
                                     query_offset=qoff, num_queries=nq)
        out[f"idx_pre_{name}_logits"] = lg.numpy().copy()
        out[f"idx_pre_{name}_range"] = np.array([qoff, nq])
    out.update({"idx_pre_q": bits16(q), "idx_pre_kc": bits16(kc), "idx_pre_table": table.numpy(),
                "idx_pre_qsl": qsl.numpy(), "idx_pre_visible": visible.numpy(),
                "idx_pre_width": np.array(logits_width)})

    # ---------------- C/D: sparse paged attention ----------------
    def attention_case(case, rows, hq, hkv, d, page, nblk, token_topk, ratio, physical,
                       gate, splits, block_n, requests):
        kv = bf16ish(nblk, page, hkv, 2 * d, gen=gen)
        kc, vc = kv.split(d, dim=-1)
        q = bf16ish(rows, hq, d, gen=gen, scale=d ** -0.5)
        width = token_topk + ratio - 1
        t_width = (nblk // requests)
        table = torch.randperm(nblk, generator=gen)[: requests * t_width].view(requests, t_width)
        table = table.to(torch.int32).contiguous()
        table[0, -1] = -1                                     # an unmapped logical page
        token_to_req = torch.randint(0, requests, (rows,), generator=gen).to(torch.int32)
        token_to_req[-1] = -1                                 # padding row
        if physical:
            idx = torch.randint(-1, nblk * page, (rows, width), generator=gen).to(torch.int32)
            counts = torch.randint(0, width + 1, (rows,), generator=gen).to(torch.int32)
            counts[0] = width
        else:
            idx = torch.randint(-1, t_width * page + page, (rows, width), generator=gen)
            idx = idx.to(torch.int32)
            counts = None
        g = bf16ish(rows, hq, d, gen=gen) if gate else None
        group = hq // hkv
        block_m = max(16, 1 << (group - 1).bit_length())
        o = torch.zeros(rows, hq, d)
        if splits == 1:
            po, pl = o, o
        else:
            po = torch.zeros(splits, rows, hq, d)
            pl = torch.zeros(splits, rows, hq)
        gate_ptr = g if g is not None else o
        gate_strides = g.stride() if g is not None else (0, 0, 0)
        qsa._qsa_sparse_paged_gqa_splitk_kernel[(rows, hkv, splits)](
            q, kc, vc, idx, table, token_to_req, po, pl, o, gate_ptr,
            counts if counts is not None else idx,
            q.stride(0), q.stride(1), kc.stride(0), kc.stride(1), kc.stride(2),
            vc.stride(0), vc.stride(1), vc.stride(2), idx.stride(0), table.stride(0),
            o.stride(0), o.stride(1), *gate_strides, rows, nblk, requests,
            TOPK=width, PAGE_SIZE=page, PAGE_TABLE_WIDTH=t_width, GROUP_SIZE=group,
            HEAD_DIM=d, NUM_QUERY_HEADS=hq, NUM_SPLITS=splits,
            NUM_TILES=-(-width // block_n), BLOCK_M=block_m, BLOCK_N=block_n,
            HAS_OUTPUT_GATE=g is not None, INDICES_ARE_PHYSICAL=physical,
            HAS_VALID_COUNTS=counts is not None, num_warps=4, num_stages=1,
        )
        rec = {"kv": bits16(kv), "q": bits16(q), "idx": idx.numpy(), "table": table.numpy(),
               "t2r": token_to_req.numpy(),
               "cfg": np.array([rows, hq, hkv, d, page, nblk, int(physical), splits, block_n])}
        if counts is not None:
            rec["counts"] = counts.numpy()
        if g is not None:
            rec["gate"] = bits16(g)
        if splits == 1:
            rec["out"] = o.numpy()
        else:
            rec["part_o"] = po.numpy()
            rec["part_lse"] = pl.numpy()
        out.update({f"{case}_{k}": v for k, v in rec.items()})

    attention_case("att_dec", rows=5, hq=16, hkv=2, d=128, page=16, nblk=16, token_topk=64,
                   ratio=4, physical=True, gate=True, splits=1, block_n=32, requests=4)
    attention_case("att_dec_split", rows=4, hq=16, hkv=2, d=128, page=16, nblk=16,
                   token_topk=64, ratio=4, physical=True, gate=False, splits=2, block_n=32,
                   requests=4)
    attention_case("att_pre", rows=6, hq=16, hkv=2, d=128, page=16, nblk=16, token_topk=64,
                   ratio=4, physical=False, gate=False, splits=1, block_n=16, requests=2)
    attention_case("att_pre_split", rows=5, hq=8, hkv=2, d=64, page=16, nblk=16, token_topk=64,
                   ratio=4, physical=False, gate=True, splits=4, block_n=16, requests=2)

    # ---------------- E: expansion rules ----------------
    rows, ratio, token_topk, page, requests = 7, 4, 32, 16, 3
    block_topk = token_topk // ratio
    seq = torch.tensor([50, 13, 70], dtype=torch.int32)
    t2r = torch.tensor([0, 0, 1, 2, 2, -1, 1], dtype=torch.int32)
    pos = torch.tensor([49, 20, 12, 69, 33, 5, 2], dtype=torch.int64)
    blocks = torch.randint(-1, 18, (rows, block_topk), generator=gen).to(torch.int32)
    mtable = torch.randperm(40, generator=gen)[: requests * 5].view(requests, 5).to(torch.int32)
    mtable[1, 0] = -1
    for name, table in {"logical": None, "physical": mtable}.items():
        counts = torch.zeros(rows, dtype=torch.int32)
        res = qsa.expand_qsa_block_indices_cuda(
            blocks, pos, seq, t2r, ratio, token_topk, main_block_table=table,
            main_page_size=page, valid_counts_out=counts)
        out[f"exp_{name}_out"] = res.numpy()
        out[f"exp_{name}_counts"] = counts.numpy()
    out.update({"exp_blocks": blocks.numpy(), "exp_seq": seq.numpy(), "exp_t2r": t2r.numpy(),
                "exp_pos": pos.numpy(), "exp_table": mtable.numpy(),
                "exp_cfg": np.array([ratio, token_topk, page])})

    np.savez_compressed(HERE / "reference_triton.npz", **out)
    shutil.rmtree(tmp, ignore_errors=True)
    print("wrote", HERE / "reference_triton.npz", len(out), "arrays")


if __name__ == "__main__":
    main(*sys.argv[1:])
