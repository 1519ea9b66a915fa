"""Time the reference's own GPU path beside this package's, on the same inputs.

TEST / MEASUREMENT INFRASTRUCTURE ONLY.  The reference's decode and prefill
GPU path is its Triton scoring kernels and split-K attention (reference
ops/indexer.py:24-223 launched by select_paged_tokens :346-393,
ops/qsa.py:109-362 launched by qsa_sparse_paged_attention :594-688) plus its
CUDA top-k (ops/csrc/topk.cu).  This script imports the reference package
from a temporary copy of REFERENCE_ROOT, with two modules replaced:

* ``graph_dispatch`` (needs vLLM 0.30 internals): ``decode_logits_columns``
  comes from this package, which implements the same column buckets;
* ``ops.topk`` (JIT-builds topk.cu for sm_80 only): its two wrappers call the
  unmodified topk.cu built for sm_100a by ``oracle/build_ref.py``
  (``torch.ops.yulan_qsa_ref_kernels``), with the reference wrapper's
  argument conventions.

For each configuration it runs one QSA layer step both ways on the same
seeded synthetic inputs (unit head weights, as the reference computes),
checks that they agree, and times them with CUDA events, eager and replayed
from a CUDA graph, with the L2 flushed before every timed step.  One JSON line
per configuration.

    python oracle/time_reference.py REFERENCE_ROOT [--configs cfg2_32k cfg3 cfg1]
"""

from __future__ import annotations

import argparse
import json
import shutil
import sys
import tempfile
import types
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
REF_TOPK = ROOT / "oracle" / "_ref" / "libqsa_ref_topk.so"


def import_reference(ref_root: Path):
    """The reference's ops.indexer and ops.qsa modules, from a temporary copy."""
    from qsa_vllm_b200.graph_dispatch import decode_logits_columns
    torch.ops.load_library(str(REF_TOPK))
    ref_ops = torch.ops.yulan_qsa_ref_kernels
    tmp = Path(tempfile.mkdtemp(prefix="qsa_ref_"))
    shutil.copytree(ref_root / "yulan_qsa_vllm", tmp / "yulan_qsa_vllm")
    sys.path.insert(0, str(tmp))
    gd = types.ModuleType("yulan_qsa_vllm.graph_dispatch")
    gd.decode_logits_columns = decode_logits_columns
    tk = types.ModuleType("yulan_qsa_vllm.ops.topk")

    def topk_expand(scores, lengths, query_positions, sequence_lengths, token_to_req, output,
                    compress_ratio, *, main_block_table=None, main_page_size=1,
                    valid_counts_out=None):
        ref_ops.topk_expand(
            scores, lengths, query_positions, sequence_lengths, token_to_req,
            main_block_table if main_block_table is not None else output,
            output, valid_counts_out if valid_counts_out is not None else output,
            compress_ratio, main_page_size, main_block_table is not None,
            valid_counts_out is not None)

    def topk(scores, lengths, output):
        ref_ops.topk(scores, lengths, output)

    tk.topk_expand, tk.topk = topk_expand, topk
    sys.modules["yulan_qsa_vllm.graph_dispatch"] = gd
    sys.modules["yulan_qsa_vllm.ops.topk"] = tk
    from yulan_qsa_vllm.ops import indexer, qsa  # noqa: E402
    return indexer, qsa, tmp


def step_fn(mods, w, out_idx, counts, out):
    """One layer step (selection, then attention) through the given modules'
    select_paged_tokens / qsa_sparse_paged_attention."""
    indexer, qsa = mods
    decode = w.is_decode
    rows = w.rows

    def step():
        indexer.select_paged_tokens(
            w.index_q, w.index_cache, w.index_table, w.token_to_req, w.positions, w.seq_lens,
            w.token_topk, w.ratio, out_idx, query_start_loc=w.query_start_loc,
            max_query_len=w.max_query_len, max_seq_len=w.max_seq_len,
            num_decodes=rows // w.decode_query_len if decode else 0,
            num_decode_tokens=rows if decode else 0, decode_query_len=w.decode_query_len,
            visible_blocks=w.visible_blocks,
            main_block_table=w.block_table if decode else None, main_page_size=w.page_size,
            valid_counts_out=counts if decode else None)
        qsa.qsa_sparse_paged_attention(
            w.q, w.k_cache, w.v_cache, out_idx, w.block_table, w.token_to_req, out,
            output_gate=w.gate, use_decode_kernel=decode, indices_are_physical=decode,
            valid_counts=counts if decode else None)
    return step


def time_ms(fn, steps, dev, flush):
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(steps)]
    for a, b in evs:
        flush()
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize(dev)
    ms = sorted(a.elapsed_time(b) for a, b in evs)
    return ms[len(ms) // 2]


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("reference_root")
    ap.add_argument("--configs", nargs="+", default=["cfg2_32k", "cfg3", "cfg1"])
    ap.add_argument("--steps", type=int, default=30)
    a = ap.parse_args()
    dev = torch.device("cuda")
    from qsa_vllm_b200 import indexer as our_indexer
    from qsa_vllm_b200 import qsa as our_qsa
    from qsa_vllm_b200.indexer import compute_visible_blocks
    from qsa_vllm_b200.synthetic import make_workload
    ref_indexer, ref_qsa, tmp = import_reference(Path(a.reference_root))
    flush_w = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    flush_r = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=dev)

    def flush():
        flush_w.zero_()
        flush_r.sum()

    for cfg in a.configs:
        w = make_workload(cfg, device=dev, seed=0, head_weights=False)
        w.visible_blocks = compute_visible_blocks(w.positions, w.seq_lens, w.token_to_req,
                                                  w.ratio)
        width = w.token_topk + w.ratio - 1
        res = {"config": cfg, "rows": w.rows}
        outs = {}
        for name, mods in (("reference", (ref_indexer, ref_qsa)),
                           ("b200", (our_indexer, our_qsa))):
            idx = torch.full((w.rows, width), -7, dtype=torch.int32, device=dev)
            cnt = torch.zeros(w.rows, dtype=torch.int32, device=dev)
            out = torch.zeros_like(w.q)
            fn = step_fn(mods, w, idx, cnt, out)
            fn()
            torch.cuda.synchronize(dev)
            outs[name] = (idx.clone(), cnt.clone(), out.float().clone())
            for _ in range(3):
                fn()
            res[f"{name}_eager_ms"] = time_ms(fn, a.steps, dev, flush)
            try:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    fn()
                g.replay()
                torch.cuda.synchronize(dev)
                res[f"{name}_graph_ms"] = time_ms(g.replay, a.steps, dev, flush)
                del g
            except Exception as e:  # the reference's host code may not capture
                res[f"{name}_graph_ms"] = None
                res[f"{name}_graph_error"] = str(e).splitlines()[0][:200]
        (ri, rc, ro), (bi, bc, bo) = outs["reference"], outs["b200"]
        res["selection_agreement"] = float((ri == bi).float().mean())
        res["counts_equal"] = bool(torch.equal(rc, bc))
        res["attention_max_abs_diff"] = float((ro - bo).abs().max())
        print(json.dumps(res), flush=True)
    shutil.rmtree(tmp, ignore_errors=True)


if __name__ == "__main__":
    main()
