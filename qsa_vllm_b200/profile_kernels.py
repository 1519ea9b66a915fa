"""Run one stage of the QSA path in a loop, for profilers (ncu) and quick timing.

    python -m qsa_vllm_b200.profile_kernels --kernel attention --config cfg2_32k \
        --batch 16 --iters 3 [--contiguous-tables] [--time]

``--kernel``: ``indexer`` | ``topk`` | ``select`` (the fused decode
indexer + top-k launch) | ``attention`` | ``step`` (selection and attention) |
``prepare`` (index-query norm/RoPE, key compression, cache writes) | ``layer``
(``prepare`` then ``step``, the reference layer's forward).
Inputs are the synthetic workload of ``--config`` with ``--batch`` rows (the
same per-row shapes as the benchmark, a smaller device footprint for ncu
captures).  ``--contiguous-tables`` replaces the random block tables with the
identity layout (each request's pages consecutive in memory), which isolates
the cost of scattered pages.  ``--time`` prints CUDA-event timings of graph
replays with the L2 flushed before every iteration (a 256 MiB write, then a
256 MiB read so no dirty write-back lands in the timed region).
"""

from __future__ import annotations

import argparse
import json

import torch

from .graph_dispatch import decode_logits_columns
from .indexer import (compute_visible_blocks, indexer_scores, select_decode_fused,
                      select_paged_tokens)
from .qsa import qsa_sparse_paged_attention
from .prepare import qsa_prepare
from .synthetic import make_prepare_inputs, make_workload
from .topk import topk_expand


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--kernel", default="attention",
                    choices=["indexer", "topk", "select", "attention", "step", "prepare",
                             "layer"])
    ap.add_argument("--config", default="cfg2_32k")
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--contiguous-tables", action="store_true")
    ap.add_argument("--shard", type=int, nargs=2, metavar=("TP", "RANK"), default=None,
                    help="one rank's head share under tensor parallelism TP (as the "
                         "multi-GPU benchmark shards): H_q/TP query heads, its KV head(s)")
    ap.add_argument("--time", action="store_true")
    ap.add_argument("--visible-kernel", action="store_true",
                    help="step: compute visible counts with qsa_visible_blocks first and "
                         "pass them in (instead of the kernels deriving them)")
    a = ap.parse_args()
    dev = torch.device("cuda")
    w = make_workload(a.config, device=dev, seed=0, batch=a.batch)
    if a.shard is not None:
        w = w.shard_heads(*a.shard)
    if a.contiguous_tables:
        for name in ("block_table", "index_table"):
            t = getattr(w, name)
            pages = (t >= 0).sum(1)
            start = torch.cumsum(pages, 0) - pages
            ident = start[:, None] + torch.arange(t.shape[1], device=dev)[None, :]
            setattr(w, name, torch.where(t >= 0, ident, t).to(torch.int32))
    rows = w.rows
    width = w.token_topk + w.ratio - 1
    r = w.ratio
    vis = torch.minimum((w.positions + 1) // r, w.seq_lens.long()[w.token_to_req.long()] // r)
    vis = vis.to(torch.int32)
    cols = w.index_table.shape[1] * w.index_cache.shape[1]
    logits = torch.zeros(rows, cols, device=dev)
    idx = torch.empty(rows, width, dtype=torch.int32, device=dev)
    cnt = torch.empty(rows, dtype=torch.int32, device=dev)
    out = torch.empty_like(w.q)

    # decode rows: one page-table row per request; prefill: packed rows
    prefill = (dict(decode_query_len=w.decode_query_len) if w.is_decode else
               dict(query_start_loc=w.query_start_loc, max_query_len=w.max_query_len))

    def run_indexer():
        indexer_scores(w.index_q, w.index_cache, w.index_table, vis, logits,
                       weights=w.index_weights, scale=w.index_scale, **prefill)

    def run_topk():
        topk_expand(logits, vis, w.positions, w.seq_lens, w.token_to_req, idx, r,
                    main_block_table=w.block_table, main_page_size=w.page_size,
                    valid_counts_out=cnt)

    def run_select():
        columns = decode_logits_columns(w.max_seq_len, r, cols)
        if not select_decode_fused(w.index_q, w.index_cache, w.index_table, vis, r,
                                   w.decode_query_len, idx, columns,
                                   query_positions=w.positions, sequence_lengths=w.seq_lens,
                                   token_to_req=w.token_to_req, main_block_table=w.block_table,
                                   main_page_size=w.page_size, valid_counts_out=cnt,
                                   weights=w.index_weights, scale=w.index_scale):
            raise SystemExit("the fused selection declined this workload")

    def run_attention():
        qsa_sparse_paged_attention(w.q, w.k_cache, w.v_cache, idx, w.block_table, w.token_to_req,
                                   out, output_gate=w.gate, use_decode_kernel=True,
                                   indices_are_physical=True, valid_counts=cnt)

    def run_step():
        # visible counts arrive with the step's metadata (as in the reference
        # layer), unless --visible-kernel recomputes them inside the step
        given = (compute_visible_blocks(w.positions, w.seq_lens, w.token_to_req, r)
                 if a.visible_kernel else vis)
        select_paged_tokens(
            w.index_q, w.index_cache, w.index_table, w.token_to_req, w.positions, w.seq_lens,
            w.token_topk, r, idx, **w.select_kwargs(),
            main_block_table=w.block_table, main_page_size=w.page_size, valid_counts_out=cnt,
            weights=w.index_weights, scale=w.index_scale, visible_blocks=given)
        run_attention()

    prep = make_prepare_inputs(w) if a.kernel in ("prepare", "layer") else None

    def run_prepare():
        qsa_prepare(**prep)

    def run_layer():
        run_prepare()
        run_step()

    run_indexer()
    run_topk()
    fn = {"indexer": run_indexer, "topk": run_topk, "select": run_select,
          "attention": run_attention,
          "step": run_step, "prepare": run_prepare, "layer": run_layer}[a.kernel]
    for _ in range(a.warmup):
        fn()
    torch.cuda.synchronize()
    if not a.time:
        for _ in range(a.iters):
            fn()
        torch.cuda.synchronize()
        return
    graph = torch.cuda.CUDAGraph()   # replay: no host launch gaps inside the events
    with torch.cuda.graph(graph):
        fn()
    graph.replay()
    flush_w = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    flush_r = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(a.iters)]
    for s, e in ev:
        flush_w.zero_()  # evict, then read clean lines so no dirty write-back is timed
        flush_r.sum()
        s.record()
        graph.replay()
        e.record()
    torch.cuda.synchronize()
    ms = [s.elapsed_time(e) for s, e in ev]
    print(json.dumps({"kernel": a.kernel, "config": a.config, "rows": rows, "shard": a.shard,
                      "contiguous_tables": a.contiguous_tables, "ms_min": min(ms),
                      "ms_median": sorted(ms)[len(ms) // 2]}))


if __name__ == "__main__":
    main()
