"""Host-side tests that need no GPU: the C-ABI library, graph buckets, sharding,
and the indexer/top-k chunking logic (kernels replaced by the CPU oracle)."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import qsa_oracle as O

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "qsa_b200.h"


def header_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"QSA_API\s+[\w\s\*]+?\b(qsa_\w+)\s*\(", text)


def test_header_declares_the_three_stages():
    names = header_functions()
    for n in ("qsa_indexer_scores", "qsa_topk_expand", "qsa_topk", "qsa_sparse_attention",
              "qsa_sparse_attention_workspace_bytes", "qsa_last_error", "qsa_status_string"):
        assert n in names


def test_library_loads_and_exports_every_header_symbol():
    from qsa_vllm_b200 import _lib
    lib = _lib.load_library()
    for name in header_functions():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
    raw = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in header_functions():
        getattr(raw, name)


def test_host_only_entry_points():
    from qsa_vllm_b200 import _lib
    lib = _lib.load_library()
    assert b"sm_100a" in lib.qsa_version()
    assert lib.qsa_status_string(0) == b"ok"
    assert lib.qsa_status_string(3) == b"workspace too small"
    # rows == 0 is a no-op that never touches the device
    assert lib.qsa_topk_expand(None, 0, 0, 0, None, None, None, 0, None, None, 0, 0, None, 0, 1,
                               7, None, 4, 16, 1, None) == 0
    assert lib.qsa_sparse_attention(None, 0, 0, 0, 32, 128, None, 0, 0, 0, None, 0, 0, 0, 0, 16,
                                    4, None, 0, 0, None, 0, 0, 0, None, None, None, 0, 0, 0, None,
                                    0, 0, 1, 1, None, 0, None) == 0


def test_argument_errors_are_reported_not_launched():
    from qsa_vllm_b200 import _lib
    lib = _lib.load_library()
    st = lib.qsa_topk_expand(None, 0, 1, 8, None, None, None, 0, None, None, 0, 0, None, 0, 1,
                             7, None, 0, 16, 1, None)
    assert st == 1 and b"ratio" in lib.qsa_last_error()
    st = lib.qsa_indexer_scores(1024, 64, 64, 4, 96, 1024, 0, 0, 1, 16, 1024, 0, 1, 1, 1024,
                                None, None, 0, None, 0,
                                None, 1, 1, 0, 1, None, 0, 0, 1.0, 1024, 0, 8, None)
    assert st == 2 and b"head_dim" in lib.qsa_last_error()
    # no visible counts and nothing to derive them from
    st = lib.qsa_indexer_scores(1024, 64, 64, 4, 64, 1024, 0, 0, 1, 16, 1024, 0, 1, 1, None,
                                None, None, 0, None, 0,
                                None, 1, 1, 0, 1, None, 0, 0, 1.0, 1024, 0, 8, None)
    assert st == 1 and b"positions" in lib.qsa_last_error()
    st = lib.qsa_sparse_attention(1024, 0, 0, 1, 48, 128, 1024, 0, 0, 0, 1024, 0, 0, 0, 1, 16,
                                  2, 1024, 0, 8, None, 0, 0, 0, None, None, None, 0, 0, 0, 1024,
                                  0, 0, 1, 1, None, 0, None)
    assert st == 2 and b"group" in lib.qsa_last_error()
    # non-positive head counts are refused before any launch (0 and -8 are
    # multiples of 8 / of the KV heads, so they need their own check)
    for heads in (0, -8):
        st = lib.qsa_indexer_scores(1024, 64, 64, heads, 64, 1024, 0, 0, 1, 16, 1024, 0, 1, 1,
                                    1024, None, None, 0, None, 0,
                                    None, 1, 1, 0, 1, None, 0, 0, 1.0, 1024, 0, 8, None)
        assert st == 2 and b"heads" in lib.qsa_last_error(), heads
        st = lib.qsa_sparse_attention(1024, 0, 0, 1, heads, 128, 1024, 0, 0, 0, 1024, 0, 0, 0,
                                      1, 16, 2, 1024, 0, 8, None, 0, 0, 0, None, None, None, 0,
                                      0, 0, 1024, 0, 0, 1, 1, None, 0, None)
        assert st == 1 and b"query heads" in lib.qsa_last_error(), heads
        assert lib.qsa_sparse_attention_workspace_bytes(64, heads, 4, 128, 2051, 1) == 0
    assert lib.qsa_sparse_attention_workspace_bytes(64, 30, 4, 128, 2051, 1) == 0
    assert lib.qsa_sparse_attention_workspace_bytes(64, 32, 4, 128, -1, 1) == 0
    # a top-k beyond what one row's selection holds in shared memory (49152
    # blocks) is refused with its own message, not a launch error
    st = lib.qsa_topk(1024, 4096, 1, 4096, 1024, 1024, 49153, 49153, None)
    assert st == 2 and b"top-k" in lib.qsa_last_error()
    with pytest.raises(_lib.QSAError):
        _lib.check(1, "probe")


def _prepare_args(**over):
    """qsa_prepare's 58 C arguments (null pointers, unit strides), by name."""
    names = ("index_qk index_row_stride num_tokens num_index_heads index_head_dim positions "
             "positions_stride q_norm_weight k_norm_weight cos_sin_cache cos_sin_rows rotary_dim "
             "eps index_q_out state_cache state_block_stride state_token_stride state_blocks "
             "state_size state_slots state_table state_table_stride query_start_loc num_requests "
             "logical_positions compressed_cache compressed_block_stride compressed_token_stride "
             "compressed_blocks compressed_page_size compressed_slots k_work num_k_work "
             "compress_ratio main_key mk0 mk1 mk2 main_value mv0 mv1 mv2 main_key_cache kc0 kc1 "
             "kc2 kc3 main_value_cache vc0 vc1 vc2 vc3 main_blocks main_page_size main_slots "
             "num_main_kv_heads main_head_dim stream").split()
    assert len(names) == 58
    vals = dict.fromkeys(names, None)
    vals.update(index_row_stride=576, num_tokens=4, num_index_heads=8, index_head_dim=64,
                positions_stride=1, cos_sin_rows=4096, rotary_dim=64, eps=1e-6,
                state_block_stride=8192, state_token_stride=64, state_blocks=4, state_size=128,
                state_table_stride=1, num_requests=1, compressed_block_stride=4096,
                compressed_token_stride=64, compressed_blocks=4, compressed_page_size=64,
                num_k_work=1, compress_ratio=4, mk0=512, mk1=128, mk2=1, mv0=512, mv1=128,
                mv2=1, kc0=32768, kc1=512, kc2=128, kc3=1, vc0=32768, vc1=512, vc2=128, vc3=1,
                main_blocks=4, main_page_size=64, num_main_kv_heads=4, main_head_dim=128)
    vals.update(over)
    return [vals[n] for n in names]


def test_prepare_argument_errors_are_reported_not_launched():
    from qsa_vllm_b200 import _lib
    lib = _lib.load_library()
    # nothing to do: no device access
    assert lib.qsa_prepare(*_prepare_args(num_tokens=0, num_k_work=0)) == 0
    assert lib.qsa_prepare(*_prepare_args(index_head_dim=96)) == 2
    assert b"index head dim" in lib.qsa_last_error()
    assert lib.qsa_prepare(*_prepare_args(rotary_dim=33)) == 1
    assert b"rotary" in lib.qsa_last_error()
    assert lib.qsa_prepare(*_prepare_args(compress_ratio=0)) == 1
    # a real launch needs the projection, weights and caches
    assert lib.qsa_prepare(*_prepare_args()) == 1
    assert b"null" in lib.qsa_last_error()


def test_prepare_fails_loudly_without_a_gpu():
    from types import SimpleNamespace

    from qsa_vllm_b200 import _lib
    from qsa_vllm_b200.prepare import qsa_prepare
    bf = torch.bfloat16
    i64 = torch.zeros(4, dtype=torch.int64)
    raw = SimpleNamespace(slot_mapping=i64, block_table=torch.zeros(1, 1, dtype=torch.int32),
                          query_start_loc=torch.tensor([0, 4], dtype=torch.int32),
                          logical_positions=i64)
    comp = SimpleNamespace(slot_mapping=i64, k_work_metadata=torch.zeros(1, 2, dtype=torch.int32))
    with pytest.raises(_lib.QSAError):
        qsa_prepare(torch.zeros(4, 576, dtype=bf), i64, torch.ones(64, dtype=bf),
                    torch.ones(64, dtype=bf), torch.zeros(16, 64, dtype=bf), 1e-6, raw, comp,
                    torch.zeros(2, 8, 64, dtype=bf), torch.zeros(2, 16, 64, dtype=bf),
                    torch.zeros(4, 2, 128, dtype=bf), torch.zeros(4, 2, 128, dtype=bf),
                    torch.zeros(2, 16, 2, 128, dtype=bf), torch.zeros(2, 16, 2, 128, dtype=bf),
                    i64, num_index_heads=8, index_head_dim=64, rotary_dim=64, compress_ratio=4)


def test_attention_workspace_query_is_deterministic():
    from qsa_vllm_b200.qsa import attention_workspace_bytes
    a = attention_workspace_bytes(64, 32, 4, 128, 2051, True)
    assert a == attention_workspace_bytes(64, 32, 4, 128, 2051, True)
    # pairs cut by CTA range boundaries leave per-warp partials for the merge
    assert attention_workspace_bytes(8192, 16, 2, 128, 1027, False) > 0


def test_attention_workspace_is_bounded_by_the_cta_count():
    """Two slot groups per CTA of one partial per consumer warp (8) for the
    GQA group, whatever the rows (148 SMs assumed without a device); 0 when
    no pair is cut (one CTA per unit and every pair on one CTA)."""
    from qsa_vllm_b200.qsa import attention_workspace_bytes
    for hq, hkv, d in ((32, 4, 128), (16, 2, 128), (32, 2, 128), (16, 1, 64), (8, 8, 128)):
        bound = 256 + 2 * 148 * 8 * (hq // hkv) * (d + 1) * 4
        for rows in (1, 3, 64, 1000, 8192, 1 << 20):
            for width in (1, 515, 2051, 65539):
                need = attention_workspace_bytes(rows, hq, hkv, d, width, True)
                assert 0 <= need <= bound, (hq, hkv, d, rows, width, need)
    # 4 rows x 1 pair x 1 tile: 4 units on 4 CTAs, no pair cut
    assert attention_workspace_bytes(4, 32, 4, 128, 16, True) == 0


def test_attention_query_rows_are_realigned_by_copy():
    """A contiguous query view that starts 2 bytes past a 16-byte boundary is
    copied (``.contiguous()`` would hand the same misaligned view back); an
    aligned one, or one with aligned strides inside a wider row, is kept."""
    from qsa_vllm_b200.qsa import aligned_head_rows
    rows, hq, d = 3, 4, 128
    base = torch.arange(1 + rows * hq * d, dtype=torch.float32).to(torch.bfloat16)
    q = base[1:].view(rows, hq, d)
    assert q.is_contiguous() and q.data_ptr() % 16 == 2
    fixed = aligned_head_rows(q)
    assert fixed.data_ptr() != q.data_ptr() and fixed.data_ptr() % 16 == 0
    assert torch.equal(fixed, q)
    aligned = torch.zeros(rows, hq, d, dtype=torch.bfloat16)
    assert aligned_head_rows(aligned) is aligned
    wide = torch.zeros(rows, hq + 2, d, dtype=torch.bfloat16)[:, 1:hq + 1]
    assert aligned_head_rows(wide) is wide
    odd_stride = torch.zeros(rows, hq * d + 4, dtype=torch.bfloat16)[:, :hq * d].view(rows, hq, d)
    assert aligned_head_rows(odd_stride).stride(0) == hq * d


def test_operators_fail_loudly_without_a_gpu():
    from qsa_vllm_b200 import _lib
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    q = torch.zeros(2, 8, 128, dtype=torch.bfloat16)
    kv = torch.zeros(4, 16, 1, 256, dtype=torch.bfloat16)
    with pytest.raises(_lib.QSAError):
        qsa_sparse_paged_attention(q, kv[..., :128], kv[..., 128:],
                                   torch.zeros(2, 7, dtype=torch.int32),
                                   torch.zeros(1, 1, dtype=torch.int32),
                                   torch.zeros(2, dtype=torch.int32), indices_are_physical=True)


# ------------------------------------------------------------ graph buckets
def test_decode_column_buckets():
    from qsa_vllm_b200 import graph_dispatch as gd
    assert gd.decode_column_bucket(131072) == 32768
    assert gd.decode_column_bucket(131073 + 3) == 0
    assert gd.decode_logits_columns(4096, 4, 8192) == 8192        # bucket clipped to capacity
    assert gd.decode_logits_columns(524288, 4, 131072) == 131072  # full capacity
    with gd.capture_column_scope(0):
        assert gd.decode_logits_columns(10, 4, 5000) == 5000
    with gd.capture_column_scope(32768):
        assert gd.decode_logits_columns(10 ** 7, 4, 40000) == 32768
    assert gd.decode_logits_columns(4096, 4, 40000) == 32768


def test_graph_dispatch_patch_with_fake_vllm():
    from dataclasses import dataclass
    from types import SimpleNamespace

    from qsa_vllm_b200 import graph_dispatch as gd

    FULL, PIECE = "FULL", "PIECEWISE"

    @dataclass(frozen=True)
    class Desc:
        cg_mode: str
        num_tokens: int

    class GraphManager:
        def capture(self, create_forward_fn, progress_bar_desc=""):
            return [create_forward_fn(d, False)("run") for d in self._capture_descs[FULL]]

    class ModelGraphManager(GraphManager):
        def _init_candidates(self):
            self._capture_descs = {FULL: [Desc(FULL, 8)], PIECE: [Desc(PIECE, 8)]}

        def dispatch(self, n):
            return Desc(FULL, n)

    class Runner:
        def gather_batch_req_state(self, scheduler_output, dummy_run):
            return scheduler_output, True

    gd.install_short_decode_dispatch(ModelGraphManager, GraphManager, Runner, FULL, Desc)
    m = ModelGraphManager()
    m._init_candidates()
    cols = sorted(d.logits_columns for d in m._capture_descs[FULL])
    assert cols == [0, 32768]
    seen = m.capture(lambda desc, warm: (lambda mode: gd.decode_logits_columns(10, 4, 50000)))
    assert sorted(seen) == [32768, 50000]
    runner = Runner()
    runner.req_states = SimpleNamespace(num_computed_tokens_np=np.array([100, 600000]))
    batch = SimpleNamespace(idx_mapping_np=np.array([0]), num_scheduled_tokens=np.array([1]))
    runner.gather_batch_req_state(batch, False)
    assert gd.runtime_columns() == 32768 and m.dispatch(8).logits_columns == 32768
    batch.idx_mapping_np = np.array([1])
    runner.gather_batch_req_state(batch, False)
    assert gd.runtime_columns() == 0 and m.dispatch(8).logits_columns == 0


# ----------------------------------------------------------------- sharding
def test_head_shard_rule():
    from qsa_vllm_b200.sharding import head_shard
    assert head_shard(32, 4, 1, 0) == (slice(0, 32), slice(0, 4))
    assert head_shard(32, 4, 2, 1) == (slice(16, 32), slice(2, 4))
    assert head_shard(32, 4, 4, 3) == (slice(24, 32), slice(3, 4))
    # tp > kv heads: KV heads replicated, each rank keeps the one its queries use
    assert [head_shard(32, 4, 8, r)[1] for r in range(8)] == [slice(r // 2, r // 2 + 1)
                                                            for r in range(8)]
    with pytest.raises(ValueError):
        head_shard(32, 4, 3, 0)


def _sharded_worker(rank, world, port, result_path):
    import torch.distributed as dist
    from qsa_vllm_b200.sharding import head_shard
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        g = torch.Generator().manual_seed(0)
        rows, hq, hkv, d, page, nblk = 4, 16, 2, 64, 16, 12
        kv = torch.randn(nblk, page, hkv, 2 * d, generator=g).to(torch.bfloat16)
        q = (torch.randn(rows, hq, d, generator=g) * 0.2).to(torch.bfloat16)
        idx = torch.randint(-1, nblk * page, (rows, 35), generator=g).to(torch.int32)
        t2r = torch.zeros(rows, dtype=torch.int32)
        table = torch.zeros(1, 1, dtype=torch.int32)
        qs, ks = head_shard(hq, hkv, world, rank)
        part = O.sparse_attention(q[:, qs], kv[:, :, ks, :d], kv[:, :, ks, d:], idx, table, t2r,
                                  indices_are_physical=True, use_decode_kernel=True,
                                  block_n=32, num_splits=1)
        parts = [torch.empty_like(part) for _ in range(world)]
        dist.all_gather(parts, part)       # test-only: reassemble the head shards
        if rank == 0:
            full = O.sparse_attention(q, kv[..., :d], kv[..., d:], idx, table, t2r,
                                      indices_are_physical=True, use_decode_kernel=True,
                                      block_n=32, num_splits=1)
            ok = torch.equal(torch.cat(parts, dim=1), full)
            Path(result_path).write_text("ok" if ok else "mismatch")
    finally:
        dist.destroy_process_group()


def test_head_sharded_attention_two_gloo_ranks(tmp_path):
    """Each rank computes only its heads (no collective in the path); the
    concatenated shards equal the unsharded result exactly."""
    import socket

    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    res = tmp_path / "res.txt"
    mp.start_processes(_sharded_worker, args=(2, port, str(res)), nprocs=2, join=True,
                       start_method="spawn")
    assert res.read_text() == "ok"


# -------------------------------------------------- indexer host chunking
@pytest.mark.parametrize("given_visible", [False, True])
def test_select_paged_tokens_chunking_with_oracle_kernels(monkeypatch, given_visible):
    """The host loop (workspace chunks, decode/prefill split, visible blocks
    given or derived in the kernels) driven with the oracle standing in for the
    two kernels must reproduce the oracle's one-shot result."""
    import qsa_vllm_b200.indexer as I

    def fake_scores(q, k_cache, page_table, visible, logits, *, decode_query_len=1,
                    query_start_loc=None, max_query_len=0, query_offset=0, num_rows=None,
                    weights=None, scale=None, query_positions=None, sequence_lengths=None,
                    token_to_req=None, compress_ratio=0):
        rows = q.shape[0] if num_rows is None else num_rows
        if visible is None:   # what the kernel derives (same row indexing as q)
            visible = O.visible_blocks(query_positions, sequence_lengths, token_to_req,
                                       compress_ratio)
        if query_start_loc is None:
            res = O.indexer_scores(q, k_cache, page_table, visible, logits.shape[1],
                                   decode_query_len=decode_query_len, weights=weights,
                                   scale=scale)
            logits.copy_(torch.nan_to_num(res, nan=0.0))
        else:
            res = O.indexer_scores(q, k_cache, page_table, visible, logits.shape[1],
                                   query_start_loc=query_start_loc, weights=weights, scale=scale)
            logits.copy_(torch.nan_to_num(res[query_offset:query_offset + rows], nan=0.0))

    def fake_topk(scores, lengths, positions, seq_lens, t2r, output, ratio, *,
                  main_block_table=None, main_page_size=1, valid_counts_out=None):
        out, counts = O.topk_expand(scores, lengths, positions, seq_lens, t2r, main_block_table,
                                    output.shape[1], ratio, page_size=main_page_size)
        output.copy_(torch.from_numpy(out))
        if valid_counts_out is not None:
            valid_counts_out.copy_(torch.from_numpy(counts))

    def fake_topk_visible(scores, positions, seq_lens, t2r, output, ratio, **kw):
        fake_topk(scores, O.visible_blocks(positions, seq_lens, t2r, ratio), positions,
                  seq_lens, t2r, output, ratio, **kw)

    monkeypatch.setattr(I, "indexer_scores", fake_scores)
    monkeypatch.setattr(I, "_topk_expand", fake_topk)
    monkeypatch.setattr(I, "_topk_expand_visible", fake_topk_visible)
    monkeypatch.setattr(I, "compute_visible_blocks",
                        lambda pos, seq, t2r, ratio: O.visible_blocks(pos, seq, t2r, ratio))
    monkeypatch.setattr(I, "_INDEXER_WORKSPACE_BYTES", 3 * 64 * 4)   # force many chunks
    g = torch.Generator().manual_seed(0)
    ratio, page, topk = 4, 16, 32
    seq = torch.tensor([300, 180, 260], dtype=torch.int32)
    # 2 decode requests then one prefill request of 5 tokens
    t2r = torch.tensor([0, 1, 2, 2, 2, 2, 2], dtype=torch.int32)
    pos = torch.tensor([299, 179, 255, 256, 257, 258, 259], dtype=torch.int64)
    qsl = torch.tensor([0, 1, 2, 7], dtype=torch.int32)
    nblk = 30
    kc = torch.randn(nblk, page, 1, 64, generator=g).to(torch.bfloat16)
    table = torch.randperm(nblk, generator=g)[:15].view(3, 5).to(torch.int32)
    q = torch.randn(7, 4, 64, generator=g).to(torch.bfloat16)
    out = torch.empty(7, topk + ratio - 1, dtype=torch.int32)
    vis = O.visible_blocks(pos, seq, t2r, ratio)
    I.select_paged_tokens(q, kc, table, t2r, pos, seq, topk, ratio, out, query_start_loc=qsl,
                          max_query_len=5, max_seq_len=300, num_decodes=2, num_decode_tokens=2,
                          visible_blocks=vis.clone() if given_visible else None)
    logits = torch.zeros(7, 80)
    for r in range(7):
        req = int(t2r[r])
        logits[r] = torch.nan_to_num(O.indexer_scores(q[r:r + 1], kc, table[req:req + 1],
                                                      vis[r:r + 1], 80), nan=0.0)[0]
    ref, _ = O.topk_expand(logits, vis, pos, seq, t2r, None, topk + ratio - 1, ratio)
    assert np.array_equal(out.numpy(), ref)


# ------------------------------------------------------- synthetic workloads
def test_select_kwargs_decode_mtp_and_prefill():
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg2_32k_mtp2", device="cpu", batch=3, seq_len=1024)
    k = w.select_kwargs()
    assert w.rows == 6 and k["num_decodes"] == 3 and k["num_decode_tokens"] == 6
    assert k["decode_query_len"] == 2 and k["max_query_len"] == 2
    assert w.positions.tolist() == [1022, 1023] * 3
    p = make_workload("cfg1", device="cpu", batch=2, seq_len=512, new_tokens=64)
    kp = p.select_kwargs()
    assert "num_decodes" not in kp and kp["max_query_len"] == 64


def test_prepare_inputs_metadata_follow_the_workload():
    from qsa_vllm_b200.synthetic import make_prepare_inputs, make_workload
    w = make_workload("cfg2", device="cpu", seed=8, batch=8)
    a = make_prepare_inputs(w, state_size=64)
    pos = w.positions
    r, page = w.ratio, w.page_size
    comp = a["compressed_metadata"].slot_mapping
    # compressed slots exactly at compression boundaries
    assert torch.equal(comp >= 0, (pos + 1) % r == 0)
    # main slots: the token's page in its request's block table
    req = w.token_to_req.long()
    expect = w.block_table.long()[req, pos // page] * page + pos % page
    assert torch.equal(a["main_slots"], expect)
    # one work item per request for decode rows (max(groups, 1))
    kw = a["compressed_metadata"].k_work_metadata
    assert kw.shape == (8, 2) and kw[:, 1].eq(0).all()
    assert torch.equal(a["raw_metadata"].slot_mapping, req * 64 + pos % 64)
