"""Pin the CPU oracle against vectors produced by the reference itself.

``reference_triton.npz`` comes from the reference Triton kernels run under the
Triton CPU interpreter (``tests/golden/make_golden.py``), with fp32 storage of
bf16-representable values, hence ``round_p=False, round_out=False`` below.
``reference_topk.npz`` (when present) comes from the reference ``topk.cu``
compiled for sm_100a and run on a B200 (``tests/golden/make_topk_golden.py``).
"""

import numpy as np
import pytest
import torch

from golden_io import GOLDEN, from_bits16, load
from oracle import qsa_oracle as O

G = load("reference_triton.npz")


def _check_logits(ref: np.ndarray, got: torch.Tensor):
    got = got.numpy()
    written = ~np.isnan(ref)
    # The oracle writes exactly the columns the reference wrote.
    assert np.array_equal(written, ~np.isnan(got))
    np.testing.assert_allclose(got[written], ref[written], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", ["idx_dec1", "idx_dec2"])
def test_indexer_decode_matches_reference(case):
    q = from_bits16(G[f"{case}_q"])
    kc = from_bits16(G[f"{case}_kc"])
    table = torch.from_numpy(G[f"{case}_table"])
    vis = torch.from_numpy(G[f"{case}_visible"])
    ref = G[f"{case}_logits"]
    got = O.indexer_scores(q, kc, table, vis, ref.shape[1],
                           decode_query_len=int(G[f"{case}_dql"]))
    _check_logits(ref, got)


@pytest.mark.parametrize("name", ["full", "chunk"])
def test_indexer_prefill_matches_reference(name):
    q = from_bits16(G["idx_pre_q"])
    kc = from_bits16(G["idx_pre_kc"])
    table = torch.from_numpy(G["idx_pre_table"])
    qsl = torch.from_numpy(G["idx_pre_qsl"])
    vis = torch.from_numpy(G["idx_pre_visible"])
    width = int(G["idx_pre_width"])
    qoff, nq = (int(x) for x in G[f"idx_pre_{name}_range"])
    ref = G[f"idx_pre_{name}_logits"]
    full = O.indexer_scores(q, kc, table, vis, width, query_start_loc=qsl)
    _check_logits(ref, full[qoff:qoff + nq])


@pytest.mark.parametrize("case", ["att_dec", "att_dec_split", "att_pre", "att_pre_split"])
def test_attention_matches_reference(case):
    cfg = G[f"{case}_cfg"]
    rows, hq, hkv, d, page, nblk, physical, splits, block_n = (int(x) for x in cfg)
    kv = from_bits16(G[f"{case}_kv"])
    kc, vc = kv.split(d, dim=-1)
    q = from_bits16(G[f"{case}_q"])
    idx = torch.from_numpy(G[f"{case}_idx"])
    table = torch.from_numpy(G[f"{case}_table"])
    t2r = torch.from_numpy(G[f"{case}_t2r"])
    counts = torch.from_numpy(G[f"{case}_counts"]) if f"{case}_counts" in G else None
    gate = from_bits16(G[f"{case}_gate"]) if f"{case}_gate" in G else None
    out, po, pl = O.sparse_attention(
        q, kc, vc, idx, table, t2r, output_gate=gate, indices_are_physical=bool(physical),
        use_decode_kernel=bool(physical), valid_counts=counts, block_n=block_n,
        num_splits=splits, round_p=False, round_out=False, return_partials=True)
    if splits == 1:
        np.testing.assert_allclose(out.numpy(), G[f"{case}_out"], rtol=1e-5, atol=1e-6)
    else:
        np.testing.assert_allclose(po.numpy(), G[f"{case}_part_o"], rtol=1e-5, atol=1e-6)
        ref_lse = G[f"{case}_part_lse"]
        got_lse = pl.numpy()
        assert np.array_equal(np.isinf(ref_lse), np.isinf(got_lse))
        fin = np.isfinite(ref_lse)
        np.testing.assert_allclose(got_lse[fin], ref_lse[fin], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", ["logical", "physical"])
def test_expansion_rules_match_reference(name):
    ratio, token_topk, page = (int(x) for x in G["exp_cfg"])
    table = G["exp_table"] if name == "physical" else None
    out, counts = O.expand_block_indices(
        G["exp_blocks"], G["exp_pos"], G["exp_seq"], G["exp_t2r"], ratio, token_topk,
        main_block_table=table, main_page_size=page)
    assert np.array_equal(out, G[f"exp_{name}_out"])
    assert np.array_equal(counts, G[f"exp_{name}_counts"])


@pytest.mark.parametrize("name", ["logical", "physical"])
def test_topk_writer_agrees_with_expansion_rules(name):
    """The topk.cu writer and the Triton expansion are two statements of one rule:
    feed the oracle's selection through both and require identical output."""
    ratio, token_topk, page = (int(x) for x in G["exp_cfg"])
    rng = np.random.default_rng(7)
    rows = G["exp_pos"].shape[0]
    width = 18
    scores = torch.from_numpy(rng.random((rows, width), dtype=np.float32))
    lengths = torch.full((rows,), width, dtype=torch.int32)
    table = torch.from_numpy(G["exp_table"]) if name == "physical" else None
    pos = torch.from_numpy(G["exp_pos"])
    seq = torch.from_numpy(G["exp_seq"])
    t2r = torch.from_numpy(G["exp_t2r"])
    out, counts = O.topk_expand(scores, lengths, pos, seq, t2r, table,
                                token_topk + ratio - 1, ratio, page_size=page)
    blocks = np.stack([O.select_blocks(scores[r].numpy(), width, token_topk // ratio)
                       for r in range(rows)])
    ref, ref_counts = O.expand_block_indices(blocks, pos.numpy(), seq.numpy(), t2r.numpy(),
                                             ratio, token_topk,
                                             main_block_table=None if table is None
                                             else table.numpy(), main_page_size=page)
    assert np.array_equal(out, ref)
    mapped = t2r.numpy() >= 0
    assert np.array_equal(counts[mapped], ref_counts[mapped])


@pytest.mark.skipif(not (GOLDEN / "reference_topk.npz").exists(),
                    reason="reference topk.cu golden vectors not generated yet")
def test_topk_matches_reference_cuda():
    T = load("reference_topk.npz")
    for case in sorted({k.split("__")[0] for k in T}):
        f = lambda k: torch.from_numpy(T[f"{case}__{k}"])  # noqa: E731
        cfg = T[f"{case}__cfg"]
        ratio, page, physical, store_counts = (int(x) for x in cfg)
        table = f("table") if physical else None
        out, counts = O.topk_expand(f("scores"), f("lengths"), f("positions"), f("seq_lens"),
                                    f("token_to_req"), table, T[f"{case}__output"].shape[1],
                                    ratio, page_size=page)
        assert np.array_equal(out, T[f"{case}__output"]), case
        if store_counts:
            assert np.array_equal(counts, T[f"{case}__counts"]), case


def test_select_blocks_bit_order_semantics():
    """-0.0 ranks above positives, ties go to the lowest id, output ascending."""
    row = np.array([1.0, -0.0, 2.0, 2.0, 0.5, 2.0, 0.0], dtype=np.float32)
    assert list(O.select_blocks(row, 7, 3)) == [1, 2, 3]
    assert list(O.select_blocks(row, 7, 5)) == [0, 1, 2, 3, 5]
    assert list(O.select_blocks(row, 2, 3)) == [0, 1, -1]
    assert list(O.select_blocks(row, 0, 2)) == [-1, -1]


# ------------------------------------------------------------- qsa_prepare
def _prepare_inputs(d, name):
    g = lambda k: torch.from_numpy(d[f"{name}_in_{k}"].copy())  # noqa: E731
    consts = {k: int(d[f"{name}_in_{k}"]) for k in ("heads", "dim", "rotary", "ratio")}
    return g, consts, float(d[f"{name}_in_eps"])


@pytest.mark.parametrize("name", ["rot64", "rot32"])
def test_prepare_oracle_matches_reference_interpreter(name):
    """qsa_prepare (index queries, compressed keys, ring commit, main K/V) equals
    the reference kernel run under the Triton interpreter, bit for bit, with the
    interpreter's truncating bf16 conversion."""
    d = load("reference_prepare.npz")
    g, c, eps = _prepare_inputs(d, name)
    caches = {k: g(k) for k in ("state_cache", "compressed_cache", "main_key_cache",
                                "main_value_cache")}
    q = O.qsa_prepare(
        g("index_qk"), g("positions"), g("q_weight"), g("k_weight"), g("cos_sin"), eps,
        caches["state_cache"], g("state_slots"), g("state_table"), g("query_start_loc"),
        g("logical_positions"), caches["compressed_cache"], g("compressed_slots"), g("k_work"),
        g("main_key"), g("main_value"), caches["main_key_cache"], caches["main_value_cache"],
        g("main_slots"), num_index_heads=c["heads"], index_head_dim=c["dim"],
        rotary_dim=c["rotary"], compress_ratio=c["ratio"], rounding="truncate")
    assert torch.equal(q, torch.from_numpy(d[f"{name}_out_index_q"]))
    for k, v in caches.items():
        assert torch.equal(v, torch.from_numpy(d[f"{name}_out_{k}"])), k


def test_prefill_step_composes_the_pinned_pieces():
    """oracle.prefill_step (the prefill CPU baseline of bench.py) is the pinned
    indexer, top-k and attention functions chained: logical ids inside each
    row's causal window, counts as the expansion rules give them."""
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg1", device="cpu", seed=0, batch=1, new_tokens=3, seq_len=2048)
    out, idx, counts, logits = O.prefill_step(w)
    assert out.shape == w.q.shape and idx.shape == (3, w.token_topk + w.ratio - 1)
    pos, seq, rr = w.positions.numpy(), int(w.seq_lens[0]), w.ratio
    for r in range(3):
        valid = idx[r][idx[r] >= 0]
        complete = min((pos[r] + 1) // rr, seq // rr, w.token_topk // rr)
        assert valid.size == counts[r] == min(complete * rr + (pos[r] + 1) % rr, seq)
        assert valid.max() <= pos[r] and len(set(valid.tolist())) == valid.size
    vis = O.visible_blocks(w.positions, w.seq_lens, w.token_to_req, w.ratio)
    ref, _ = O.topk_expand(logits, vis, w.positions, w.seq_lens, w.token_to_req, None,
                           w.token_topk + w.ratio - 1, w.ratio)
    assert np.array_equal(idx, ref)
