"""GPU parity of the fused decode selection (``qsa_select_decode``).

The fused kernel must give, bit for bit, what the two-call path gives on the
same inputs: ``qsa_indexer_scores`` into fp32 logits, then
``qsa_topk_expand`` on them (the reference's qsa_select_paged_decode,
ops/indexer.py:227-279).  Its optional scores copy must equal the scoring
kernel's logits bit for bit and the oracle's within 1e-3 relative; its
selection must equal the oracle top-k applied to those scores.  Shapes cover
cluster widths 1..16, decode_query_len 1 / 2 / 4, head dims 64 / 128, tied
scores (zero weights), negative scores (uint32 bit-pattern order), unmapped
pages, rows at or below the budget, the logits bucket clipping rows, and
visible counts derived in the kernel.  Every call goes through the C ABI.
"""

from __future__ import annotations

import zlib

import numpy as np
import pytest
import torch

from oracle import qsa_oracle as O

pytestmark = pytest.mark.gpu

SCORE_RTOL, SCORE_ATOL = 1e-3, 1e-5


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qsa_vllm_b200  # noqa: F401
    return torch.device("cuda")


def _case(seed, *, requests, dql, heads, dim, page, pages_per_req, ratio, topk_tokens,
          main_page=64, weights="rand", unmapped=True, short_rows=True, one_sided=False):
    g = torch.Generator().manual_seed(seed)
    rows = requests * dql
    cap_tokens = pages_per_req * page * ratio
    seq = torch.randint(max(dql, cap_tokens // 4), cap_tokens + 1, (requests,), generator=g)
    if short_rows and requests > 2:
        seq[1] = min(int(seq[1]), topk_tokens // 2 + 3)   # at or below the budget
        seq[2] = dql                                      # almost nothing visible
    if one_sided:
        # rows a little above the budget, all within the first CTA's columns:
        # that CTA's candidates alone make up the selection
        seq[:] = topk_tokens + ratio * (8 + torch.arange(requests) % 80)
    seq = seq.to(torch.int32)
    t2r = torch.arange(requests, dtype=torch.int32).repeat_interleave(dql)
    pos = (seq.long().repeat_interleave(dql) - dql
           + torch.arange(dql).repeat(requests)).clamp_min(0)
    nblk = requests * pages_per_req + 3
    kc = torch.randn(nblk, page, 1, dim, generator=g).to(torch.bfloat16)
    table = torch.randperm(nblk, generator=g)[: requests * pages_per_req]
    table = table.view(requests, pages_per_req).to(torch.int32).contiguous()
    if unmapped:
        table[0, 1] = -1
        table[-1, 0] = nblk + 50          # out of range: zero keys, as the reference
    q = (torch.randn(rows, heads, dim, generator=g) * dim ** -0.5).to(torch.bfloat16)
    if weights == "rand":
        w = torch.rand(rows, heads, generator=g)
    elif weights == "zero":
        w = torch.zeros(rows, heads)     # every score 0.0: all ties
    elif weights == "neg":
        w = -torch.rand(rows, heads, generator=g)
    else:
        w = None
    mp = -(-cap_tokens // main_page)
    main_table = torch.randperm(requests * mp + 5, generator=g)[: requests * mp]
    main_table = main_table.view(requests, mp).to(torch.int32).contiguous()
    return dict(q=q, kc=kc, table=table, seq=seq, t2r=t2r, pos=pos, w=w, ratio=ratio,
                topk_tokens=topk_tokens, main_table=main_table, main_page=main_page, dql=dql)


def _run_both(c, dev, *, columns=None, derive_visible=False):
    from qsa_vllm_b200 import _lib
    from qsa_vllm_b200.indexer import (compute_visible_blocks, indexer_scores,
                                       select_decode_fused)
    from qsa_vllm_b200.topk import topk_expand
    d = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
    rows = d["q"].shape[0]
    ratio = c["ratio"]
    width = c["topk_tokens"] + ratio - 1
    cap = d["table"].shape[1] * d["kc"].shape[1]
    cols = cap if columns is None else columns
    vis = compute_visible_blocks(d["pos"], d["seq"], d["t2r"], ratio)
    out_f = torch.full((rows, width), -7, dtype=torch.int32, device=dev)
    cnt_f = torch.full((rows,), -7, dtype=torch.int32, device=dev)
    sc_f = torch.full((rows, cols), float("nan"), device=dev)
    launched = select_decode_fused(
        d["q"], d["kc"], d["table"], None if derive_visible else vis, ratio, c["dql"], out_f,
        cols, query_positions=d["pos"], sequence_lengths=d["seq"], token_to_req=d["t2r"],
        main_block_table=d["main_table"], main_page_size=c["main_page"],
        valid_counts_out=cnt_f, weights=d["w"], scores_out=sc_f)
    if not launched:
        raise AssertionError("the fused kernel declined these shapes: "
                             + _lib.load_library().qsa_last_error().decode())
    logits = torch.full((rows, cols), float("nan"), device=dev)
    indexer_scores(d["q"], d["kc"], d["table"], vis, logits, decode_query_len=c["dql"],
                   weights=d["w"])
    out_t = torch.full((rows, width), -7, dtype=torch.int32, device=dev)
    cnt_t = torch.full((rows,), -7, dtype=torch.int32, device=dev)
    topk_expand(logits.nan_to_num(), vis, d["pos"], d["seq"], d["t2r"], out_t, ratio,
                main_block_table=d["main_table"], main_page_size=c["main_page"],
                valid_counts_out=cnt_t)
    torch.cuda.synchronize()
    return (out_f.cpu(), cnt_f.cpu(), sc_f.cpu(), out_t.cpu(), cnt_t.cpu(), logits.cpu(),
            vis.cpu(), cols)


CASES = {
    # name: (case kwargs, columns (None = table capacity))
    "h8_d64_c2": (dict(requests=64, dql=1, heads=8, dim=64, page=64, pages_per_req=128,
                       ratio=4, topk_tokens=2048), None),
    "cluster16": (dict(requests=4, dql=1, heads=8, dim=64, page=64, pages_per_req=512,
                       ratio=4, topk_tokens=2048), None),
    "cluster1_many_requests": (dict(requests=100, dql=1, heads=8, dim=64, page=16,
                                    pages_per_req=40, ratio=4, topk_tokens=512), None),
    "mtp2": (dict(requests=20, dql=2, heads=8, dim=64, page=16, pages_per_req=96, ratio=4,
                  topk_tokens=1024), None),
    "dql4_h8_nq32": (dict(requests=12, dql=4, heads=8, dim=64, page=32, pages_per_req=40,
                          ratio=4, topk_tokens=512), None),
    "d128_h4": (dict(requests=9, dql=1, heads=4, dim=128, page=32, pages_per_req=64,
                     ratio=4, topk_tokens=1024), None),
    "d128_h16_dql2": (dict(requests=7, dql=2, heads=16, dim=128, page=16, pages_per_req=50,
                           ratio=4, topk_tokens=512), None),
    "ratio1": (dict(requests=8, dql=1, heads=8, dim=64, page=64, pages_per_req=128, ratio=1,
                    topk_tokens=2048), None),
    "ties_zero_weights": (dict(requests=10, dql=1, heads=8, dim=64, page=64, pages_per_req=32,
                               ratio=4, topk_tokens=512, weights="zero"), None),
    "negative_scores": (dict(requests=10, dql=1, heads=8, dim=64, page=64, pages_per_req=32,
                             ratio=4, topk_tokens=512, weights="neg"), None),
    "unit_weights_h1": (dict(requests=6, dql=1, heads=1, dim=64, page=8, pages_per_req=100,
                             ratio=4, topk_tokens=256, weights=None), None),
    "bucket_clips_rows": (dict(requests=16, dql=1, heads=8, dim=64, page=64, pages_per_req=64,
                               ratio=4, topk_tokens=1024), 1500),
    "candidates_from_one_cta": (dict(requests=64, dql=1, heads=8, dim=64, page=64,
                                     pages_per_req=128, ratio=4, topk_tokens=2048,
                                     one_sided=True, short_rows=False), None),
}


@pytest.mark.parametrize("name", list(CASES))
def test_select_decode_fused_matches_two_call_path(dev, name):
    kwargs, columns = CASES[name]
    c = _case(zlib.crc32(name.encode()) % 1000, **kwargs)
    out_f, cnt_f, sc_f, out_t, cnt_t, logits, vis, cols = _run_both(c, dev, columns=columns)
    # scores: the same bits as the scoring kernel, written exactly where it writes
    assert torch.equal(torch.isnan(sc_f), torch.isnan(logits)), name
    assert torch.equal(sc_f.nan_to_num(), logits.nan_to_num()), name
    # selection, expansion and counts: bit-exact against the two-call path ...
    assert torch.equal(out_f, out_t), f"{name}: first diff {torch.nonzero(out_f != out_t)[:5]}"
    assert torch.equal(cnt_f, cnt_t), name
    # ... and against the oracle's top-k on the same scores
    ref_idx, ref_cnt = O.topk_expand(sc_f.nan_to_num(), vis, c["pos"], c["seq"], c["t2r"],
                                     c["main_table"], out_f.shape[1], c["ratio"],
                                     page_size=c["main_page"])
    assert np.array_equal(out_f.numpy(), ref_idx), name
    assert np.array_equal(cnt_f.numpy(), ref_cnt), name
    # scores against the oracle's restatement of the reference math
    ref = O.indexer_scores(c["q"], c["kc"], c["table"], vis, cols, decode_query_len=c["dql"],
                           weights=c["w"])
    m = ~torch.isnan(ref)
    assert torch.equal(m, ~torch.isnan(sc_f)), name
    torch.testing.assert_close(sc_f[m], ref[m], rtol=SCORE_RTOL, atol=SCORE_ATOL)


def test_select_decode_fused_derives_visible_counts(dev):
    """visible=None: the fused kernel derives each row's count from positions,
    sequence lengths and token_to_req, as qsa_visible_blocks does."""
    c = _case(5, requests=32, dql=1, heads=8, dim=64, page=64, pages_per_req=64, ratio=4,
              topk_tokens=1024)
    out_f, cnt_f, sc_f, out_t, cnt_t, logits, _, _ = _run_both(c, dev, derive_visible=True)
    assert torch.equal(out_f, out_t) and torch.equal(cnt_f, cnt_t)
    assert torch.equal(sc_f.nan_to_num(), logits.nan_to_num())


def test_select_decode_repeated_calls_agree(dev):
    """Two calls in a row on the same inputs give the same bits (no state is
    carried between launches)."""
    c = _case(11, requests=64, dql=1, heads=8, dim=64, page=64, pages_per_req=128, ratio=4,
              topk_tokens=2048)
    a = _run_both(c, dev)
    b = _run_both(c, dev)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_select_decode_declines_shapes_outside_its_range(dev):
    """Pages that a TMA box cannot address (page % 8 != 0) and non power-of-two
    head counts are declined without a launch; select_paged_tokens then takes
    the two-call path with the same results."""
    from qsa_vllm_b200 import _lib
    from qsa_vllm_b200.indexer import select_decode_fused
    for kw in (dict(heads=8, page=12), dict(heads=6, page=16)):
        c = _case(7, requests=4, dql=1, dim=64, pages_per_req=20, ratio=4, topk_tokens=256,
                  **kw)
        d = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in c.items()}
        out = torch.empty(4, 259, dtype=torch.int32, device=dev)
        n0 = _lib.kernel_launches()
        assert not select_decode_fused(
            d["q"], d["kc"], d["table"], None, 4, 1, out, 20 * kw["page"],
            query_positions=d["pos"], sequence_lengths=d["seq"], token_to_req=d["t2r"],
            weights=d["w"])
        assert _lib.kernel_launches() == n0


def test_select_decode_no_device_errors(dev):
    from qsa_vllm_b200 import _lib
    assert _lib.device_error_poll() == 0
