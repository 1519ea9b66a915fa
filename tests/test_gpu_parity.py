"""GPU parity of the sm_100a kernels against the CPU oracle (and the reference top-k).

Bars: top-k / expansion / counts bit-exact; indexer scores within 1e-3
relative (+1e-5 absolute, fp32); attention outputs within max-abs 2e-2 (bf16)
and, because synthetic attention outputs are small, also within 2% of the
output's scale.  Every call goes through the C ABI (ctypes) of
``qsa_vllm_b200/libqsa_b200.so``.
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import qsa_oracle as O
from topk_cases import aligned_rows, make_case, standard_cases

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
REF_TOPK = ROOT / "oracle" / "_ref" / "libqsa_ref_topk.so"

SCORE_RTOL, SCORE_ATOL = 1e-3, 1e-5
ATT_ATOL, ATT_REL = 2e-2, 2e-2


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qsa_vllm_b200  # noqa: F401  (registers torch.ops.yulan_qsa_kernels)
    return torch.device("cuda")


def run_topk_expand(case: dict, dev, col_stride: int = 1, aligned: bool = False,
                    score_offset: int = 0):
    from qsa_vllm_b200.topk import topk_expand
    g = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    if aligned:
        g["scores"] = aligned_rows(g["scores"])
    if score_offset:
        s = g["scores"]
        buf = torch.zeros(s.shape[0], s.shape[1] + score_offset, dtype=s.dtype, device=dev)
        buf[:, score_offset:] = s
        g["scores"] = buf[:, score_offset:]
    rows = case["scores"].shape[0]
    width = case["output_width"]
    base = torch.full((rows, width * col_stride), -7, dtype=torch.int32, device=dev)
    out = base[:, ::col_stride]
    counts = torch.full((rows,), -7, dtype=torch.int32, device=dev)
    topk_expand(g["scores"], g["lengths"], g["positions"], g["seq_lens"], g["token_to_req"], out,
                case["ratio"], main_block_table=g["table"] if case["physical"] else None,
                main_page_size=case["page_size"],
                valid_counts_out=counts if case["store_counts"] else None)
    torch.cuda.synchronize()
    return out.cpu().numpy(), counts.cpu().numpy()


def oracle_topk_expand(case: dict):
    return O.topk_expand(case["scores"], case["lengths"], case["positions"], case["seq_lens"],
                         case["token_to_req"], case["table"] if case["physical"] else None,
                         case["output_width"], case["ratio"], page_size=case["page_size"])


@pytest.mark.parametrize("name", list(standard_cases().keys()))
def test_topk_expand_matches_oracle(dev, name):
    case = standard_cases()[name]
    got, counts = run_topk_expand(case, dev)
    ref, ref_counts = oracle_topk_expand(case)
    assert np.array_equal(got, ref), f"{name}: first diff at {np.argwhere(got != ref)[:5]}"
    if case["store_counts"]:
        assert np.array_equal(counts, ref_counts)


def test_topk_expand_unaligned_score_rows(dev):
    """Rows that are not 16-byte aligned take the scalar load path."""
    case = make_case(22, 9, 777, 128, kind="relu")
    ref, ref_counts = oracle_topk_expand(case)
    for off in (0, 1, 3):
        got, counts = run_topk_expand(case, dev, score_offset=off)
        assert np.array_equal(got, ref), off
        assert np.array_equal(counts, ref_counts)


def test_topk_expand_strided_output(dev):
    case = make_case(21, 7, 3000, 512, kind="ties")
    got, _ = run_topk_expand(case, dev, col_stride=3)
    ref, _ = oracle_topk_expand(case)
    assert np.array_equal(got, ref)


@pytest.mark.parametrize("rows,width,topk", [(1, 131072, 512), (8, 32768, 512),
                                             (64, 8192, 512), (300, 2048, 256),
                                             (3, 70000, 4096), (1, 200000, 2048)])
def test_topk_expand_cluster_widths(dev, rows, width, topk):
    """Cluster widths 1..16 CTAs per row, 8 or 32 keys per thread (set by the width)."""
    for kind in ("relu", "ties"):
        case = make_case(rows * 7 + width, rows, width, topk * 4, kind=kind, lengths="full")
        got, counts = run_topk_expand(case, dev)
        ref, ref_counts = oracle_topk_expand(case)
        assert np.array_equal(got, ref), kind
        assert np.array_equal(counts, ref_counts)


@pytest.mark.parametrize("rows,width,token_topk", [(1779, 2048, 1024), (1803, 2000, 1200),
                                                   (1801, 2048, 4096), (1790, 1500, 4400),
                                                   (1777, 700, 0), (33, 2048, 1024),
                                                   (12, 700, 0)])
def test_topk_expand_warp_rows(dev, rows, width, token_topk):
    """Many rows of <= 2048 keys (>= 12 per SM) run one warp per row: row
    counts that do not fill the CTA's 8 warps, both selection buffer sizes
    (top-k <= 256, <= 1024), the block kernel above top-k 1024 and for few
    rows, and top-k 0 (only the causal tail)."""
    for i, kind in enumerate(("relu", "ties", "signed", "zeros")):
        case = make_case(rows * 13 + width + i, rows, width, token_topk, kind=kind)
        got, counts = run_topk_expand(case, dev)
        ref, ref_counts = oracle_topk_expand(case)
        assert np.array_equal(got, ref), (kind, np.argwhere(got != ref)[:5])
        assert np.array_equal(counts, ref_counts), kind


def test_topk_plain_matches_oracle(dev):
    from qsa_vllm_b200.topk import topk
    for seed, (rows, width, k) in enumerate([(5, 100, 16), (4, 9000, 512), (2, 40000, 2048)]):
        case = make_case(seed + 40, rows, width, k, kind="ties" if seed % 2 else "relu")
        out = torch.full((rows, k), -7, dtype=torch.int32, device=dev)
        topk(case["scores"].to(dev), case["lengths"].to(dev), out)
        ref = O.topk_plain(case["scores"], case["lengths"], k)
        assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.skipif(not REF_TOPK.exists(), reason="reference topk.cu not built (oracle/build_ref.py)")
def test_topk_expand_matches_reference_cuda(dev):
    """Bit-exact against the reference topk.cu itself, compiled for sm_100a."""
    torch.ops.load_library(str(REF_TOPK))
    ref_op = torch.ops.yulan_qsa_ref_kernels.topk_expand
    cases = dict(standard_cases())
    cases["decode_64x8192"] = make_case(77, 64, 8192, 2048, kind="relu", lengths="full")
    cases["decode_8x32768"] = make_case(78, 8, 32768, 2048, kind="relu", lengths="full")
    for name, case in cases.items():
        got, counts = run_topk_expand(case, dev, aligned=True)
        g = {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
        g["scores"] = aligned_rows(g["scores"])   # the reference needs 16-byte aligned rows
        rows = case["scores"].shape[0]
        out = torch.full((rows, case["output_width"]), -7, dtype=torch.int32, device=dev)
        cnt = torch.full((rows,), -7, dtype=torch.int32, device=dev)
        ref_op(g["scores"], g["lengths"], g["positions"], g["seq_lens"], g["token_to_req"],
               g["table"] if case["physical"] else out, out,
               cnt if case["store_counts"] else out, case["ratio"], case["page_size"],
               case["physical"], case["store_counts"])
        torch.cuda.synchronize()
        assert np.array_equal(got, out.cpu().numpy()), name
        if case["store_counts"]:
            assert np.array_equal(counts, cnt.cpu().numpy()), name


# ------------------------------------------------------------------ indexer
def _indexer_case(dev, *, rows_per_req, requests, heads, dim, page, width, seed, weights):
    g = torch.Generator().manual_seed(seed)
    rows = requests * rows_per_req
    nblk = requests * width + 3
    q = (torch.randn(rows, heads, dim, generator=g) * dim ** -0.5).to(torch.bfloat16)
    kc = torch.randn(nblk, page, 1, dim, generator=g).to(torch.bfloat16)
    table = torch.randperm(nblk, generator=g)[: requests * width].view(requests, width)
    table = table.to(torch.int32).contiguous()
    table[0, -1] = -1
    vis = torch.randint(0, width * page + 1, (rows,), generator=g).to(torch.int32)
    vis[0] = width * page
    w = torch.rand(rows, heads, generator=g) if weights else None
    return q, kc, table, vis, w


# page % 8 == 0 runs the tcgen05/TMA kernel; other pages (4, 12, 60, 20) run
# the mma.sync kernel, the path for pages a TMA box cannot address
@pytest.mark.parametrize("heads,dim,page,dql,weights", [
    (8, 64, 64, 1, True), (4, 64, 16, 1, False), (4, 128, 16, 2, True),
    (16, 64, 32, 1, True), (1, 64, 16, 1, False), (2, 128, 8, 4, False),
    (64, 64, 64, 2, True), (48, 128, 24, 1, True), (8, 64, 128, 1, True),
    (8, 64, 256, 1, True), (8, 64, 4, 1, True), (4, 128, 12, 2, True),
    (8, 64, 60, 1, True), (4, 128, 20, 2, True)])
def test_indexer_decode_matches_oracle(dev, heads, dim, page, dql, weights):
    from qsa_vllm_b200.indexer import indexer_scores
    q, kc, table, vis, w = _indexer_case(dev, rows_per_req=dql, requests=5, heads=heads, dim=dim,
                                         page=page, width=40, seed=heads * dim + page,
                                         weights=weights)
    cols = 40 * page
    logits = torch.full((q.shape[0], cols), float("nan"), device=dev)
    indexer_scores(q.to(dev), kc.to(dev), table.to(dev), vis.to(dev), logits,
                   decode_query_len=dql, weights=None if w is None else w.to(dev))
    ref = O.indexer_scores(q, kc, table, vis, cols, decode_query_len=dql, weights=w)
    got = logits.cpu()
    assert torch.equal(torch.isnan(got), torch.isnan(ref))
    m = ~torch.isnan(ref)
    torch.testing.assert_close(got[m], ref[m], rtol=SCORE_RTOL, atol=SCORE_ATOL)


@pytest.mark.parametrize("heads,dim,page", [
    (4, 64, 16), (8, 64, 16), (4, 128, 16), (64, 64, 16),
    (48, 128, 16), (8, 64, 64), (8, 64, 6), (8, 64, 12)])
def test_indexer_prefill_matches_oracle(dev, heads, dim, page):
    from qsa_vllm_b200.indexer import indexer_scores
    g = torch.Generator().manual_seed(heads + dim + page)
    width, requests = 384 // page, 3
    qlens = [70, 1, 45]
    qsl = torch.tensor([0, 70, 71, 116], dtype=torch.int32)
    rows = sum(qlens)
    nblk = requests * width
    q = (torch.randn(rows, heads, dim, generator=g) * dim ** -0.5).to(torch.bfloat16)
    kc = torch.randn(nblk, page, 1, dim, generator=g).to(torch.bfloat16)
    table = torch.randperm(nblk, generator=g).view(requests, width).to(torch.int32)
    vis = torch.randint(0, width * page + 1, (rows,), generator=g).to(torch.int32)
    lw = 320
    for qoff, nq in ((0, rows), (50, 40)):
        logits = torch.full((nq, lw), float("nan"), device=dev)
        indexer_scores(q.to(dev), kc.to(dev), table.to(dev), vis.to(dev), logits,
                       query_start_loc=qsl.to(dev), max_query_len=70, query_offset=qoff,
                       num_rows=nq)
        ref = O.indexer_scores(q, kc, table, vis, lw, query_start_loc=qsl)[qoff:qoff + nq]
        got = logits.cpu()
        assert torch.equal(torch.isnan(got), torch.isnan(ref))
        m = ~torch.isnan(ref)
        torch.testing.assert_close(got[m], ref[m], rtol=SCORE_RTOL, atol=SCORE_ATOL)


def test_indexer_decode_many_segments_per_cta(dev):
    """More (request, key tile) units than resident CTAs: each persistent CTA
    walks several requests (segment slots reused) with random visible counts."""
    from qsa_vllm_b200.indexer import indexer_scores
    q, kc, table, vis, w = _indexer_case(dev, rows_per_req=1, requests=300, heads=8, dim=64,
                                         page=16, width=24, seed=11, weights=True)
    vis[::7] = 0
    cols = 24 * 16
    logits = torch.full((q.shape[0], cols), float("nan"), device=dev)
    indexer_scores(q.to(dev), kc.to(dev), table.to(dev), vis.to(dev), logits, weights=w.to(dev))
    ref = O.indexer_scores(q, kc, table, vis, cols, weights=w)
    got = logits.cpu()
    assert torch.equal(torch.isnan(got), torch.isnan(ref))
    m = ~torch.isnan(ref)
    torch.testing.assert_close(got[m], ref[m], rtol=SCORE_RTOL, atol=SCORE_ATOL)


@pytest.mark.parametrize("heads,dim", [(8, 64), (4, 128)])
def test_indexer_prefill_many_row_tiles(dev, heads, dim):
    """Long prefill requests: many row tiles per request, partial last tiles."""
    from qsa_vllm_b200.indexer import indexer_scores
    g = torch.Generator().manual_seed(7 + heads)
    page, width = 32, 12
    qlens = [333, 17, 250]
    qsl = torch.tensor([0, 333, 350, 600], dtype=torch.int32)
    rows, requests = sum(qlens), len(qlens)
    nblk = requests * width + 5
    q = (torch.randn(rows, heads, dim, generator=g) * dim ** -0.5).to(torch.bfloat16)
    kc = torch.randn(nblk, page, 1, dim, generator=g).to(torch.bfloat16)
    table = torch.randperm(nblk, generator=g)[: requests * width].view(requests, width)
    table = table.to(torch.int32).contiguous()
    vis = torch.randint(0, width * page + 1, (rows,), generator=g).to(torch.int32)
    w = torch.rand(rows, heads, generator=g)
    lw = width * page
    for qoff, nq in ((0, rows), (100, 333)):
        logits = torch.full((nq, lw), float("nan"), device=dev)
        indexer_scores(q.to(dev), kc.to(dev), table.to(dev), vis.to(dev), logits,
                       query_start_loc=qsl.to(dev), max_query_len=333, query_offset=qoff,
                       num_rows=nq, weights=w.to(dev))
        ref = O.indexer_scores(q, kc, table, vis, lw, query_start_loc=qsl, weights=w)
        ref = ref[qoff:qoff + nq]
        got = logits.cpu()
        assert torch.equal(torch.isnan(got), torch.isnan(ref))
        m = ~torch.isnan(ref)
        torch.testing.assert_close(got[m], ref[m], rtol=SCORE_RTOL, atol=SCORE_ATOL)


def test_indexer_rejects_decode_rows_without_table_rows(dev):
    """Decode rows need one page-table row per request: the call is refused on
    the host before any launch (no out-of-range table reads)."""
    from qsa_vllm_b200._lib import QSAError
    from qsa_vllm_b200.indexer import indexer_scores
    q, kc, table, vis, _ = _indexer_case(dev, rows_per_req=1, requests=4, heads=8, dim=64,
                                         page=16, width=8, seed=5, weights=False)
    logits = torch.zeros(q.shape[0], 8 * 16, device=dev)
    with pytest.raises(QSAError, match="page-table rows"):
        indexer_scores(q.to(dev), kc.to(dev), table[:2].to(dev), vis.to(dev), logits)


@pytest.mark.parametrize("config", ["cfg2", "cfg0"])
def test_kernels_derive_visible_counts_like_the_visible_kernel(dev, config):
    """visible_blocks=None: the indexer and top-k kernels derive each row's
    count themselves; results equal the path fed by qsa_visible_blocks."""
    from qsa_vllm_b200.indexer import compute_visible_blocks, indexer_scores
    from qsa_vllm_b200.synthetic import make_workload
    from qsa_vllm_b200.topk import topk_expand, topk_expand_visible
    w = make_workload(config, device=dev, seed=3, batch=16)
    vis = compute_visible_blocks(w.positions, w.seq_lens, w.token_to_req, w.ratio)
    cols = w.index_table.shape[1] * w.index_cache.shape[1]
    a = torch.full((w.rows, cols), float("nan"), device=dev)
    b = torch.full((w.rows, cols), float("nan"), device=dev)
    common = dict(weights=w.index_weights, scale=w.index_scale)
    indexer_scores(w.index_q, w.index_cache, w.index_table, vis, a, **common)
    indexer_scores(w.index_q, w.index_cache, w.index_table, None, b, query_positions=w.positions,
                   sequence_lengths=w.seq_lens, token_to_req=w.token_to_req,
                   compress_ratio=w.ratio, **common)
    assert torch.equal(torch.isnan(a), torch.isnan(b)) and torch.equal(a.nan_to_num(), b.nan_to_num())
    width = w.token_topk + w.ratio - 1
    outs = []
    for derived in (False, True):
        out = torch.empty(w.rows, width, dtype=torch.int32, device=dev)
        cnt = torch.empty(w.rows, dtype=torch.int32, device=dev)
        kw = dict(main_block_table=w.block_table, main_page_size=w.page_size,
                  valid_counts_out=cnt)
        if derived:
            topk_expand_visible(a.nan_to_num(), w.positions, w.seq_lens, w.token_to_req, out,
                                w.ratio, **kw)
        else:
            topk_expand(a.nan_to_num(), vis, w.positions, w.seq_lens, w.token_to_req, out,
                        w.ratio, **kw)
        outs.append((out, cnt))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


# ---------------------------------------------------------------- attention
def _attention_check(got: torch.Tensor, ref: torch.Tensor):
    got = got.float().cpu()
    err = (got - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert err <= ATT_ATOL, f"max-abs {err}"
    assert err <= ATT_REL * max(scale, 1e-6) + 1e-4, f"max-abs {err} vs scale {scale}"


@pytest.mark.parametrize("rows,hq,hkv,d,physical,gate,counts", [
    (5, 16, 2, 128, True, True, True),      # decode, few rows -> split-K
    (64, 32, 4, 128, True, True, True),     # decode at the headline head shape
    (7, 16, 4, 64, True, False, True),      # group 4, head_dim 64
    (6, 32, 2, 128, False, False, False),   # prefill (logical ids), group 16
    (300, 16, 2, 128, False, True, False),  # prefill, many rows -> one split
    (3, 8, 8, 128, True, True, False),      # MHA (group 1)
])
def test_attention_matches_oracle(dev, rows, hq, hkv, d, physical, gate, counts):
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    g = torch.Generator().manual_seed(rows * hq + d)
    page, nblk, requests = 16, 96, 3
    width = 515
    kv = torch.randn(nblk, page, hkv, 2 * d, generator=g).to(torch.bfloat16)
    q = (torch.randn(rows, hq, d, generator=g) * d ** -0.5 * 4).to(torch.bfloat16)
    t_width = nblk // requests
    table = torch.randperm(nblk, generator=g)[: requests * t_width].view(requests, t_width)
    table = table.to(torch.int32).contiguous()
    table[0, 1] = -1
    t2r = torch.randint(0, requests, (rows,), generator=g).to(torch.int32)
    t2r[-1] = -1
    if physical:
        idx = torch.randint(-1, nblk * page, (rows, width), generator=g).to(torch.int32)
    else:
        idx = torch.randint(-1, t_width * page + 2 * page, (rows, width), generator=g)
        idx = idx.to(torch.int32)
    vc = torch.randint(0, width + 1, (rows,), generator=g).to(torch.int32) if counts else None
    if vc is not None:
        vc[0] = width
        # Contract of valid_counts (what topk_expand writes): columns at or beyond
        # the count hold -1.  The reference's kernel would also read valid ids
        # there up to the end of its BLOCK_N tile, a schedule-dependent artifact.
        idx[torch.arange(width)[None, :] >= vc[:, None]] = -1
    gt = torch.randn(rows, hq, d, generator=g).to(torch.bfloat16) if gate else None
    kvd = kv.to(dev)
    out = torch.full((rows, hq, d), float("nan"), dtype=torch.bfloat16, device=dev)
    qsa_sparse_paged_attention(
        q.to(dev), kvd[..., :d], kvd[..., d:], idx.to(dev), table.to(dev), t2r.to(dev), out,
        output_gate=None if gt is None else gt.to(dev), use_decode_kernel=physical,
        indices_are_physical=physical, valid_counts=None if vc is None else vc.to(dev))
    torch.cuda.synchronize()
    ref = O.sparse_attention(q, kv[..., :d], kv[..., d:], idx, table, t2r, output_gate=gt,
                             use_decode_kernel=physical, indices_are_physical=physical,
                             valid_counts=vc)
    _attention_check(out, ref)


@pytest.mark.parametrize("rows,hq,hkv,d,physical", [(300, 16, 2, 128, False), (5, 16, 2, 128, True),
                                                   (200, 8, 2, 64, False), (40, 32, 2, 128, False)])
def test_attention_strided_gate_and_output(dev, rows, hq, hkv, d, physical):
    """Gate with a non-unit dim stride and output rows that are only 4-byte
    aligned: the scalar gate loads and 4-byte output stores, on pairs finished
    in the main kernel (many rows) and on split pairs (few rows)."""
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    g = torch.Generator().manual_seed(rows + d)
    page, nblk = 16, 64
    width = 259
    kv = torch.randn(nblk, page, hkv, 2 * d, generator=g).to(torch.bfloat16)
    q = (torch.randn(rows, hq, d, generator=g) * d ** -0.5 * 4).to(torch.bfloat16)
    table = torch.randperm(nblk, generator=g)[:nblk // 2].view(2, nblk // 4).to(torch.int32)
    t2r = torch.randint(0, 2, (rows,), generator=g).to(torch.int32)
    hi = nblk * page if physical else (nblk // 4) * page
    idx = torch.randint(-1, hi, (rows, width), generator=g).to(torch.int32)
    gate_t = torch.randn(rows, d, hq, generator=g).to(torch.bfloat16)
    gate = gate_t.to(dev).permute(0, 2, 1)            # dim stride hq
    assert gate.stride(2) != 1
    buf = torch.full((rows, hq, d + 2), float("nan"), dtype=torch.bfloat16, device=dev)
    out = buf[:, :, 2:]                                # rows start 4 bytes past 16-byte alignment
    qsa_sparse_paged_attention(q.to(dev), kv.to(dev)[..., :d], kv.to(dev)[..., d:], idx.to(dev),
                               table.to(dev), t2r.to(dev), out, output_gate=gate,
                               use_decode_kernel=physical, indices_are_physical=physical)
    torch.cuda.synchronize()
    ref = O.sparse_attention(q, kv[..., :d], kv[..., d:], idx, table, t2r,
                             output_gate=gate_t.permute(0, 2, 1), use_decode_kernel=physical,
                             indices_are_physical=physical)
    _attention_check(out, ref)
    assert torch.isnan(buf[:, :, :2].float()).all()   # nothing written outside the view


def test_attention_misaligned_query_view(dev):
    """A contiguous query view 2 bytes past a 16-byte boundary: the wrapper
    copies it to aligned rows, and the output equals the aligned call's."""
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    g = torch.Generator().manual_seed(11)
    rows, hq, hkv, d, page, nblk = 6, 16, 2, 128, 16, 40
    kv = torch.randn(nblk, page, hkv, 2 * d, generator=g).to(torch.bfloat16).to(dev)
    q = (torch.randn(rows, hq, d, generator=g) * 0.3).to(torch.bfloat16).to(dev)
    base = torch.empty(1 + rows * hq * d, dtype=torch.bfloat16, device=dev)
    q_view = base[1:].view(rows, hq, d)
    q_view.copy_(q)
    assert q_view.is_contiguous() and q_view.data_ptr() % 16 == 2
    idx = torch.randint(-1, nblk * page, (rows, 131), generator=g).to(torch.int32).to(dev)
    table = torch.zeros(1, 1, dtype=torch.int32, device=dev)
    t2r = torch.zeros(rows, dtype=torch.int32, device=dev)
    outs = []
    for qq in (q, q_view):
        outs.append(qsa_sparse_paged_attention(qq, kv[..., :d], kv[..., d:], idx, table, t2r,
                                               use_decode_kernel=True, indices_are_physical=True))
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])


def test_attention_separate_kv_buffers(dev):
    """K and V in different allocations (two bulk copies per token)."""
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    g = torch.Generator().manual_seed(5)
    rows, hq, hkv, d, page, nblk = 9, 16, 2, 128, 16, 40
    k = torch.randn(nblk, page, hkv, d, generator=g).to(torch.bfloat16)
    v = torch.randn(nblk, page, hkv, d, generator=g).to(torch.bfloat16)
    q = (torch.randn(rows, hq, d, generator=g) * 0.3).to(torch.bfloat16)
    idx = torch.randint(-1, nblk * page, (rows, 131), generator=g).to(torch.int32)
    table = torch.zeros(1, 1, dtype=torch.int32)
    t2r = torch.zeros(rows, dtype=torch.int32)
    out = torch.empty(rows, hq, d, dtype=torch.bfloat16, device=dev)
    qsa_sparse_paged_attention(q.to(dev), k.to(dev), v.to(dev), idx.to(dev), table.to(dev),
                               t2r.to(dev), out, use_decode_kernel=True,
                               indices_are_physical=True)
    torch.cuda.synchronize()
    ref = O.sparse_attention(q, k, v, idx, table, t2r, use_decode_kernel=True,
                             indices_are_physical=True)
    _attention_check(out, ref)


# -------------------------------------------------------- whole decode step
def _decode_step(w, dev):
    from qsa_vllm_b200.indexer import select_paged_tokens
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    rows = w.rows
    out_idx = torch.empty(rows, w.token_topk + w.ratio - 1, dtype=torch.int32, device=dev)
    counts = torch.empty(rows, dtype=torch.int32, device=dev)
    select_paged_tokens(
        w.index_q, w.index_cache, w.index_table, w.token_to_req, w.positions, w.seq_lens,
        w.token_topk, w.ratio, out_idx, **w.select_kwargs(),
        main_block_table=w.block_table, main_page_size=w.page_size, valid_counts_out=counts,
        weights=w.index_weights, scale=w.index_scale)
    out = torch.empty_like(w.q)
    qsa_sparse_paged_attention(w.q, w.k_cache, w.v_cache, out_idx, w.block_table,
                               w.token_to_req, out, output_gate=w.gate, use_decode_kernel=True,
                               indices_are_physical=True, valid_counts=counts)
    torch.cuda.synchronize()
    return out_idx, counts, out


def _check_decode_rows(w, dev, out_idx, counts, out, rows_to_check):
    """Indexer scores (tolerance), selection on the GPU's own scores (bit-exact)
    and attention (tolerance) for a subset of rows."""
    from qsa_vllm_b200.indexer import indexer_scores
    vis = O.visible_blocks(w.positions.cpu(), w.seq_lens.cpu(), w.token_to_req.cpu(), w.ratio)
    cols = w.index_table.shape[1] * w.index_cache.shape[1]
    logits = torch.zeros(w.rows, cols, device=dev)
    dql = w.decode_query_len
    indexer_scores(w.index_q, w.index_cache, w.index_table, vis.to(dev), logits,
                   decode_query_len=dql, weights=w.index_weights, scale=w.index_scale)
    gl = logits.cpu()
    sel = torch.tensor(rows_to_check)
    ref_l = O.indexer_scores(w.index_q.cpu()[sel], w.index_cache.cpu(),
                             w.index_table.cpu()[sel // dql], vis[sel], cols,
                             weights=w.index_weights.cpu()[sel], scale=w.index_scale)
    for i, r in enumerate(rows_to_check):
        n = int(vis[r])
        torch.testing.assert_close(gl[r, :n], ref_l[i, :n], rtol=SCORE_RTOL, atol=SCORE_ATOL)
    # selection: oracle top-k applied to the GPU's own fp32 scores -> bit-exact
    ref_idx, ref_cnt = O.topk_expand(gl, vis, w.positions.cpu(), w.seq_lens.cpu(),
                                     w.token_to_req.cpu(), w.block_table.cpu(),
                                     w.token_topk + w.ratio - 1, w.ratio, page_size=w.page_size)
    assert np.array_equal(out_idx.cpu().numpy(), ref_idx)
    assert np.array_equal(counts.cpu().numpy(), ref_cnt)
    # attention on the selected rows: gather the touched pages into a compact cache
    idx = out_idx.cpu()[sel]
    cnt = counts.cpu()[sel]
    pages = torch.unique(idx[idx >= 0] // w.page_size)
    remap = torch.full((w.kv.shape[0],), -1, dtype=torch.int64)
    remap[pages] = torch.arange(pages.numel())
    compact = w.kv[pages.to(dev)].cpu()
    cidx = torch.where(idx >= 0, remap[(idx.clamp_min(0) // w.page_size).long()] * w.page_size
                       + idx.clamp_min(0) % w.page_size, torch.full_like(idx, -1)).to(torch.int32)
    d = w.d
    ref = O.sparse_attention(w.q.cpu()[sel], compact[..., :d], compact[..., d:], cidx,
                             torch.zeros(1, 1, dtype=torch.int32), w.token_to_req.cpu()[sel],
                             output_gate=w.gate.cpu()[sel], use_decode_kernel=True,
                             indices_are_physical=True, valid_counts=cnt)
    _attention_check(out[sel.to(dev)], ref)


def test_decode_step_cfg0(dev):
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg0", device=dev, seed=0)
    out_idx, counts, out = _decode_step(w, dev)
    _check_decode_rows(w, dev, out_idx, counts, out, list(range(w.rows)))


def test_decode_step_cfg2_mixed_lengths(dev):
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg2", device=dev, seed=3)
    out_idx, counts, out = _decode_step(w, dev)
    _check_decode_rows(w, dev, out_idx, counts, out, list(range(0, w.rows, 3)))


def test_decode_step_cfg2_32k_full_size(dev):
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg2_32k", device=dev, seed=1)
    out_idx, counts, out = _decode_step(w, dev)
    _check_decode_rows(w, dev, out_idx, counts, out, list(range(w.rows)))
    # size-independent property: every row selects K_blk*ratio + tail valid slots
    assert bool((counts == w.token_topk + (w.positions + 1) % w.ratio).all())


def test_decode_step_cfg3_long_context(dev):
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg3", device=dev, seed=2)
    out_idx, counts, out = _decode_step(w, dev)
    _check_decode_rows(w, dev, out_idx, counts, out, list(range(w.rows)))


def test_decode_step_ratio1(dev):
    """Per-token index keys (compress ratio 1): 32768-wide score rows, the
    clustered top-k, no causal tail."""
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg2_32k_r1", device=dev, seed=4, batch=8)
    out_idx, counts, out = _decode_step(w, dev)
    _check_decode_rows(w, dev, out_idx, counts, out, [0, 5])
    assert bool((counts == w.token_topk).all())


def test_decode_step_mtp2(dev):
    """Multi-token decode: two query rows per request share its page-table row;
    the second row sees one more token (and possibly one more block)."""
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg2_32k_mtp2", device=dev, seed=5, batch=8, seq_len=(8190, 8195))
    assert w.rows == 16 and w.decode_query_len == 2
    out_idx, counts, out = _decode_step(w, dev)
    _check_decode_rows(w, dev, out_idx, counts, out, [0, 1, 14, 15])


@pytest.mark.parametrize("config,tp,rank", [("cfg2_32k", 4, 3), ("cfg2_32k", 8, 5),
                                             ("cfg3", 4, 1), ("cfg3", 8, 6)])
def test_decode_step_head_shard(dev, config, tp, rank):
    """One rank's share under head sharding (the multi-GPU benchmark's layout):
    tp 4 keeps 8 query heads / 1 KV head, tp 8 keeps 4 query heads of a KV
    head replicated on two ranks; the indexer and top-k are replicated."""
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload(config, device=dev, seed=9, batch=8).shard_heads(tp, rank)
    assert w.q.shape[1] == 32 // tp and w.kv.shape[2] == 1
    out_idx, counts, out = _decode_step(w, dev)
    _check_decode_rows(w, dev, out_idx, counts, out, [0, 3, 7])


def test_prefill_step_cfg1(dev):
    """Chunked prefill: logical ids, per-row causal visibility, many rows."""
    from qsa_vllm_b200.indexer import indexer_scores, select_paged_tokens
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg1", device=dev, seed=0, head_weights=False)
    rows = w.rows
    out_idx = torch.empty(rows, w.token_topk + w.ratio - 1, dtype=torch.int32, device=dev)
    select_paged_tokens(
        w.index_q, w.index_cache, w.index_table, w.token_to_req, w.positions, w.seq_lens,
        w.token_topk, w.ratio, out_idx, query_start_loc=w.query_start_loc,
        max_query_len=w.max_query_len, max_seq_len=w.max_seq_len)
    out = torch.empty_like(w.q)
    qsa_sparse_paged_attention(w.q, w.k_cache, w.v_cache, out_idx, w.block_table,
                               w.token_to_req, out, output_gate=w.gate)
    torch.cuda.synchronize()
    vis = O.visible_blocks(w.positions.cpu(), w.seq_lens.cpu(), w.token_to_req.cpu(), w.ratio)
    lw = -(-(-(-w.max_seq_len // w.ratio)) // 64) * 64
    logits = torch.zeros(rows, lw, device=dev)
    indexer_scores(w.index_q, w.index_cache, w.index_table, vis.to(dev), logits,
                   query_start_loc=w.query_start_loc, max_query_len=w.max_query_len)
    gl = logits.cpu()
    # 70 rows: every 128th row of both requests plus each request's first and
    # last rows and the chunk boundaries
    check = sorted(set(range(0, rows, 128)) | {1, 2047, 4095, 4096, 6000, rows - 1})
    ref_l = O.indexer_scores(w.index_q.cpu(), w.index_cache.cpu(), w.index_table.cpu(), vis, lw,
                             query_start_loc=w.query_start_loc.cpu())
    for r in check:
        n = int(vis[r])
        torch.testing.assert_close(gl[r, :n], ref_l[r, :n], rtol=SCORE_RTOL, atol=SCORE_ATOL)
    ref_idx, _ = O.topk_expand(gl, vis, w.positions.cpu(), w.seq_lens.cpu(), w.token_to_req.cpu(),
                               None, w.token_topk + w.ratio - 1, w.ratio)
    assert np.array_equal(out_idx.cpu().numpy(), ref_idx)
    sel = torch.tensor(check)
    ref = O.sparse_attention(w.q.cpu()[sel], w.k_cache.cpu(), w.v_cache.cpu(),
                             out_idx.cpu()[sel], w.block_table.cpu(),
                             w.token_to_req.cpu()[sel], output_gate=w.gate.cpu()[sel])
    _attention_check(out[sel.to(dev)], ref)


def test_no_device_errors_recorded(dev):
    from qsa_vllm_b200 import _lib
    assert _lib.device_error_poll() == 0


def test_visible_blocks_kernel_matches_reference_formula(dev):
    from qsa_vllm_b200.indexer import compute_visible_blocks
    g = torch.Generator().manual_seed(3)
    seq = torch.randint(0, 5000, (9,), generator=g).to(torch.int32)
    t2r = torch.randint(-1, 9, (300,), generator=g).to(torch.int32)
    pos = torch.randint(-6, 6000, (300,), generator=g).to(torch.int64)
    for ratio in (1, 4, 7):
        got = compute_visible_blocks(pos.to(dev), seq.to(dev), t2r.to(dev), ratio).cpu()
        assert torch.equal(got, O.visible_blocks(pos, seq, t2r, ratio))


def test_bounded_wait_expires_reports_and_leaves_the_context_usable(dev):
    """The error path shared by every kernel's bounded waits: a wait on a
    barrier phase that nothing completes gives up after its 1 s limit, sets
    QSA_DEVICE_ERR_WAIT_TIMEOUT in the device error word, and the next calls
    run normally with no error recorded."""
    from qsa_vllm_b200 import _lib
    from qsa_vllm_b200.topk import topk
    lib = _lib.load_library()
    assert _lib.device_error_poll() == 0
    _lib.check(lib.qsa_selftest_wait_timeout(_lib.stream_ptr(dev)), "wait-timeout self-test")
    torch.cuda.synchronize()
    assert _lib.device_error_poll() == 1      # QSA_DEVICE_ERR_WAIT_TIMEOUT
    assert _lib.device_error_poll() == 0      # read-and-clear
    case = make_case(91, 3, 500, 64, kind="relu")
    out = torch.full((3, 64), -7, dtype=torch.int32, device=dev)
    topk(case["scores"].to(dev), case["lengths"].to(dev), out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.topk_plain(case["scores"], case["lengths"], 64))
    assert _lib.device_error_poll() == 0
