"""CPU oracle for the QSA sparse-attention hot path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` import it.
It restates in numpy / PyTorch-eager CPU code what the reference plugin
(clotholza/qsa_vllm, package ``yulan_qsa_vllm``) computes on its hot path:

1. ``visible_blocks``      ops/indexer.py:363-369
2. ``indexer_scores``      ops/indexer.py:24-114 (uniform decode kernel) and
                           ops/indexer.py:117-223 (packed prefill kernel)
3. ``topk_expand``         ops/csrc/topk.cu:107-180 (expansion writer),
                           :182-350 (exact selection), :410-501 (launchers)
4. ``expand_block_indices``ops/qsa.py:18-106 (the unused Triton expansion,
                           a second statement of the same expansion rules)
5. ``sparse_attention``    ops/qsa.py:109-303 (split-K paged GQA kernel),
                           :306-362 (split merge), :594-688 (launch table)
6. ``qsa_prepare``         ops/prepare.py:16-46 (norm + RoPE with bf16 rounding
                           steps), :49-166 (index queries, key compression,
                           raw-key ring commit, main K/V cache writes)

Parity pin.  The reference ships no tests or golden vectors.  This oracle is
pinned against fixtures produced from the reference itself:
``tests/golden/make_golden.py`` runs the reference Triton kernels under the
Triton CPU interpreter (fp32 storage of bf16-representable values, because
the interpreter mishandles bf16 tensors), and ``tests/golden/make_topk_golden.py``
runs the reference ``topk.cu`` compiled for sm_100a (``oracle/build_ref.py``)
on a B200.  ``tests/test_oracle_golden.py`` checks this module against both.

Ordering contract of the selection (topk.cu:182-350): scores are compared as
their raw uint32 bit patterns, largest first, ties to the lowest column id, and
the chosen ids are emitted in ascending id order.  ``-0.0`` (0x80000000)
therefore ranks above every positive score, exactly as in the reference.
NaN scores carrying the sign bit are outside the contract (the reference's
fp16 coarse binning is not monotone for them).
"""

from __future__ import annotations

import numpy as np
import torch

LOG2E = 1.4426950408889634


# --------------------------------------------------------------------------
# 1. visible blocks  (ops/indexer.py:363-369)
# --------------------------------------------------------------------------
def visible_blocks(positions: torch.Tensor, sequence_lengths: torch.Tensor,
                   token_to_req: torch.Tensor, ratio: int) -> torch.Tensor:
    """Number of complete compressed blocks each query row may see."""
    safe = token_to_req.clamp_min(0).long()
    vis = torch.minimum(
        (positions.long() + 1) // ratio,
        sequence_lengths.long().index_select(0, safe) // ratio,
    ).to(torch.int32)
    return torch.where(token_to_req >= 0, vis, torch.zeros_like(vis))


# --------------------------------------------------------------------------
# 2. indexer scores  (ops/indexer.py:24-114, 117-223)
# --------------------------------------------------------------------------
def _row_requests(rows: int, decode_query_len: int | None,
                  query_start_loc: torch.Tensor | None) -> np.ndarray:
    if query_start_loc is None:
        return np.arange(rows) // int(decode_query_len or 1)
    qsl = query_start_loc.cpu().numpy().astype(np.int64)
    qsl = qsl - qsl[0]
    req = np.full(rows, -1, dtype=np.int64)
    for r in range(len(qsl) - 1):
        req[qsl[r]:min(qsl[r + 1], rows)] = r
    return req


def indexer_scores(q: torch.Tensor, k_cache: torch.Tensor, page_table: torch.Tensor,
                   visible: torch.Tensor, columns: int, *,
                   decode_query_len: int | None = 1,
                   query_start_loc: torch.Tensor | None = None,
                   weights: torch.Tensor | None = None,
                   scale: float | None = None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """logits[r, c] = scale * sum_h w[r,h] * relu(q[r,h] . key(c)) for c < visible[r].

    ``k_cache`` is ``[num_blocks, page, (1,) dim]``; key(c) lives in
    ``k_cache[page_table[req, c // page], c % page]``.  Columns at or beyond
    ``min(visible[r], page_table_width * page, columns)`` are left as they were
    in ``out`` (the reference leaves the workspace untouched there).
    A physical page outside ``[0, num_blocks)`` contributes a zero key (the
    reference reads out of bounds there; such metadata is invalid).
    Reference weights are all ones and scale is ``dim ** -0.5``
    (ops/indexer.py:107, :213).
    """
    q = q.float().cpu()
    rows, heads, dim = q.shape
    kc = k_cache.cpu()
    kc = kc.reshape(kc.shape[0], kc.shape[1], -1)[..., :dim]
    nblk, page = kc.shape[0], kc.shape[1]
    table = page_table.cpu().long()
    width = table.shape[1]
    num_columns = width * page
    vis = visible.cpu().long()
    if scale is None:
        scale = float(np.float32(dim ** -0.5))
    if weights is None:
        w = torch.ones(rows, heads)
    else:
        w = weights.float().cpu().expand(rows, heads)
    if out is None:
        out = torch.full((rows, columns), float("nan"))
    req_of = _row_requests(rows, decode_query_len, query_start_loc)
    for r in range(rows):
        req = int(req_of[r])
        n = min(int(vis[r]), num_columns, columns)
        if req < 0 or n <= 0:
            continue
        cols = torch.arange(n)
        phys = table[req, cols // page]
        ok = (phys >= 0) & (phys < nblk)
        keys = torch.zeros(n, dim)
        keys[ok] = kc[phys[ok], (cols % page)[ok]].float()
        s = keys @ q[r].T                                   # [n, heads] fp32
        s = torch.clamp_min(s, 0.0) * w[r][None, :]
        out[r, :n] = (s.sum(dim=1) * np.float32(scale)).to(out.dtype)
    return out


# --------------------------------------------------------------------------
# 3. top-k selection + expansion  (ops/csrc/topk.cu)
# --------------------------------------------------------------------------
def float_bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)


def select_blocks(row_scores: np.ndarray, length: int, topk: int) -> np.ndarray:
    """Exact top-k column ids of one row in ascending id order (topk.cu:182-350).

    Returns ``topk`` entries; when ``length <= topk`` these are ``0..length-1``
    followed by ``-1`` (topk.cu:187-191), irrespective of the scores.
    """
    out = np.full(topk, -1, dtype=np.int64)
    if length <= topk:
        n = max(length, 0)
        out[:n] = np.arange(n)
        return out
    keys = float_bits(row_scores[:length]).astype(np.int64)
    order = np.argsort(-keys, kind="stable")[:topk]     # key desc, id asc
    out[:] = np.sort(order)
    return out


def _div(a: int, b: int) -> int:
    """C integer division (truncates toward zero), as in topk.cu."""
    q = abs(a) // abs(b)
    return q if (a >= 0) == (b >= 0) else -q


def topk_expand(scores: torch.Tensor, lengths: torch.Tensor, positions: torch.Tensor,
                sequence_lengths: torch.Tensor, token_to_req: torch.Tensor,
                table: torch.Tensor | None, output_width: int, ratio: int,
                page_size: int = 1) -> tuple[np.ndarray, np.ndarray]:
    """Selection + expansion of ``yulan_qsa_kernels::topk_expand``.

    Returns ``(output[rows, output_width] int32, counts[rows] int32)``.
    ``table`` given means physical output (slot = page_id * page + offset),
    as ``physical=True`` in topk.cu:503-525.  ``lengths[r]`` beyond the score
    row width is clamped to the width (the reference would read past the row).
    """
    sc = scores.float().cpu().numpy()
    rows, width = sc.shape
    lens = lengths.cpu().numpy().astype(np.int64)
    pos = positions.cpu().numpy().astype(np.int64)
    seqs = sequence_lengths.cpu().numpy().astype(np.int64)
    t2r = token_to_req.cpu().numpy().astype(np.int64)
    tab = table.cpu().numpy().astype(np.int64) if table is not None else None
    num_requests = len(seqs)
    topk = output_width // ratio
    output = np.full((rows, output_width), -1, dtype=np.int32)
    counts = np.zeros(rows, dtype=np.int32)
    for r in range(rows):
        req = int(t2r[r])
        mapped = 0 <= req < num_requests
        seq = int(seqs[req]) if mapped else 0
        p = int(pos[r])
        complete = min(min(_div(p + 1, ratio), _div(seq, ratio)), topk)
        tail_start = _div(p + 1, ratio) * ratio
        tail_count = p + 1 - tail_start
        trow = tab[req if mapped else 0] if tab is not None else None

        def map_tokens(tok: np.ndarray) -> np.ndarray:
            ok = (tok >= 0) & (tok < seq)
            if trow is None:
                return np.where(ok, tok, -1)
            lp = np.where(ok, tok, 0) // page_size
            ok &= lp < trow.shape[0]
            phys = trow[np.minimum(lp, trow.shape[0] - 1)]
            ok &= phys >= 0
            return np.where(ok, phys * page_size + np.where(ok, tok, 0) % page_size, -1)

        length = min(int(lens[r]), width)
        blocks = select_blocks(sc[r], length, topk)
        nc = max(complete, 0)
        if nc:
            tok = blocks[:nc, None] * ratio + np.arange(ratio)[None, :]
            tok = np.where(blocks[:nc, None] >= 0, tok, -1).reshape(-1)
            output[r, :nc * ratio] = map_tokens(tok)
        expanded = complete * ratio
        cols = np.arange(max(expanded, 0), output_width)
        off = cols - expanded
        tail_ok = (off < tail_count) & (off < ratio - 1)
        output[r, cols] = np.where(tail_ok, map_tokens(np.where(tail_ok, tail_start + off, -1)), -1)
        counts[r] = min(expanded + tail_count, seq)
    return output, counts


def topk_plain(scores: torch.Tensor, lengths: torch.Tensor, topk: int) -> np.ndarray:
    """``yulan_qsa_kernels::topk`` (topk.cu:362-371, 527-545): ids only."""
    sc = scores.float().cpu().numpy()
    lens = lengths.cpu().numpy().astype(np.int64)
    out = np.full((sc.shape[0], topk), -1, dtype=np.int32)
    for r in range(sc.shape[0]):
        out[r] = select_blocks(sc[r], min(int(lens[r]), sc.shape[1]), topk)
    return out


# --------------------------------------------------------------------------
# 4. expansion of given block ids  (ops/qsa.py:18-106)
# --------------------------------------------------------------------------
def expand_block_indices(block_indices: np.ndarray, positions, sequence_lengths,
                         token_to_req, ratio: int, token_topk: int,
                         main_block_table=None, main_page_size: int = 1):
    """Expansion rules of ``_expand_qsa_indices_kernel`` (dead code upstream,
    same semantics as the topk.cu writer).  Returns (output, counts)."""
    bi = np.asarray(block_indices, dtype=np.int64)
    pos = np.asarray(positions, dtype=np.int64)
    seqs = np.asarray(sequence_lengths, dtype=np.int64)
    t2r = np.asarray(token_to_req, dtype=np.int64)
    tab = None if main_block_table is None else np.asarray(main_block_table, dtype=np.int64)
    rows = bi.shape[0]
    block_topk = token_topk // ratio
    width = token_topk + ratio - 1
    out = np.full((rows, width), -1, dtype=np.int32)
    counts = np.zeros(rows, dtype=np.int32)
    for r in range(rows):
        req = int(t2r[r])
        mapped = 0 <= req < len(seqs)
        seq = int(seqs[req]) if mapped else 0
        p = int(pos[r])
        complete = min((p + 1) // ratio, seq // ratio, block_topk)
        expanded = complete * ratio
        tail_start = ((p + 1) // ratio) * ratio
        tail_count = p + 1 - tail_start
        counts[r] = min(expanded + tail_count, seq) if mapped else 0
        safe_req = min(max(req, 0), len(seqs) - 1)
        for c in range(width):
            if c < expanded:
                token = int(bi[r, min(c // ratio, block_topk - 1)]) * ratio + c % ratio
                ok = True
            else:
                off = c - expanded
                token = tail_start + off
                ok = off < tail_count and off < ratio - 1
            ok = ok and 0 <= token < seq
            if ok and tab is not None:
                lp = token // main_page_size
                phys = int(tab[safe_req, lp]) if lp < tab.shape[1] else -1
                ok = phys >= 0
                token = phys * main_page_size + token % main_page_size
            out[r, c] = token if ok else -1
    return out, counts


# --------------------------------------------------------------------------
# 5. sparse paged GQA attention  (ops/qsa.py:109-362, 594-688)
# --------------------------------------------------------------------------
def reference_launch_config(rows: int, num_q_heads: int, num_kv_heads: int,
                            topk_width: int, use_decode_kernel: bool,
                            decode_config=None) -> tuple[int, int]:
    """(BLOCK_N, NUM_SPLITS) chosen by qsa_sparse_paged_attention (ops/qsa.py:617-645)."""
    group = num_q_heads // num_kv_heads
    base = rows * num_kv_heads
    if use_decode_kernel:
        if decode_config is not None:
            block_n, target = decode_config[0], decode_config[1]
        elif base <= 8:
            block_n, target = 32, 64
        elif base <= 32:
            block_n, target = 32, 16
        elif base <= 128:
            block_n, target = 32, 4
        else:
            block_n, target = 64, 1
    else:
        small = 8 if group <= 8 else 4
        if base <= small:
            block_n, target = 16, 32
        elif base < 32:
            block_n, target = 32, 16
        elif base <= 256:
            block_n, target = 64, 8
        elif base <= 512:
            block_n, target = 64, 4
        else:
            block_n, target = 64, 1
    tiles = -(-topk_width // block_n)
    max_useful = 1 << (tiles.bit_length() - 1)
    return block_n, min(max_useful, target)


def _bf16(x: torch.Tensor) -> torch.Tensor:
    return x.to(torch.bfloat16).float()


def sparse_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     indices: torch.Tensor, block_table: torch.Tensor,
                     token_to_req: torch.Tensor, *, output_gate: torch.Tensor | None = None,
                     use_decode_kernel: bool = False, indices_are_physical: bool = False,
                     valid_counts: torch.Tensor | None = None,
                     block_n: int | None = None, num_splits: int | None = None,
                     round_p: bool = True, round_out: bool = True,
                     return_partials: bool = False):
    """Restatement of the split-K paged GQA kernel plus merge.

    The tile schedule (BLOCK_N, NUM_SPLITS) defaults to the reference launch
    table, so the online-softmax rescaling points match the reference.
    ``round_p`` casts P to bf16 before P.V (ops/qsa.py:242-246); ``round_out``
    rounds the attention output to bf16 before the gate and at the store.
    Both are True for real bf16 runs; the interpreter golden vectors use fp32
    storage and are compared with both False.
    Returns fp32 [rows, H_q, d] holding the stored values (bf16-representable
    when ``round_out``); with ``return_partials`` also (partial_o, partial_lse)
    of shape [splits, rows, H_q, d] / [splits, rows, H_q].
    """
    qf = q.float().cpu()
    rows, hq, d = qf.shape
    kc = k_cache.cpu()   # gathered rows are converted to fp32 after the gather
    vc = v_cache.cpu()
    nblk, page, hkv = kc.shape[0], kc.shape[1], kc.shape[2]
    group = hq // hkv
    idx = indices.cpu().long()
    topk_width = idx.shape[1]
    table = block_table.cpu().long()
    t2r = token_to_req.cpu().long()
    num_requests = table.shape[0]
    width = table.shape[1]
    if block_n is None or num_splits is None:
        bn, ns = reference_launch_config(rows, hq, hkv, topk_width, use_decode_kernel)
        block_n = block_n or bn
        num_splits = num_splits or ns
    scale_log2 = np.float32((d ** -0.5) * LOG2E)

    # Resolve every (row, column) to a physical (page, offset) and validity.
    safe_tok = idx.clamp_min(0)
    lpage = safe_tok // page
    off = safe_tok % page
    if indices_are_physical:
        phys = lpage
        valid = (idx >= 0) & (phys < nblk)
    else:
        req_ok = (t2r >= 0) & (t2r < num_requests)
        safe_req = t2r.clamp(0, num_requests - 1)
        valid = req_ok[:, None] & (idx >= 0) & (lpage < width)
        phys = table[safe_req[:, None], lpage.clamp_max(width - 1)]
        phys = torch.where(valid, phys, torch.full_like(phys, -1))
        valid &= (phys >= 0) & (phys < nblk)
    phys_safe = phys.clamp(0, nblk - 1)

    if valid_counts is not None:
        vc_rows = valid_counts.cpu().long().clamp(max=topk_width)
        row_tiles = -(-vc_rows // block_n)
    else:
        row_tiles = torch.full((rows,), -(-topk_width // block_n), dtype=torch.long)

    part_o = torch.zeros(num_splits, rows, hq, d)
    part_lse = torch.full((num_splits, rows, hq), float("-inf"))
    for s in range(num_splits):
        t_lo = s * row_tiles // num_splits
        t_hi = (s + 1) * row_tiles // num_splits
        m = torch.full((rows, hkv, group), -1.0e20)
        l = torch.zeros(rows, hkv, group)
        acc = torch.zeros(rows, hkv, group, d)
        max_t = int(t_hi.max()) if rows else 0
        for t in range(int(t_lo.min()) if rows else 0, max_t):
            active = (t >= t_lo) & (t < t_hi)                 # [rows]
            if not bool(active.any()):
                continue
            cols = torch.arange(t * block_n, (t + 1) * block_n)
            in_range = cols < topk_width
            cc = cols.clamp_max(topk_width - 1)
            v_ok = valid[:, cc] & in_range[None, :]              # [rows, bn]
            pg = phys_safe[:, cc]
            of = off[:, cc]
            K = kc[pg, of].float()                               # [rows, bn, hkv, d]
            V = vc[pg, of].float()
            K = torch.where(v_ok[..., None, None], K, torch.zeros(()))
            V = torch.where(v_ok[..., None, None], V, torch.zeros(()))
            qg = qf.view(rows, hkv, group, d)
            sc = torch.einsum("rgjd,rngd->rgjn", qg, K) * scale_log2   # [rows,hkv,group,bn]
            sc = torch.where(v_ok[:, None, None, :], sc, torch.full((), -1.0e20))
            nm = torch.maximum(m, sc.amax(dim=-1))
            alpha = torch.exp2(m - nm)
            p = torch.where(v_ok[:, None, None, :], torch.exp2(sc - nm[..., None]),
                            torch.zeros(()))
            pv = _bf16(p) if round_p else p
            a = active[:, None, None]
            acc = torch.where(a[..., None], acc * alpha[..., None]
                              + torch.einsum("rgjn,rngd->rgjd", pv, V), acc)
            l = torch.where(a, l * alpha + p.sum(dim=-1), l)
            m = torch.where(a, nm, m)
        has = l > 0
        o = torch.where(has[..., None], acc / l.clamp_min(1.0e-20)[..., None],
                        torch.zeros(()))
        part_o[s] = o.reshape(rows, hq, d)
        part_lse[s] = torch.where(has, m + torch.log2(l.clamp_min(1.0e-20)),
                                  torch.full((), float("-inf"))).reshape(rows, hq)

    if num_splits == 1:
        merged = part_o[0]
    else:
        lse_max = part_lse.amax(dim=0)
        hv = lse_max > float("-inf")
        shifted = torch.where(hv[None], part_lse - lse_max[None],
                              torch.full((), float("-inf")))
        w = torch.exp2(shifted)
        den = w.sum(dim=0)
        merged = (part_o * w[..., None]).sum(dim=0)
        merged = torch.where((den > 0)[..., None], merged / den.clamp_min(1e-38)[..., None],
                             torch.zeros(()))
    if output_gate is not None:
        g = output_gate.float().cpu()
        base = _bf16(merged) if round_out else merged
        merged = base * torch.sigmoid(g)
    out = _bf16(merged) if round_out else merged
    if return_partials:
        return out, part_o, part_lse
    return out


# --------------------------------------------------------------------------
# whole decode step (indexer -> top-k -> attention), used as the CPU baseline
# --------------------------------------------------------------------------
def decode_step(w, *, round_p: bool = True):
    """One QSA decode step on CPU tensors of a ``SyntheticQSA`` workload ``w``.

    Returns (attention_out fp32 [rows, H_q, d], topk_indices, counts, logits).
    """
    vis = visible_blocks(w.positions, w.seq_lens, w.token_to_req, w.ratio)
    columns = w.index_table.shape[1] * w.index_cache.shape[1]
    logits = indexer_scores(w.index_q, w.index_cache, w.index_table, vis, columns,
                            decode_query_len=getattr(w, "decode_query_len", 1),
                            weights=w.index_weights,
                            scale=w.index_scale)
    idx, counts = topk_expand(logits, vis, w.positions, w.seq_lens, w.token_to_req,
                              w.block_table, w.token_topk + w.ratio - 1, w.ratio,
                              page_size=w.page_size)
    out = sparse_attention(w.q, w.k_cache, w.v_cache, torch.from_numpy(idx),
                           w.block_table, w.token_to_req, output_gate=w.gate,
                           use_decode_kernel=True, indices_are_physical=True,
                           valid_counts=torch.from_numpy(counts), round_p=round_p)
    return out, idx, counts, logits


def prefill_step(w, *, round_p: bool = True):
    """One QSA chunked-prefill step on CPU tensors of a ``SyntheticQSA``
    workload ``w``: scores over each row's causal visible blocks
    (ops/indexer.py:282-343, logits width as :262-263), top-k expanded to
    logical token ids (no block table), attention through the request's block
    table (ops/qsa.py:594-688 with use_decode_kernel=False).

    Returns (attention_out fp32 [rows, H_q, d], topk_indices, counts, logits).
    """
    vis = visible_blocks(w.positions, w.seq_lens, w.token_to_req, w.ratio)
    columns = -(-(-(-int(w.max_seq_len) // w.ratio)) // 64) * 64
    logits = indexer_scores(w.index_q, w.index_cache, w.index_table, vis, columns,
                            query_start_loc=w.query_start_loc, weights=w.index_weights,
                            scale=w.index_scale)
    idx, counts = topk_expand(logits, vis, w.positions, w.seq_lens, w.token_to_req, None,
                              w.token_topk + w.ratio - 1, w.ratio)
    out = sparse_attention(w.q, w.k_cache, w.v_cache, torch.from_numpy(idx), w.block_table,
                           w.token_to_req, output_gate=w.gate, round_p=round_p)
    return out, idx, counts, logits


def _bf16_trunc(x: torch.Tensor) -> torch.Tensor:
    """fp32 -> bf16 rounding toward zero (low 16 bits cleared), returned as fp32."""
    return (x.float().contiguous().view(torch.int32) & -65536).view(torch.float32)


def norm_rope(x: torch.Tensor, positions: torch.Tensor, gamma: torch.Tensor,
              cos_sin: torch.Tensor, eps: float, rotary: int, *,
              rounding: str = "nearest") -> torch.Tensor:
    """RMSNorm + rotate-half RoPE over the first ``rotary`` dims with the
    reference's bf16 rounding after every post-norm step (ops/prepare.py:16-46).

    x: [n, dim] (bf16 values); positions: [n]; gamma: [dim]; cos_sin:
    [max_pos, rotary] with cosines in the first half, sines in the second.
    Returns fp32 holding bf16 values.  ``rounding``: "nearest" (the GPU's
    round-to-nearest-even conversion) or "truncate" (the Triton CPU
    interpreter's conversion, for checking against interpreter fixtures).
    """
    _bf16r = _bf16 if rounding == "nearest" else _bf16_trunc
    x = x.float()
    dim = x.shape[1]
    inv_rms = torch.rsqrt((x * x).sum(dim=1) / dim + eps)
    normalized = _bf16r(x * inv_rms[:, None])
    scaled = _bf16r(normalized * gamma.float()[None, :])
    half = rotary // 2
    dims = torch.arange(dim)
    partner_dims = torch.where(dims < half, dims + half, dims - half).clamp(max=dim - 1)
    partner = scaled[:, partner_dims]
    rotated = _bf16r(torch.where(dims[None, :] < half, -partner, partner))
    channel = dims % max(half, 1)
    in_rot = dims < rotary
    pos = positions.long()
    cs = cos_sin.float()
    cosine = torch.where(in_rot[None, :], cs[pos][:, channel.clamp(max=rotary - 1)],
                         torch.zeros(()))
    sine = torch.where(in_rot[None, :], cs[pos][:, (half + channel).clamp(max=rotary - 1)],
                       torch.zeros(()))
    first = _bf16r(scaled * cosine)
    second = _bf16r(rotated * sine)
    combined = _bf16r(first + second)
    return torch.where(in_rot[None, :], combined, scaled)


def qsa_prepare(index_qk: torch.Tensor, positions: torch.Tensor, q_weight: torch.Tensor,
                k_weight: torch.Tensor, cos_sin: torch.Tensor, eps: float,
                state_cache: torch.Tensor, state_slots: torch.Tensor,
                state_table: torch.Tensor, query_start_loc: torch.Tensor,
                logical_positions: torch.Tensor, compressed_cache: torch.Tensor,
                compressed_slots: torch.Tensor, k_work: torch.Tensor,
                main_key: torch.Tensor, main_value: torch.Tensor,
                main_key_cache: torch.Tensor, main_value_cache: torch.Tensor,
                main_slots: torch.Tensor, *, num_index_heads: int, index_head_dim: int,
                rotary_dim: int, compress_ratio: int,
                rounding: str = "nearest") -> torch.Tensor:
    """The reference's one-launch indexer preparation (ops/prepare.py:49-228),
    updating the four caches in place and returning the index queries.

    * index queries (:99-118): RMSNorm + RoPE of each head's row of
      ``index_qk`` at the token's position, with ``q_weight``;
    * key compression (:120-152): per (request, work item) of ``k_work``, the
      mean of ``compress_ratio`` raw keys ending at the group boundary (from this
      chunk's ``index_qk`` key part, or from the request's ring ``state_cache``
      for positions before the chunk), rounded to bf16, then RMSNorm + RoPE at
      the group's first position with ``k_weight``, stored at the boundary
      token's compressed slot;
    * ring commit (:154-166): work item 0 of a request writes the chunk's last
      ``min(query_len, state_size)`` raw keys to their state slots, after its
      own group has read the ring;
    * main K/V (:81-97): each token's key / value rows to ``main_slots``.
    Slots < 0 are skipped.  Tensors hold bf16 values (fp32 or bf16 storage).
    ``rounding`` as in ``norm_rope``.
    """
    H, D, R = num_index_heads, index_head_dim, compress_ratio
    tokens = index_qk.shape[0]
    qk = index_qk.float()
    state_size = state_cache.shape[1]
    comp_page = compressed_cache.shape[1]
    # index queries
    rows = qk[:, :H * D].reshape(tokens * H, D)
    pos_rows = positions.long().repeat_interleave(H)
    query = norm_rope(rows, pos_rows, q_weight, cos_sin, eps, rotary_dim,
                      rounding=rounding).reshape(tokens, H, D)
    _bf16r = _bf16 if rounding == "nearest" else _bf16_trunc
    # key compression + ring commit, work item by work item (item 0 first
    # within a request: its group reads the ring before the commit)
    key_part = qk[:, H * D:H * D + D]
    for request, work in k_work.tolist():
        if request < 0:
            continue
        q0, q1 = int(query_start_loc[request]), int(query_start_loc[request + 1])
        qlen = q1 - q0
        chunk_end = int(logical_positions[q1 - 1])
        chunk_start = chunk_end - qlen + 1
        groups = (chunk_end + 1) // R - chunk_start // R
        if work < groups:
            first_boundary = ((chunk_start + R) // R) * R - 1
            end = first_boundary + work * R
            boundary_token = q0 + end - chunk_start
            block = int(state_table[request, 0])
            acc = torch.zeros(D)
            for m in range(R):
                src = end - (R - 1) + m
                if src >= chunk_start:
                    acc = acc + key_part[q0 + src - chunk_start]
                else:
                    acc = acc + state_cache[block, src % state_size].float()
            pooled = _bf16r(acc / R)
            comp = norm_rope(pooled[None, :], torch.tensor([end - (R - 1)]), k_weight,
                             cos_sin, eps, rotary_dim, rounding=rounding)[0]
            cslot = int(compressed_slots[boundary_token])
            if cslot >= 0:
                compressed_cache[cslot // comp_page, cslot % comp_page] = \
                    comp.to(compressed_cache.dtype)
        if work == 0:
            suffix = min(qlen, state_size)
            for t in range(q1 - suffix, q1):
                slot = int(state_slots[t])
                if slot >= 0:
                    state_cache[slot // state_size, slot % state_size] = \
                        key_part[t].to(state_cache.dtype)
    # main K/V
    main_page = main_key_cache.shape[1]
    for t in range(tokens):
        slot = int(main_slots[t])
        if slot >= 0:
            main_key_cache[slot // main_page, slot % main_page] = main_key[t]
            main_value_cache[slot // main_page, slot % main_page] = main_value[t]
    return query


__all__ = [
    "norm_rope", "qsa_prepare",
    "visible_blocks", "indexer_scores", "select_blocks", "topk_expand", "topk_plain",
    "expand_block_indices", "reference_launch_config", "sparse_attention",
    "decode_step", "float_bits", "LOG2E",
]
