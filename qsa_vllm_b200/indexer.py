"""Indexer scoring + fused top-k selection (drop-in for the reference ops/indexer.py).

Host logic mirrors the reference (ops/indexer.py:227-393): decode rows are
scored against the column bucket chosen by ``graph_dispatch`` and prefill rows
against ``round64(ceil(max_seq_len / ratio))`` columns, both through an fp32
logits workspace chunked by ``QSA_INDEXER_WORKSPACE_MB`` (default 64 MiB),
each chunk followed by the top-k/expansion op.  The scoring itself is the
sm_100a ``qsa_indexer_scores`` kernel; selection is ``topk_expand``.

Two optional keyword arguments extend the reference signature: ``weights``
(fp32 per-row head weights, ``[rows, heads]``, broadcastable) and ``scale``
(default ``head_dim ** -0.5``).  Without them the math is the reference's
(unit head weights, ops/indexer.py:107,213).
"""

from __future__ import annotations

import os

import numpy as np
import torch

from . import _lib
from .graph_dispatch import decode_logits_columns
from .topk import topk_expand as _topk_expand
from .topk import topk_expand_visible as _topk_expand_visible

_INDEXER_WORKSPACE_BYTES = int(os.environ.get("QSA_INDEXER_WORKSPACE_MB", "64")) * 1024 * 1024


def _cdiv(a: int, b: int) -> int:
    return -(-a // b)


def indexer_scores(q: torch.Tensor, k_cache: torch.Tensor, page_table: torch.Tensor,
                   visible: torch.Tensor, logits: torch.Tensor, *,
                   decode_query_len: int = 1, query_start_loc: torch.Tensor | None = None,
                   max_query_len: int = 0, query_offset: int = 0, num_rows: int | None = None,
                   weights: torch.Tensor | None = None, scale: float | None = None,
                   query_positions: torch.Tensor | None = None,
                   sequence_lengths: torch.Tensor | None = None,
                   token_to_req: torch.Tensor | None = None, compress_ratio: int = 0) -> None:
    """Write ``logits[r - query_offset, c]`` for the packed rows of this call.

    Decode (``query_start_loc is None``): ``q`` holds ``requests * decode_query_len``
    rows and ``page_table`` one row per request.  Prefill: ``q``/``visible`` are
    the full packed tensors indexed by absolute row, the call covers rows
    ``[query_offset, query_offset + num_rows)`` (as ``_prefill_logits``,
    ops/indexer.py:282-302).  With ``visible=None`` the kernel derives each
    row's count from ``query_positions`` / ``sequence_lengths`` /
    ``token_to_req`` (indexed like ``visible``) and ``compress_ratio``.
    """
    rows = q.shape[0] if num_rows is None else num_rows
    if rows == 0:
        return
    _lib.ensure_device(q.device)
    if q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16:
        raise TypeError("indexer q and key cache must be bfloat16")
    if logits.dtype != torch.float32 or logits.stride(-1) != 1:
        raise TypeError("logits must be float32 with unit column stride")
    if page_table.dtype != torch.int32 or (visible is not None and visible.dtype != torch.int32):
        raise TypeError("page_table and visible must be int32")
    if visible is None:
        if query_positions is None or sequence_lengths is None or token_to_req is None \
                or compress_ratio <= 0:
            raise ValueError("visible=None needs query_positions, sequence_lengths, "
                             "token_to_req and compress_ratio")
        if query_positions.dtype != torch.int64 or sequence_lengths.dtype != torch.int32 \
                or token_to_req.dtype != torch.int32:
            raise TypeError("positions int64, sequence_lengths / token_to_req int32 expected")
    if q.stride(-1) != 1 or k_cache.stride(-1) != 1:
        raise ValueError("q and k_cache need a unit head-dim stride")
    w_ptr, w_rs, w_hs = None, 0, 0
    if weights is not None:
        if weights.dtype != torch.float32:
            raise TypeError("weights must be float32")
        w = weights.expand(q.shape[0], q.shape[1])
        w_ptr, w_rs, w_hs = w.data_ptr(), w.stride(0), w.stride(1)
    dim = q.shape[2]
    if scale is None:
        scale = float(np.float32(dim ** -0.5))
    qsl = query_start_loc
    if qsl is not None and qsl.dtype != torch.int32:
        raise TypeError("query_start_loc must be int32")
    lib = _lib.load_library()
    with torch.cuda.device(q.device):
        _lib.check(lib.qsa_indexer_scores(
            q.data_ptr(), q.stride(0), q.stride(1), q.shape[1], dim,
            k_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.shape[0],
            k_cache.shape[1], page_table.data_ptr(), page_table.stride(0), page_table.shape[1],
            page_table.shape[0] if qsl is None else qsl.numel() - 1,
            None if visible is None else visible.data_ptr(),
            None if visible is not None else query_positions.data_ptr(),
            None if visible is not None else sequence_lengths.data_ptr(),
            0 if visible is not None else sequence_lengths.numel(),
            None if visible is not None else token_to_req.data_ptr(),
            0 if visible is not None else int(compress_ratio),
            None if qsl is None else qsl.data_ptr(),
            int(decode_query_len), int(max_query_len), int(query_offset), int(rows),
            w_ptr, w_rs, w_hs, float(scale), logits.data_ptr(), logits.stride(0),
            logits.shape[1], _lib.stream_ptr(q.device)), "indexer_scores")


def compute_visible_blocks(query_positions: torch.Tensor, sequence_lengths: torch.Tensor,
                           token_to_req: torch.Tensor, compress_ratio: int) -> torch.Tensor:
    """min((pos + 1) // ratio, seq_len // ratio) per row, 0 for unmapped rows
    (ops/indexer.py:363-369), in one sm_100a launch."""
    rows = token_to_req.shape[0]
    out = torch.empty(rows, dtype=torch.int32, device=token_to_req.device)
    if rows == 0:
        return out
    _lib.ensure_device(token_to_req.device)
    if query_positions.dtype != torch.int64 or sequence_lengths.dtype != torch.int32 \
            or token_to_req.dtype != torch.int32:
        raise TypeError("positions int64, sequence_lengths / token_to_req int32 expected")
    lib = _lib.load_library()
    with torch.cuda.device(token_to_req.device):
        _lib.check(lib.qsa_visible_blocks(
            query_positions.data_ptr(), sequence_lengths.data_ptr(), sequence_lengths.numel(),
            token_to_req.data_ptr(), rows, int(compress_ratio), out.data_ptr(),
            _lib.stream_ptr(token_to_req.device)), "visible_blocks")
    return out


_QSA_ERR_UNSUPPORTED = 2


def select_decode_fused(q, k_cache, page_table, visible_blocks, compress_ratio, decode_query_len,
                        out, columns, *, query_positions, sequence_lengths, token_to_req,
                        main_block_table=None, main_page_size=1, valid_counts_out=None,
                        weights=None, scale=None, scores_out=None) -> bool:
    """Scores, top-k and expansion of decode rows in one launch (``qsa_select_decode``).

    Same results as ``indexer_scores`` over ``columns`` logits followed by
    ``topk_expand`` (bit for bit), without the fp32 logits round trip.
    ``visible_blocks=None`` derives each row's count in the kernel.  Returns
    False, having launched nothing, for shapes outside the fused kernel's
    range; other failures raise ``QSAError``.  ``scores_out`` (optional fp32
    ``[rows, columns]``) receives the scores as well.
    """
    rows = q.shape[0]
    if rows == 0:
        return True
    _lib.ensure_device(q.device)
    if q.dtype != torch.bfloat16 or k_cache.dtype != torch.bfloat16:
        raise TypeError("indexer q and key cache must be bfloat16")
    if page_table.dtype != torch.int32 or out.dtype != torch.int32:
        raise TypeError("page_table and out must be int32")
    if visible_blocks is not None and visible_blocks.dtype != torch.int32:
        raise TypeError("visible_blocks must be int32")
    if query_positions.dtype != torch.int64 or sequence_lengths.dtype != torch.int32 \
            or token_to_req.dtype != torch.int32:
        raise TypeError("positions int64, sequence_lengths / token_to_req int32 expected")
    if q.stride(-1) != 1 or k_cache.stride(-1) != 1:
        raise ValueError("q and k_cache need a unit head-dim stride")
    w_ptr, w_rs, w_hs = None, 0, 0
    if weights is not None:
        if weights.dtype != torch.float32:
            raise TypeError("weights must be float32")
        w = weights.expand(q.shape[0], q.shape[1])
        w_ptr, w_rs, w_hs = w.data_ptr(), w.stride(0), w.stride(1)
    dim = q.shape[2]
    if scale is None:
        scale = float(np.float32(dim ** -0.5))
    physical = main_block_table is not None
    if physical and main_block_table.dtype != torch.int32:
        raise TypeError("main_block_table must be int32")
    if valid_counts_out is not None and valid_counts_out.dtype != torch.int32:
        raise TypeError("valid_counts_out must be int32")
    if scores_out is not None and (scores_out.dtype != torch.float32
                                   or scores_out.stride(-1) != 1):
        raise TypeError("scores_out must be float32 with unit column stride")
    lib = _lib.load_library()
    with torch.cuda.device(q.device):
        status = lib.qsa_select_decode(
            q.data_ptr(), q.stride(0), q.stride(1), q.shape[1], dim,
            k_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.shape[0],
            k_cache.shape[1], page_table.data_ptr(), page_table.stride(0), page_table.shape[1],
            page_table.shape[0], _lib.ptr(visible_blocks), query_positions.data_ptr(),
            sequence_lengths.data_ptr(), sequence_lengths.numel(), token_to_req.data_ptr(),
            int(compress_ratio), int(decode_query_len), rows, w_ptr, w_rs, w_hs, float(scale),
            int(columns),
            main_block_table.data_ptr() if physical else None,
            main_block_table.stride(0) if physical else 0,
            main_block_table.shape[1] if physical else 0, int(main_page_size), int(physical),
            out.data_ptr(), out.stride(0), out.stride(1), out.shape[1],
            _lib.ptr(valid_counts_out), _lib.ptr(scores_out),
            scores_out.stride(0) if scores_out is not None else 0,
            _lib.stream_ptr(q.device))
    if status == _QSA_ERR_UNSUPPORTED:
        return False
    _lib.check(status, "select_decode")
    return True


def qsa_select_paged_decode(q, k_cache, page_table, visible_blocks, token_topk, compress_ratio,
                            decode_query_len, out, max_seq_len, *, query_positions,
                            sequence_lengths, token_to_req, main_block_table=None,
                            main_page_size=1, valid_counts_out=None, weights=None, scale=None):
    """Score decode queries and write the expanded selection (ops/indexer.py:227-279).

    The reference's structure: scoring into fp32 logits chunks, each followed
    by ``topk_expand``.  (``select_decode_fused`` does both in one launch with
    identical results; on B200 it measures slower at the benchmark shapes,
    because its selection phase is latency-bound on the scoring CTAs, so it
    is not the default.)
    """
    num_requests = q.shape[0] // decode_query_len
    columns = decode_logits_columns(max_seq_len, compress_ratio,
                                    page_table.shape[1] * k_cache.shape[1])
    if visible_blocks is None:
        # one small launch: its counts stay in L2 for both the indexer and the top-k
        visible_blocks = compute_visible_blocks(query_positions, sequence_lengths, token_to_req,
                                                compress_ratio)
    requests_per_chunk = max(1, _INDEXER_WORKSPACE_BYTES // (columns * 4 * decode_query_len))
    workspace_rows = min(num_requests, requests_per_chunk) * decode_query_len
    logits_workspace = torch.empty((workspace_rows, columns), dtype=torch.float32,
                                   device=q.device)
    for first in range(0, num_requests, requests_per_chunk):
        last = min(first + requests_per_chunk, num_requests)
        r0, r1 = first * decode_query_len, last * decode_query_len
        logits = logits_workspace[:r1 - r0]
        vis = None if visible_blocks is None else visible_blocks[r0:r1]
        indexer_scores(q[r0:r1], k_cache, page_table[first:last], vis, logits,
                       decode_query_len=decode_query_len,
                       weights=None if weights is None else weights[r0:r1], scale=scale,
                       query_positions=query_positions[r0:r1],
                       sequence_lengths=sequence_lengths, token_to_req=token_to_req[r0:r1],
                       compress_ratio=compress_ratio)
        select = dict(main_block_table=main_block_table, main_page_size=main_page_size,
                      valid_counts_out=(valid_counts_out[r0:r1]
                                        if valid_counts_out is not None else None))
        if vis is None:
            _topk_expand_visible(logits, query_positions[r0:r1], sequence_lengths,
                                 token_to_req[r0:r1], out[r0:r1], compress_ratio, **select)
        else:
            _topk_expand(logits, vis, query_positions[r0:r1], sequence_lengths,
                         token_to_req[r0:r1], out[r0:r1], compress_ratio, **select)


def _prefill_logits(q, k_cache, page_table, query_start_loc, visible_blocks, logits_workspace,
                    max_query_len, logits_width, query_offset, num_queries, *, weights=None,
                    scale=None, query_positions=None, sequence_lengths=None, token_to_req=None,
                    compress_ratio=0):
    """Score packed prefill rows [query_offset, query_offset+num_queries) (ops/indexer.py:282-302)."""
    logits = logits_workspace[:num_queries * logits_width].view(num_queries, logits_width)
    indexer_scores(q, k_cache, page_table, visible_blocks, logits,
                   query_start_loc=query_start_loc, max_query_len=max_query_len,
                   query_offset=query_offset, num_rows=num_queries, weights=weights, scale=scale,
                   query_positions=query_positions, sequence_lengths=sequence_lengths,
                   token_to_req=token_to_req, compress_ratio=compress_ratio)
    return logits


def qsa_select_paged_prefill(q, k_cache, page_table, query_start_loc, visible_blocks, token_topk,
                             compress_ratio, max_query_len, out, max_seq_len, *, query_positions,
                             sequence_lengths, token_to_req, main_block_table=None,
                             main_page_size=1, valid_counts_out=None, weights=None, scale=None):
    """Packed prefill scoring and fused selection write-out (ops/indexer.py:305-343)."""
    rows = q.shape[0]
    columns = page_table.shape[1] * k_cache.shape[1]
    logits_width = _cdiv(_cdiv(max_seq_len, compress_ratio), 64) * 64
    logits_width = min(max(64, logits_width), columns)
    rows_per_chunk = max(1, _INDEXER_WORKSPACE_BYTES // (logits_width * 4))
    logits_workspace = torch.empty(min(rows, rows_per_chunk) * logits_width,
                                   dtype=torch.float32, device=q.device)
    for start in range(0, rows, rows_per_chunk):
        end = min(start + rows_per_chunk, rows)
        logits = _prefill_logits(q, k_cache, page_table, query_start_loc, visible_blocks,
                                 logits_workspace, max_query_len, logits_width,
                                 query_offset=start, num_queries=end - start,
                                 weights=weights, scale=scale, query_positions=query_positions,
                                 sequence_lengths=sequence_lengths, token_to_req=token_to_req,
                                 compress_ratio=compress_ratio)
        select = dict(main_block_table=main_block_table, main_page_size=main_page_size,
                      valid_counts_out=(valid_counts_out[start:end]
                                        if valid_counts_out is not None else None))
        if visible_blocks is None:
            _topk_expand_visible(logits, query_positions[start:end], sequence_lengths,
                                 token_to_req[start:end], out[start:end], compress_ratio,
                                 **select)
        else:
            _topk_expand(logits, visible_blocks[start:end], query_positions[start:end],
                         sequence_lengths, token_to_req[start:end], out[start:end],
                         compress_ratio, **select)


def select_paged_tokens(q, k_cache, page_table, token_to_req, query_positions, sequence_lengths,
                        token_topk, compress_ratio, out=None, *, query_start_loc, max_query_len,
                        max_seq_len, num_decodes=0, num_decode_tokens=0, decode_query_len=1,
                        visible_blocks=None, main_block_table=None, main_page_size=1,
                        valid_counts_out=None, weights=None, scale=None):
    """Select blocks and write expanded decode/prefill tokens (ops/indexer.py:346-393).

    Decode rows come first (``[:num_decode_tokens]``, one page-table row per
    decode request), then packed prefill rows.
    """
    rows = q.shape[0]
    if out is None:
        out = torch.empty((rows, token_topk + compress_ratio - 1), dtype=torch.int32,
                          device=q.device)
    if not rows:
        return out
    # Without visible_blocks, each part computes its rows' counts in one small
    # launch, whose counts stay in L2 for both the indexer and the top-k.
    if num_decode_tokens:
        qsa_select_paged_decode(
            q[:num_decode_tokens], k_cache, page_table[:num_decodes],
            None if visible_blocks is None else visible_blocks[:num_decode_tokens], token_topk, compress_ratio, decode_query_len,
            out[:num_decode_tokens], max_seq_len,
            query_positions=query_positions[:num_decode_tokens],
            sequence_lengths=sequence_lengths, token_to_req=token_to_req[:num_decode_tokens],
            main_block_table=main_block_table, main_page_size=main_page_size,
            valid_counts_out=(valid_counts_out[:num_decode_tokens]
                              if valid_counts_out is not None else None),
            weights=None if weights is None else weights[:num_decode_tokens], scale=scale)
    if num_decode_tokens < rows:
        prefill_visible = (
            visible_blocks[num_decode_tokens:] if visible_blocks is not None
            else compute_visible_blocks(query_positions[num_decode_tokens:], sequence_lengths,
                                        token_to_req[num_decode_tokens:], compress_ratio))
        qsa_select_paged_prefill(
            q[num_decode_tokens:], k_cache, page_table[num_decodes:],
            query_start_loc[num_decodes:], prefill_visible, token_topk,
            compress_ratio, max_query_len, out[num_decode_tokens:], max_seq_len,
            query_positions=query_positions[num_decode_tokens:],
            sequence_lengths=sequence_lengths, token_to_req=token_to_req[num_decode_tokens:],
            main_block_table=main_block_table, main_page_size=main_page_size,
            valid_counts_out=(valid_counts_out[num_decode_tokens:]
                              if valid_counts_out is not None else None),
            weights=None if weights is None else weights[num_decode_tokens:], scale=scale)
    return out


__all__ = ["compute_visible_blocks", "indexer_scores", "qsa_select_paged_decode",
           "qsa_select_paged_prefill", "select_decode_fused", "select_paged_tokens"]
