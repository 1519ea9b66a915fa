"""Top-k selection operators: the ``yulan_qsa_kernels`` torch op library.

Drop-in for the reference's ``ops/topk.py`` (which JIT-builds ``topk.cu`` for
sm_80 only): registers the same op schemas (ops/csrc/topk.cu:548-557)

    yulan_qsa_kernels::topk(Tensor scores, Tensor lengths, Tensor(a!) output) -> ()
    yulan_qsa_kernels::topk_expand(Tensor scores, Tensor lengths, Tensor positions,
        Tensor sequence_lengths, Tensor token_to_req, Tensor table, Tensor(a!) output,
        Tensor(b!) counts, int ratio, int page_size, bool physical, bool store_counts) -> ()

with CUDA implementations that call the sm_100a C ABI (``qsa_topk`` /
``qsa_topk_expand``), and keeps the reference's Python wrappers ``topk`` and
``topk_expand`` (ops/topk.py:25-39) with the same arguments.
"""

from __future__ import annotations

import torch

from . import _lib

_NS = "yulan_qsa_kernels"


def _require(t: torch.Tensor, dtype: torch.dtype, name: str) -> None:
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")


def _topk_expand_impl(scores, lengths, positions, sequence_lengths, token_to_req, table,
                      output, counts, ratio, page_size, physical, store_counts) -> None:
    rows = scores.shape[0]
    if rows == 0:
        return
    _require(lengths, torch.int32, "lengths")
    _topk_expand_call(scores, lengths, positions, sequence_lengths, token_to_req, table,
                      output, counts, ratio, page_size, physical, store_counts)


def _topk_expand_call(scores, lengths, positions, sequence_lengths, token_to_req, table,
                      output, counts, ratio, page_size, physical, store_counts) -> None:
    """qsa_topk_expand; ``lengths=None`` lets the kernel derive each row's
    visible block count from positions / sequence_lengths / token_to_req."""
    rows = scores.shape[0]
    if rows == 0:
        return
    _lib.ensure_device(scores.device)
    _require(scores, torch.float32, "scores")
    _require(positions, torch.int64, "positions")
    _require(sequence_lengths, torch.int32, "sequence_lengths")
    _require(token_to_req, torch.int32, "token_to_req")
    _require(output, torch.int32, "output")
    if scores.stride(1) != 1:
        raise ValueError("scores must have unit column stride")
    if physical:
        _require(table, torch.int32, "table")
    if store_counts:
        _require(counts, torch.int32, "counts")
    lib = _lib.load_library()
    with torch.cuda.device(scores.device):
        _lib.check(lib.qsa_topk_expand(
            scores.data_ptr(), scores.stride(0), rows, scores.shape[1],
            None if lengths is None else lengths.data_ptr(), positions.data_ptr(),
            sequence_lengths.data_ptr(),
            sequence_lengths.numel(), token_to_req.data_ptr(),
            table.data_ptr() if physical else None,
            table.stride(0) if physical else 0, table.shape[1] if physical else 0,
            output.data_ptr(), output.stride(0), output.stride(1), output.shape[1],
            counts.data_ptr() if store_counts else None,
            int(ratio), int(page_size), 1 if physical else 0,
            _lib.stream_ptr(scores.device)), "topk_expand")


def _topk_impl(scores, lengths, output) -> None:
    rows = scores.shape[0]
    if rows == 0:
        return
    _lib.ensure_device(scores.device)
    _require(scores, torch.float32, "scores")
    _require(lengths, torch.int32, "lengths")
    _require(output, torch.int32, "output")
    if scores.stride(1) != 1 or output.stride(1) != 1:
        raise ValueError("scores and output must have unit column stride")
    lib = _lib.load_library()
    with torch.cuda.device(scores.device):
        _lib.check(lib.qsa_topk(
            scores.data_ptr(), scores.stride(0), rows, scores.shape[1], lengths.data_ptr(),
            output.data_ptr(), output.stride(0), output.shape[1],
            _lib.stream_ptr(scores.device)), "topk")


def _register() -> torch.library.Library | None:
    try:
        lib = torch.library.Library(_NS, "FRAGMENT")
        lib.define("topk(Tensor scores, Tensor lengths, Tensor(a!) output) -> ()")
        lib.define(
            "topk_expand(Tensor scores, Tensor lengths, Tensor positions, "
            "Tensor sequence_lengths, Tensor token_to_req, Tensor table, Tensor(a!) output, "
            "Tensor(b!) counts, int ratio, int page_size, bool physical, "
            "bool store_counts) -> ()")
    except RuntimeError:  # schemas already defined by another loader of this module
        return None
    lib.impl("topk", _topk_impl, "CUDA")
    lib.impl("topk_expand", _topk_expand_impl, "CUDA")
    lib.impl("topk", lambda *a: None, "Meta")
    lib.impl("topk_expand", lambda *a: None, "Meta")
    return lib


_LIBRARY = _register()


def topk(scores, lengths, output):
    """Plain top-k ids (ops/topk.py:25-26)."""
    torch.ops.yulan_qsa_kernels.topk(scores, lengths, output)


def topk_expand(scores, lengths, query_positions, sequence_lengths, token_to_req,
                output, compress_ratio, *, main_block_table=None, main_page_size=1,
                valid_counts_out=None):
    """Select blocks and write expanded slots, causal tail and counts in place
    (ops/topk.py:29-39; same dummy-tensor convention for unused arguments)."""
    torch.ops.yulan_qsa_kernels.topk_expand(
        scores, lengths, query_positions, sequence_lengths, token_to_req,
        main_block_table if main_block_table is not None else output,
        output, valid_counts_out if valid_counts_out is not None else output,
        compress_ratio, main_page_size, main_block_table is not None,
        valid_counts_out is not None,
    )


def topk_expand_visible(scores, query_positions, sequence_lengths, token_to_req, output,
                        compress_ratio, *, main_block_table=None, main_page_size=1,
                        valid_counts_out=None):
    """``topk_expand`` with each row's length computed in the kernel as its
    visible block count min((pos + 1) // r, seq_len // r) (ops/indexer.py:363-369),
    so no visible-count tensor is built first."""
    _topk_expand_call(
        scores, None, query_positions, sequence_lengths, token_to_req,
        main_block_table if main_block_table is not None else output,
        output, valid_counts_out if valid_counts_out is not None else output,
        compress_ratio, main_page_size, main_block_table is not None,
        valid_counts_out is not None)


__all__ = ["topk", "topk_expand", "topk_expand_visible"]
