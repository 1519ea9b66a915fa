"""Paged sparse GQA attention (drop-in for the reference ops/qsa.py entry point).

``qsa_sparse_paged_attention`` keeps the reference signature
(ops/qsa.py:594-608) and calls the sm_100a ``qsa_sparse_attention`` kernel.
The split-K plan is the library's own (it sizes the persistent grid to the
GPU); the reference's ``decode_config`` Triton tuning triple is accepted for
signature compatibility and ignored.  The split-K workspace comes from the
torch caching allocator, which is CUDA-graph-pool safe.
"""

from __future__ import annotations

import torch

from . import _lib


def attention_workspace_bytes(rows: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                              topk_width: int, use_decode_kernel: bool) -> int:
    lib = _lib.load_library()
    return int(lib.qsa_sparse_attention_workspace_bytes(
        rows, num_q_heads, num_kv_heads, head_dim, topk_width, int(use_decode_kernel)))


def aligned_head_rows(q: torch.Tensor) -> torch.Tensor:
    """``q`` itself when every head row starts on a 16-byte boundary (the kernel
    bulk-copies query rows), else a fresh contiguous copy.  ``.contiguous()``
    would not do: it returns a contiguous view unchanged even when the view
    starts at a misaligned element offset."""
    if q.data_ptr() % 16 or q.stride(0) % 8 or q.stride(1) % 8:
        return q.clone(memory_format=torch.contiguous_format)
    return q


def qsa_sparse_paged_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                               logical_indices: torch.Tensor, block_table: torch.Tensor,
                               token_to_req: torch.Tensor, out: torch.Tensor | None = None, *,
                               output_gate: torch.Tensor | None = None,
                               use_decode_kernel: bool = False,
                               indices_are_physical: bool = False,
                               valid_counts: torch.Tensor | None = None,
                               decode_config: tuple[int, int, int] | None = None,
                               workspace: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(q.K^T * d^-0.5).V over the tokens named by ``logical_indices``.

    q, out, output_gate: bf16 [rows, H_q, d]; k_cache / v_cache: bf16
    [num_blocks, page, H_kv, d]; logical_indices: int32 [rows, width] (physical
    slots when ``indices_are_physical``); valid_counts: int32 [rows] bounds the
    columns read per row.  ``decode_config`` is ignored (see module docstring).
    """
    del decode_config
    if out is None:
        out = torch.empty_like(q)
    rows = q.shape[0]
    if not rows:
        return out
    _lib.ensure_device(q.device)
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache), ("out", out)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
        if t.stride(-1) != 1:
            raise ValueError(f"{name} needs a unit head-dim stride")
    if logical_indices.dtype != torch.int32 or logical_indices.stride(-1) != 1:
        raise TypeError("indices must be int32 with unit column stride")
    if not indices_are_physical:
        if block_table.dtype != torch.int32 or token_to_req.dtype != torch.int32:
            raise TypeError("block_table and token_to_req must be int32")
    if valid_counts is not None and valid_counts.dtype != torch.int32:
        raise TypeError("valid_counts must be int32")
    gate = output_gate
    if gate is not None and gate.dtype != torch.bfloat16:
        raise TypeError("output_gate must be bfloat16")
    q = aligned_head_rows(q)
    hq, d = q.shape[1], q.shape[2]
    hkv = k_cache.shape[2]
    width = logical_indices.shape[1]
    need = attention_workspace_bytes(rows, hq, hkv, d, width, use_decode_kernel)
    if need and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    lib = _lib.load_library()
    with torch.cuda.device(q.device):
        _lib.check(lib.qsa_sparse_attention(
            q.data_ptr(), q.stride(0), q.stride(1), rows, hq, d,
            k_cache.data_ptr(), k_cache.stride(0), k_cache.stride(1), k_cache.stride(2),
            v_cache.data_ptr(), v_cache.stride(0), v_cache.stride(1), v_cache.stride(2),
            k_cache.shape[0], k_cache.shape[1], hkv,
            logical_indices.data_ptr(), logical_indices.stride(0), width,
            block_table.data_ptr() if block_table is not None else None,
            block_table.stride(0) if block_table is not None else 0,
            block_table.shape[1] if block_table is not None else 0,
            block_table.shape[0] if block_table is not None else 0,
            token_to_req.data_ptr() if token_to_req is not None else None,
            valid_counts.data_ptr() if valid_counts is not None else None,
            gate.data_ptr() if gate is not None else None,
            gate.stride(0) if gate is not None else 0, gate.stride(1) if gate is not None else 0,
            gate.stride(2) if gate is not None else 0,
            out.data_ptr(), out.stride(0), out.stride(1),
            1 if indices_are_physical else 0, 1 if use_decode_kernel else 0,
            workspace.data_ptr() if need else None, need,
            _lib.stream_ptr(q.device)), "sparse_attention")
    return out


__all__ = ["qsa_sparse_paged_attention", "attention_workspace_bytes", "aligned_head_rows"]
