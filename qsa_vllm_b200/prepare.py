"""Indexer preparation + main K/V cache writes (drop-in for the reference ops/prepare.py).

``qsa_prepare`` has the reference's signature (ops/prepare.py:169-228) and
runs the sm_100a ``qsa_prepare`` launch of ``libqsa_b200.so``:

* index queries: RMSNorm with ``q_norm_weight``, then rotate-half RoPE of the
  first ``rotary_dim`` dims at each token's position, bf16-rounded after every
  post-norm step (ops/prepare.py:16-46, :99-118);
* compressed keys: per ``k_work_metadata`` item, the mean of
  ``compress_ratio`` raw keys ending at a compression boundary (from this
  step's projection, or from the request's raw-key ring for earlier positions),
  normed with ``k_norm_weight`` and rotated at the group's first position,
  stored at the boundary token's compressed slot (:120-152);
* ring commit: each request's first work item writes the chunk's last
  ``min(query_len, ring size)`` raw keys to their ring slots, after its own
  group has read the ring (:154-166);
* main K/V: every token's key / value rows to ``main_slots`` (:81-97).

Slots < 0 are skipped.  ``raw_metadata`` needs ``slot_mapping`` (ring slots,
int64), ``block_table`` (ring block per request, int32),
``query_start_loc`` (int32) and ``logical_positions`` (int64);
``compressed_metadata`` needs ``slot_mapping`` (compressed slots, int64) and
``k_work_metadata`` (int32 ``[n, 2]`` = (request, work item)).  Index
tensors of another integer dtype are converted first.  The projection,
weights, rotary cache and caches are bf16, as the reference layer builds them
(ops/normalization.py:18-29, attention.py:88-110).
"""

from __future__ import annotations

import torch

from . import _lib


def _as(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    t = t if t.dtype == dtype else t.to(dtype)
    return t if t.is_contiguous() else t.contiguous()


def _bf16(name: str, t: torch.Tensor) -> None:
    if t.dtype != torch.bfloat16:
        raise TypeError(f"qsa_prepare: {name} must be bf16, got {t.dtype}")


def qsa_prepare(
    index_qk: torch.Tensor,
    positions: torch.Tensor,
    q_norm_weight: torch.Tensor,
    k_norm_weight: torch.Tensor,
    cos_sin_cache: torch.Tensor,
    eps: float,
    raw_metadata,
    compressed_metadata,
    state_cache: torch.Tensor,
    compressed_cache: torch.Tensor,
    main_key: torch.Tensor,
    main_value: torch.Tensor,
    main_key_cache: torch.Tensor,
    main_value_cache: torch.Tensor,
    main_slots: torch.Tensor,
    *,
    num_index_heads: int,
    index_head_dim: int,
    rotary_dim: int,
    compress_ratio: int,
) -> torch.Tensor:
    """Prepare the index queries and update the ring, compressed and main caches
    in place; returns the index queries ``[tokens, num_index_heads,
    index_head_dim]`` (bf16)."""
    tokens = index_qk.shape[0]
    H, D = int(num_index_heads), int(index_head_dim)
    query = index_qk.new_empty(tokens, H, D)
    k_work = _as(compressed_metadata.k_work_metadata, torch.int32)
    if tokens == 0 and k_work.shape[0] == 0:
        return query
    dev = index_qk.device
    _lib.ensure_device(dev)
    for name, t in (("index_qk", index_qk), ("q_norm_weight", q_norm_weight),
                    ("k_norm_weight", k_norm_weight), ("cos_sin_cache", cos_sin_cache),
                    ("state_cache", state_cache), ("compressed_cache", compressed_cache),
                    ("main_key", main_key), ("main_value", main_value),
                    ("main_key_cache", main_key_cache), ("main_value_cache", main_value_cache)):
        _bf16(name, t)
    if index_qk.dim() != 2 or index_qk.stride(1) != 1:
        raise ValueError("qsa_prepare: index_qk must be [tokens, width] with unit column stride")
    for name, cache in (("state_cache", state_cache), ("compressed_cache", compressed_cache)):
        if cache.dim() < 3 or cache.stride(-1) != 1 or cache.shape[-1] != D:
            raise ValueError(f"qsa_prepare: {name} must be [blocks, page, ..., {D}] "
                             "with contiguous rows")
    if main_key.dim() != 3 or main_value.shape != main_key.shape \
            or main_key_cache.dim() != 4 or main_value_cache.shape != main_key_cache.shape:
        raise ValueError("qsa_prepare: main key/value [tokens, kv_heads, dim] and caches "
                         "[blocks, page, kv_heads, dim] expected")
    if main_key.shape[0] < tokens or main_key_cache.shape[2:] != main_key.shape[1:]:
        raise ValueError("qsa_prepare: main key/value rows or cache heads/dim do not match")
    if positions.dim() != 1 or positions.shape[0] < tokens:
        raise ValueError("qsa_prepare: positions must be 1-D with one entry per token")
    if q_norm_weight.numel() < D or k_norm_weight.numel() < D:
        raise ValueError(f"qsa_prepare: norm weights need {D} entries")
    if k_work.dim() != 2 or k_work.shape[1] != 2:
        raise ValueError("qsa_prepare: k_work_metadata must be [n, 2]")
    for name, t in (("raw slot_mapping", raw_metadata.slot_mapping),
                    ("raw logical_positions", raw_metadata.logical_positions),
                    ("compressed slot_mapping", compressed_metadata.slot_mapping),
                    ("main_slots", main_slots)):
        if t.numel() < tokens:
            raise ValueError(f"qsa_prepare: {name} needs one entry per token")
    positions = positions if positions.dtype == torch.int64 else positions.to(torch.int64)
    q_w = q_norm_weight.contiguous()
    k_w = k_norm_weight.contiguous()
    cos_sin = cos_sin_cache.contiguous()
    state_slots = _as(raw_metadata.slot_mapping, torch.int64)
    state_table = raw_metadata.block_table
    if state_table.dtype != torch.int32:
        state_table = state_table.to(torch.int32)
    qsl = _as(raw_metadata.query_start_loc, torch.int32)
    if state_table.dim() != 2 or state_table.shape[0] < qsl.numel() - 1:
        raise ValueError("qsa_prepare: raw block_table needs one row per request")
    logical = _as(raw_metadata.logical_positions, torch.int64)
    comp_slots = _as(compressed_metadata.slot_mapping, torch.int64)
    main_slots = _as(main_slots, torch.int64)
    state_blocks = state_cache.shape[0]
    comp_blocks = compressed_cache.shape[0]
    mk, mv = main_key, main_value
    kc, vc = main_key_cache, main_value_cache
    lib = _lib.load_library()
    with torch.cuda.device(dev):
        _lib.check(lib.qsa_prepare(
            index_qk.data_ptr(), index_qk.stride(0), tokens, H, D,
            positions.data_ptr(), positions.stride(0),
            q_w.data_ptr(), k_w.data_ptr(), cos_sin.data_ptr(),
            cos_sin.numel() // int(rotary_dim), int(rotary_dim), float(eps), query.data_ptr(),
            state_cache.data_ptr(), state_cache.stride(0), state_cache.stride(1), state_blocks,
            state_cache.shape[1], state_slots.data_ptr(), state_table.data_ptr(),
            state_table.stride(0), qsl.data_ptr(), qsl.numel() - 1, logical.data_ptr(),
            compressed_cache.data_ptr(), compressed_cache.stride(0), compressed_cache.stride(1),
            comp_blocks, compressed_cache.shape[1], comp_slots.data_ptr(), k_work.data_ptr(),
            k_work.shape[0], int(compress_ratio),
            mk.data_ptr(), *mk.stride(), mv.data_ptr(), *mv.stride(),
            kc.data_ptr(), *kc.stride(), vc.data_ptr(), *vc.stride(),
            kc.shape[0], kc.shape[1], main_slots.data_ptr(), mk.shape[1], mk.shape[2],
            _lib.stream_ptr(dev)), "qsa_prepare")
    return query


__all__ = ["qsa_prepare"]
