"""Seeded top-k / expansion cases covering the reference selector's edge cases.

Each case is a dict of CPU tensors in the dtypes of the op schema plus
``ratio``, ``page_size``, ``physical``, ``store_counts`` and ``output_width``.
Covered: rows with length <= K (no score read), length 0, length == width,
all-zero rows (massive ties), few distinct values (ties at the threshold),
``-0.0`` and negative scores (uint32 ordering), +inf, widths on both sides of
the reference's 8192 (2048-bin vs 256-bin) and 32768 (partition + merge, only
for <= 32 rows) switches, page_size % ratio != 0, unmapped pages (-1),
token_to_req == -1, positions not at the end of the sequence, and a
non-contiguous output column stride.
"""

from __future__ import annotations

import numpy as np
import torch


def _scores(rng: np.random.Generator, rows: int, width: int, kind: str) -> np.ndarray:
    if kind == "uniform":
        return rng.random((rows, width), dtype=np.float32) * 4.0
    if kind == "relu":  # ReLU-summed indexer scores: many exact zeros, positive tail
        x = rng.standard_normal((rows, width)).astype(np.float32)
        return np.maximum(x, 0.0) * 3.0
    if kind == "ties":  # few distinct values: ties straddle the threshold
        return rng.integers(0, 4, (rows, width)).astype(np.float32) * 0.5
    if kind == "zeros":
        return np.zeros((rows, width), dtype=np.float32)
    if kind == "signed":  # -0.0, negatives and +inf: uint32 bit ordering
        x = rng.standard_normal((rows, width)).astype(np.float32)
        x[:, ::7] = -0.0
        x[:, 3::11] = np.inf
        return x
    raise ValueError(kind)


def make_case(seed: int, rows: int, width: int, token_topk: int, *, ratio: int = 4,
              kind: str = "uniform", physical: bool = True, page_size: int = 16,
              store_counts: bool = True, lengths: str = "mixed") -> dict:
    rng = np.random.default_rng(seed)
    scores = _scores(rng, rows, width, kind)
    requests = max(1, rows // 2)
    # sequence lengths long enough to cover `width` compressed blocks
    seq = rng.integers(width * ratio // 2, width * ratio + ratio, requests).astype(np.int32)
    t2r = rng.integers(0, requests, rows).astype(np.int32)
    if rows > 2:
        t2r[-1] = -1
    pos = np.array([rng.integers(0, max(1, seq[r])) if r >= 0 else 0 for r in t2r],
                   dtype=np.int64)
    if rows > 1 and t2r[0] >= 0:
        pos[0] = seq[t2r[0]] - 1                      # decode-like row
    vis = np.minimum((pos + 1) // ratio,
                     np.where(t2r >= 0, seq[np.maximum(t2r, 0)] // ratio, 0)).astype(np.int32)
    vis = np.where(t2r >= 0, vis, 0).astype(np.int32)
    if lengths == "full":
        vis[:] = width
    elif lengths == "mixed":
        vis = np.minimum(vis, width).astype(np.int32)
        if rows > 3:
            vis[1] = width
            vis[2] = min(width, token_topk // ratio)      # exactly K
            vis[3] = 0
    table_width = -(-(int(seq.max()) + ratio) // page_size)
    table = rng.permutation(requests * table_width + 8)[: requests * table_width]
    table = table.reshape(requests, table_width).astype(np.int32)
    table[0, rng.integers(0, table_width)] = -1          # an unmapped page
    return dict(
        scores=torch.from_numpy(scores), lengths=torch.from_numpy(vis),
        positions=torch.from_numpy(pos), seq_lens=torch.from_numpy(seq),
        token_to_req=torch.from_numpy(t2r), table=torch.from_numpy(table),
        ratio=ratio, page_size=page_size, physical=physical, store_counts=store_counts,
        output_width=token_topk + ratio - 1)


def aligned_rows(scores: torch.Tensor) -> torch.Tensor:
    """Same values in storage whose row stride is a multiple of 4 floats.

    The reference selector reads score rows with float4 loads
    (ops/csrc/topk.cu:80-88), so it requires 16-byte aligned rows; every
    caller in the reference passes widths that are multiples of 64.  Inputs
    handed to the reference checker are laid out this way.
    """
    rows, width = scores.shape
    padded = torch.zeros(rows, -(-width // 4) * 4, dtype=scores.dtype, device=scores.device)
    padded[:, :width] = scores
    return padded[:, :width]


def standard_cases() -> dict[str, dict]:
    """The named case set used by the parity tests and the golden fixtures."""
    c = {}
    c["small_uniform"] = make_case(1, 6, 40, 32)
    c["small_ties"] = make_case(2, 6, 64, 32, kind="ties")
    c["zeros"] = make_case(3, 5, 300, 64, kind="zeros")
    c["signed"] = make_case(4, 5, 500, 64, kind="signed")
    c["relu_2k"] = make_case(5, 8, 2048, 512, kind="relu")
    c["logical"] = make_case(6, 8, 1000, 256, physical=False, store_counts=False)
    c["page6"] = make_case(7, 6, 777, 128, page_size=6)           # page % ratio != 0
    c["page8_r4"] = make_case(8, 6, 900, 128, page_size=8, kind="ties")
    c["w8192"] = make_case(9, 4, 8192, 2048, kind="relu", lengths="full")
    c["w8193"] = make_case(10, 4, 8193, 2048, kind="uniform", lengths="full")
    c["w20000_ties"] = make_case(11, 3, 20000, 2048, kind="ties", lengths="full")
    c["w40000"] = make_case(12, 2, 40000, 2048, kind="relu", lengths="full")
    c["w40000_mixed"] = make_case(13, 5, 40000, 1024, kind="uniform")
    c["ratio1"] = make_case(14, 4, 3000, 512, ratio=1, page_size=16)
    return c


__all__ = ["aligned_rows", "make_case", "standard_cases"]
