"""Head sharding across tensor-parallel ranks (no collective inside the QSA path).

The reference splits query and KV heads ``// tp_size`` (attention.py:148-150)
and replicates the indexer and its caches on every rank (attention.py:39,
cache.py:6-7); the attention output slice then feeds vLLM's o_proj
all-reduce, outside this path.  ``head_shard`` returns the query-head and
KV-head slices a rank owns.  When ``tp_size`` exceeds the KV head count (for
instance 4 KV heads at tp 8, where the reference's integer division would give
zero), KV heads are replicated: each rank keeps the single KV head its query
heads attend with, as vLLM's QKVParallelLinear does.
"""

from __future__ import annotations


def head_shard(num_q_heads: int, num_kv_heads: int, tp_size: int,
               tp_rank: int) -> tuple[slice, slice]:
    if tp_size <= 0 or not 0 <= tp_rank < tp_size:
        raise ValueError(f"bad tp rank {tp_rank} of {tp_size}")
    if num_q_heads % tp_size:
        raise ValueError(f"{num_q_heads} query heads do not split over {tp_size} ranks")
    if num_q_heads % num_kv_heads:
        raise ValueError("query heads must be a multiple of KV heads")
    qn = num_q_heads // tp_size
    q0 = tp_rank * qn
    group = num_q_heads // num_kv_heads
    if tp_size <= num_kv_heads:
        if num_kv_heads % tp_size:
            raise ValueError(f"{num_kv_heads} KV heads do not split over {tp_size} ranks")
        kn = num_kv_heads // tp_size
        return slice(q0, q0 + qn), slice(tp_rank * kn, tp_rank * kn + kn)
    if group % qn:
        raise ValueError("a rank's query heads must not straddle two KV heads")
    kv = q0 // group
    return slice(q0, q0 + qn), slice(kv, kv + 1)


__all__ = ["head_shard"]
