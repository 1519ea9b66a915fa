"""B200-native (sm_100a) QSA sparse-attention hot path.

Drop-in replacements for the reference plugin's operators:

* ``qsa_vllm_b200.indexer.select_paged_tokens``  (ops/indexer.py)
* ``qsa_vllm_b200.topk.topk_expand`` / ``torch.ops.yulan_qsa_kernels.*``  (ops/topk.py)
* ``qsa_vllm_b200.qsa.qsa_sparse_paged_attention``  (ops/qsa.py)
* ``qsa_vllm_b200.prepare.qsa_prepare``  (ops/prepare.py index-query norm/RoPE, key
  compression and cache writes)
* ``qsa_vllm_b200.graph_dispatch``  (graph_dispatch.py CUDA-graph column buckets)
* ``qsa_vllm_b200.backend``  (backend.py attention-backend surface)

All compute runs in ``libqsa_b200.so`` (hand-written CUDA for sm_100a behind a
C ABI, ``include/qsa_b200.h``).  There is no CPU or Triton fallback.
"""

from . import topk as _topk_ops  # noqa: F401  registers torch.ops.yulan_qsa_kernels
from ._lib import QSAError, version  # noqa: F401

__all__ = ["QSAError", "version"]
