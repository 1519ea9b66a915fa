"""The reference layer's exact call sequence, run on this package's operators.

Replays what the plugin's YuLanQSAAttention._run_qsa and YuLanQSAImpl.forward
do per step (reference attention.py:169-214, backend.py:49-67), with the
persistent module buffers they use (attention.py:169-182): a
``topk_indices_buffer`` of ``max_num_batched_tokens`` rows and a
``topk_counts_buffer``, both left uninitialised (garbage-filled here) and
sliced to the step's token count; ``output.zero_()`` before attention; and
``use_decode_kernel = indices_are_physical = (max_query_len == 1)`` with valid
counts only for decode.  The main K / V caches are the two halves of one
``[blocks, page, H_kv, 2 d]`` buffer (backend.py:148-153).  Results are
checked against the oracle: selections bit-exact (the oracle's top-k applied
to the kernel's own scores), attention within max-abs 2e-2, and the buffer
rows past the step's tokens untouched.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import qsa_oracle as O

pytestmark = pytest.mark.gpu

MAX_BATCHED_TOKENS = 9000
SCORE_RTOL, SCORE_ATOL = 1e-3, 1e-5


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import qsa_vllm_b200  # noqa: F401
    return torch.device("cuda")


def _layer_step(w, dev, indices_buffer, counts_buffer, output):
    """attention.py:191-214 then backend.py:49-67, with this package's operators."""
    from qsa_vllm_b200.indexer import select_paged_tokens
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    count = w.rows
    is_decode = w.max_query_len == 1
    select_paged_tokens(
        w.index_q[:count], w.index_cache, w.index_table, w.token_to_req, w.positions,
        w.seq_lens, w.token_topk, w.ratio, indices_buffer[:count],
        query_start_loc=w.query_start_loc, max_query_len=w.max_query_len,
        max_seq_len=w.max_seq_len, num_decodes=w.rows if is_decode else 0,
        num_decode_tokens=w.rows if is_decode else 0, decode_query_len=1,
        visible_blocks=None,
        main_block_table=w.block_table if is_decode else None,
        main_page_size=w.kv.shape[1],
        valid_counts_out=counts_buffer[:count] if is_decode else None,
        weights=w.index_weights, scale=w.index_scale)
    key_cache, value_cache = w.kv[..., :w.d], w.kv[..., w.d:]
    output.zero_()
    qsa_sparse_paged_attention(
        w.q[:count], key_cache, value_cache, indices_buffer[:count], w.block_table,
        w.token_to_req[:count], output[:count],
        output_gate=w.gate[:count],
        use_decode_kernel=w.max_query_len == 1,
        indices_are_physical=w.max_query_len == 1,
        valid_counts=counts_buffer[:count] if w.max_query_len == 1 else None)
    torch.cuda.synchronize()


def _buffers(w, dev):
    width = w.token_topk + w.ratio - 1
    idx = torch.full((MAX_BATCHED_TOKENS, width), -7, dtype=torch.int32, device=dev)
    cnt = torch.full((MAX_BATCHED_TOKENS,), -7, dtype=torch.int32, device=dev)
    out = torch.full((MAX_BATCHED_TOKENS, w.q.shape[1], w.d), 3.0, dtype=torch.bfloat16,
                     device=dev)
    return idx, cnt, out


def _gpu_scores(w, dev, vis, cols, rows):
    from qsa_vllm_b200.indexer import indexer_scores
    logits = torch.zeros(w.rows, cols, device=dev)
    kw = (dict(decode_query_len=1) if w.max_query_len == 1 else
          dict(query_start_loc=w.query_start_loc, max_query_len=w.max_query_len))
    indexer_scores(w.index_q, w.index_cache, w.index_table, vis.to(dev), logits,
                   weights=w.index_weights, scale=w.index_scale, **kw)
    return logits.cpu()


def _check_attention(got, ref):
    err = (got.float().cpu() - ref).abs().max().item()
    assert err <= 2e-2, f"attention max-abs {err}"


@pytest.mark.parametrize("config,seed", [("cfg0", 0), ("cfg2", 1)])
def test_layer_call_sequence_decode(dev, config, seed):
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload(config, device=dev, seed=seed, batch=8 if config == "cfg2" else None)
    idx, cnt, out = _buffers(w, dev)
    _layer_step(w, dev, idx, cnt, out)
    count = w.rows
    vis = O.visible_blocks(w.positions.cpu(), w.seq_lens.cpu(), w.token_to_req.cpu(), w.ratio)
    cols = w.index_table.shape[1] * w.index_cache.shape[1]
    from qsa_vllm_b200.graph_dispatch import decode_logits_columns
    cols = decode_logits_columns(w.max_seq_len, w.ratio, cols)
    gl = _gpu_scores(w, dev, vis, cols, count)
    ref_idx, ref_cnt = O.topk_expand(gl, vis, w.positions.cpu(), w.seq_lens.cpu(),
                                     w.token_to_req.cpu(), w.block_table.cpu(),
                                     w.token_topk + w.ratio - 1, w.ratio,
                                     page_size=w.page_size)
    assert np.array_equal(idx[:count].cpu().numpy(), ref_idx)
    assert np.array_equal(cnt[:count].cpu().numpy(), ref_cnt)
    # the persistent buffers' other rows are untouched; output was zeroed whole
    assert bool((idx[count:] == -7).all()) and bool((cnt[count:] == -7).all())
    assert bool((out[count:] == 0).all())
    d = w.d
    ref = O.sparse_attention(w.q.cpu(), w.kv.cpu()[..., :d], w.kv.cpu()[..., d:],
                             idx[:count].cpu(), w.block_table.cpu(), w.token_to_req.cpu(),
                             output_gate=w.gate.cpu(), use_decode_kernel=True,
                             indices_are_physical=True, valid_counts=cnt[:count].cpu())
    _check_attention(out[:count], ref)


def test_layer_call_sequence_prefill(dev):
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg1", device=dev, seed=2, batch=2, seq_len=3000, new_tokens=700)
    assert w.max_query_len > 1
    idx, cnt, out = _buffers(w, dev)
    _layer_step(w, dev, idx, cnt, out)
    count = w.rows
    vis = O.visible_blocks(w.positions.cpu(), w.seq_lens.cpu(), w.token_to_req.cpu(), w.ratio)
    lw = -(-(-(-w.max_seq_len // w.ratio)) // 64) * 64
    gl = _gpu_scores(w, dev, vis, lw, count)
    ref_idx, _ = O.topk_expand(gl, vis, w.positions.cpu(), w.seq_lens.cpu(),
                               w.token_to_req.cpu(), None, w.token_topk + w.ratio - 1, w.ratio)
    assert np.array_equal(idx[:count].cpu().numpy(), ref_idx)
    assert bool((idx[count:] == -7).all()) and bool((cnt == -7).all())
    assert bool((out[count:] == 0).all())
    sel = torch.arange(0, count, 37)
    ref = O.sparse_attention(w.q.cpu()[sel], w.kv.cpu()[..., :w.d], w.kv.cpu()[..., w.d:],
                             idx[:count].cpu()[sel], w.block_table.cpu(),
                             w.token_to_req.cpu()[sel], output_gate=w.gate.cpu()[sel])
    _check_attention(out[:count][sel.to(dev)], ref)
