"""GPU checks of the measurement hooks bench.py relies on.

``qsa_set_attention_timing_events`` makes the library record two CUDA events
around the main attention kernel (bench.py's roofline times that kernel alone
with them, inside a replayed CUDA graph).  The hook must time something real
and must not change the attention's output.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _decode_inputs(dev):
    from qsa_vllm_b200.indexer import select_paged_tokens
    from qsa_vllm_b200.synthetic import make_workload
    w = make_workload("cfg2_32k", device=dev, seed=6, batch=8)
    idx = torch.empty(w.rows, w.token_topk + w.ratio - 1, dtype=torch.int32, device=dev)
    cnt = torch.empty(w.rows, dtype=torch.int32, device=dev)
    select_paged_tokens(
        w.index_q, w.index_cache, w.index_table, w.token_to_req, w.positions, w.seq_lens,
        w.token_topk, w.ratio, idx, **w.select_kwargs(), main_block_table=w.block_table,
        main_page_size=w.page_size, valid_counts_out=cnt, weights=w.index_weights,
        scale=w.index_scale)
    return w, idx, cnt


def test_attention_timing_events_time_the_kernel_and_change_nothing(dev):
    from qsa_vllm_b200 import _lib
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    w, idx, cnt = _decode_inputs(dev)

    def attn(out):
        qsa_sparse_paged_attention(w.q, w.k_cache, w.v_cache, idx, w.block_table,
                                   w.token_to_req, out, output_gate=w.gate,
                                   use_decode_kernel=True, indices_are_physical=True,
                                   valid_counts=cnt)

    plain = torch.empty_like(w.q)
    attn(plain)
    ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    _lib.set_attention_timing_events(*ev)
    try:
        timed = torch.empty_like(w.q)
        attn(timed)                      # eager: events on the current stream
        torch.cuda.synchronize()
        eager_ms = ev[0].elapsed_time(ev[1])
        graphed = torch.empty_like(w.q)
        g = torch.cuda.CUDAGraph()       # captured: events become graph nodes
        with torch.cuda.graph(g):
            attn(graphed)
    finally:
        _lib.set_attention_timing_events(None, None)
    g.replay()
    torch.cuda.synchronize()
    graph_ms = ev[0].elapsed_time(ev[1])
    assert torch.equal(timed, plain) and torch.equal(graphed, plain)
    # the kernel moves 8 rows x 2051 tokens x 2 KB: well above a microsecond,
    # far below a second
    for ms in (eager_ms, graph_ms):
        assert 1e-3 < ms < 1e3, ms
    # cleared: a later call records nothing into the events
    ev[1].record()
    torch.cuda.synchronize()
    before = ev[0].elapsed_time(ev[1])
    attn(plain)
    torch.cuda.synchronize()
    assert ev[0].elapsed_time(ev[1]) == before
