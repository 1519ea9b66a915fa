"""The reference layer's order on the GPU: ``qsa_prepare`` then the decode step.

``qsa_prepare`` writes this step's compressed index keys, the raw-key ring and
the current tokens' main K/V; the indexer and the attention that follow read
them, launched right behind it with programmatic dependent launch.  The step
is checked against the CPU oracle on the caches as ``qsa_prepare`` left them
(scores within tolerance, selection bit-exact on the GPU's own scores,
attention within tolerance), and the compressed keys the step scored are the
ones ``qsa_prepare`` wrote.
"""

import pytest
import torch

from test_gpu_parity import _check_decode_rows, _decode_step

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def test_prepare_then_decode_step(dev):
    from qsa_vllm_b200.prepare import qsa_prepare
    from qsa_vllm_b200.synthetic import make_prepare_inputs, make_workload
    # mixed lengths: some rows end a compression block (their new compressed
    # key is scored this step), others carry a causal tail with the new token
    w = make_workload("cfg2", device=dev, seed=8, batch=8)
    a = make_prepare_inputs(w, seed=3)
    before = w.index_cache.clone()
    w.index_q = qsa_prepare(**a)
    out_idx, counts, out = _decode_step(w, dev)   # same stream, right behind prepare
    # the compressed slots written this step changed the cache the step read
    slots = a["compressed_metadata"].slot_mapping
    page = w.index_cache.shape[1]
    written = slots[slots >= 0]
    assert written.numel() > 0
    flat_before = before.view(-1, before.shape[-1])
    flat_after = w.index_cache.view(-1, w.index_cache.shape[-1])
    assert not torch.equal(flat_before[written], flat_after[written])
    assert int((written // page).max()) < w.index_cache.shape[0]
    _check_decode_rows(w, dev, out_idx, counts, out, list(range(w.rows)))
    # rows with a causal tail select their own (just written) token
    tails = ((w.positions + 1) % w.ratio).cpu()
    assert bool((tails > 0).any())
    main_slot = a["main_slots"].cpu()
    idx = out_idx.cpu()
    for r in torch.nonzero(tails > 0).flatten().tolist():
        assert int(main_slot[r]) in idx[r].tolist()
