"""This package's layer step against golden outputs of the reference's own GPU
path on a B200 (tests/golden/make_reference_gpu_golden.py): the same seeded
inputs, rebuilt here on the CPU, must give the same selection and counts bit
for bit, and attention outputs within the bf16 tolerance; these fixtures pin
the reference's hardware bf16 rounding of P and of the gated output."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from golden_io import GOLDEN, from_bits16, load

pytestmark = pytest.mark.gpu
FIXTURE = GOLDEN / "reference_gpu.npz"
sys.path.insert(0, str(GOLDEN))

from make_reference_gpu_golden import CASES, build  # noqa: E402

ATT_ATOL = 2e-2


@pytest.mark.skipif(not FIXTURE.exists(), reason="reference GPU fixture not generated")
@pytest.mark.parametrize("name", list(CASES))
def test_layer_step_matches_reference_gpu_outputs(name):
    from oracle.time_reference import step_fn
    from qsa_vllm_b200 import indexer, qsa
    dev = torch.device("cuda")
    G = load(FIXTURE.name)
    w = build(name, dev)
    width = w.token_topk + w.ratio - 1
    idx = torch.full((w.rows, width), -7, dtype=torch.int32, device=dev)
    cnt = torch.zeros(w.rows, dtype=torch.int32, device=dev)
    out = torch.zeros_like(w.q)
    step_fn((indexer, qsa), w, idx, cnt, out)()
    torch.cuda.synchronize()
    assert np.array_equal(idx.cpu().numpy(), G[f"{name}_indices"])
    assert np.array_equal(cnt.cpu().numpy(), G[f"{name}_counts"])
    ref = from_bits16(G[f"{name}_out_bits"])
    err = (out.float().cpu() - ref).abs().max().item()
    assert err <= ATT_ATOL, f"{name}: attention max-abs {err}"
