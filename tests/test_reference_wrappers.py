"""The reference plugin's own top-k wrappers drive this package's op library.

``yulan_qsa_vllm/ops/topk.py`` (reference ops/topk.py:1-39) JIT-builds its
sm_80 extension at import and then only forwards to
``torch.ops.yulan_qsa_kernels.topk`` / ``topk_expand``.  This test imports
that file unchanged from a temporary copy (so nothing is written into the
reference tree) with ``torch.utils.cpp_extension.load`` stubbed out, after
``qsa_vllm_b200`` registered the op schemas.  Its calls must bind to those
schemas: on meta tensors (this package's Meta kernels) and on CPU tensors
through a test-only CPU kernel that runs the oracle, whose result must equal
the oracle called directly, for every argument convention the wrapper uses
(dummy table / counts tensors when unused).

Runs where the reference checkout is readable ($QSA_REFERENCE_ROOT, or a
directory ``reference`` beside this repository); skipped elsewhere.
"""

from __future__ import annotations

import importlib.util
import shutil
import sys

import numpy as np
import pytest
import torch

from oracle import build_ref
from oracle import qsa_oracle as O
from topk_cases import standard_cases

REF_TOPK = build_ref.reference_root() / "yulan_qsa_vllm" / "ops" / "topk.py"


@pytest.fixture()
def reference_topk(tmp_path, monkeypatch):
    if not REF_TOPK.exists():
        pytest.skip("reference checkout not present")
    import qsa_vllm_b200  # noqa: F401  (registers torch.ops.yulan_qsa_kernels)
    import torch.utils.cpp_extension as ce
    dst = tmp_path / "yulan_qsa_vllm" / "ops"
    dst.mkdir(parents=True)
    shutil.copy(REF_TOPK, dst / "topk.py")
    calls = []
    monkeypatch.setattr(ce, "load", lambda **kw: calls.append(kw))
    spec = importlib.util.spec_from_file_location("reference_ops_topk", dst / "topk.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    assert len(calls) == 1 and calls[0]["name"] == "yulan_qsa_topk_sm80"
    yield mod
    sys.modules.pop("reference_ops_topk", None)


def _oracle_cpu_kernels():
    """Test-only CPU kernels for the two ops, computing with the oracle."""
    lib = torch.library.Library("yulan_qsa_kernels", "IMPL")

    def topk_expand(scores, lengths, positions, seq_lens, t2r, table, output, counts, ratio,
                    page_size, physical, store_counts):
        out, cnt = O.topk_expand(scores, lengths, positions, seq_lens, t2r,
                                 table if physical else None, output.shape[1], ratio,
                                 page_size=page_size)
        output.copy_(torch.from_numpy(out))
        if store_counts:
            counts.copy_(torch.from_numpy(cnt))

    def topk(scores, lengths, output):
        output.copy_(torch.from_numpy(O.topk_plain(scores, lengths, output.shape[1])))

    lib.impl("topk_expand", topk_expand, "CPU")
    lib.impl("topk", topk, "CPU")
    return lib


def test_reference_wrappers_bind_to_registered_schemas_on_meta(reference_topk):
    case = next(c for c in standard_cases().values() if c["physical"] and c["store_counts"])
    m = {k: (v.to("meta") if isinstance(v, torch.Tensor) else v) for k, v in case.items()}
    rows, width = case["scores"].shape[0], case["output_width"]
    out = torch.empty(rows, width, dtype=torch.int32, device="meta")
    cnt = torch.empty(rows, dtype=torch.int32, device="meta")
    reference_topk.topk_expand(m["scores"], m["lengths"], m["positions"], m["seq_lens"],
                               m["token_to_req"], out, case["ratio"],
                               main_block_table=m["table"], main_page_size=case["page_size"],
                               valid_counts_out=cnt)
    reference_topk.topk_expand(m["scores"], m["lengths"], m["positions"], m["seq_lens"],
                               m["token_to_req"], out, case["ratio"])
    reference_topk.topk(m["scores"], m["lengths"], torch.empty(rows, 16, dtype=torch.int32,
                                                                device="meta"))


def test_reference_wrappers_match_oracle_through_registered_ops(reference_topk):
    lib = _oracle_cpu_kernels()
    try:
        for name, case in standard_cases().items():
            rows, width = case["scores"].shape[0], case["output_width"]
            out = torch.full((rows, width), -7, dtype=torch.int32)
            cnt = torch.full((rows,), -7, dtype=torch.int32)
            kw = {}
            if case["physical"]:
                kw.update(main_block_table=case["table"], main_page_size=case["page_size"])
            if case["store_counts"]:
                kw.update(valid_counts_out=cnt)
            reference_topk.topk_expand(case["scores"], case["lengths"], case["positions"],
                                       case["seq_lens"], case["token_to_req"], out,
                                       case["ratio"], **kw)
            ref, ref_cnt = O.topk_expand(case["scores"], case["lengths"], case["positions"],
                                         case["seq_lens"], case["token_to_req"],
                                         case["table"] if case["physical"] else None, width,
                                         case["ratio"], page_size=case["page_size"])
            assert np.array_equal(out.numpy(), ref), name
            if case["store_counts"]:
                assert np.array_equal(cnt.numpy(), ref_cnt), name
        case = next(iter(standard_cases().values()))
        plain = torch.full((case["scores"].shape[0], 16), -7, dtype=torch.int32)
        reference_topk.topk(case["scores"], case["lengths"], plain)
        assert np.array_equal(plain.numpy(), O.topk_plain(case["scores"], case["lengths"], 16))
    finally:
        del lib
