"""qsa_sparse_attention_static_scratch: the attention entry point that allocates
nothing (split-K scratch in a static device array) against qsa_sparse_attention
with a caller workspace.  It is meant for callers that cannot allocate device
memory: code running under a global-mode stream capture (cudaMalloc is refused
there), engines whose KV cache took all free memory at start-up, and C callers
without a caching allocator (cudaMalloc / cudaFree per call would synchronise
the device).

Collected last (file name), and self-contained, so it runs the same alone in a
fresh process and after the other GPU tests.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from qsa_vllm_b200 import _lib

pytestmark = pytest.mark.gpu


def _static_call(lib, q, k, v, idx, table, t2r, counts, gate, out):
    """The same arguments qsa.qsa_sparse_paged_attention passes, minus the workspace."""
    rows, hq, d = q.shape
    return lib.qsa_sparse_attention_static_scratch(
        q.data_ptr(), q.stride(0), q.stride(1), rows, hq, d,
        k.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
        v.data_ptr(), v.stride(0), v.stride(1), v.stride(2),
        k.shape[0], k.shape[1], k.shape[2],
        idx.data_ptr(), idx.stride(0), idx.shape[1],
        table.data_ptr(), table.stride(0), table.shape[1], table.shape[0],
        t2r.data_ptr(), counts.data_ptr(),
        gate.data_ptr(), gate.stride(0), gate.stride(1), gate.stride(2),
        out.data_ptr(), out.stride(0), out.stride(1),
        1, 1, torch.cuda.current_stream().cuda_stream)


def _case(dev, rows, seed, hq=32, hkv=4, d=128, page=64, nblk=256, width=2051):
    g = torch.Generator().manual_seed(seed)
    kv = torch.randn(nblk, page, hkv, 2 * d, generator=g).to(torch.bfloat16).to(dev)
    q = (torch.randn(rows, hq, d, generator=g) * d ** -0.5).to(torch.bfloat16).to(dev)
    gate = torch.randn(rows, hq, d, generator=g).to(torch.bfloat16).to(dev)
    idx = torch.randint(0, nblk * page, (rows, width), generator=g).to(torch.int32)
    counts = torch.randint(1, width + 1, (rows,), generator=g).to(torch.int32)
    idx[torch.arange(width)[None, :] >= counts[:, None]] = -1
    table = torch.zeros(1, 1, dtype=torch.int32)
    t2r = torch.zeros(rows, dtype=torch.int32)
    return (q, kv[..., :d], kv[..., d:], idx.to(dev), table.to(dev), t2r.to(dev),
            counts.to(dev), gate)


def test_static_scratch_matches_caller_workspace_on_consecutive_calls():
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.ensure_device(dev)
    lib = _lib.load_library()
    # two calls in a row with different row counts: the second call's slots sit
    # at other offsets of the shared scratch than the first call's
    for rows, seed in ((64, 1), (5, 2)):
        q, k, v, idx, table, t2r, counts, gate = _case(dev, rows, seed)
        ref = qsa_sparse_paged_attention(q, k, v, idx, table, t2r, output_gate=gate,
                                         use_decode_kernel=True, indices_are_physical=True,
                                         valid_counts=counts)
        out = torch.full_like(q, float("nan"))
        _lib.check(_static_call(lib, q, k, v, idx, table, t2r, counts, gate, out),
                   "static scratch attention")
        torch.cuda.synchronize()
        assert torch.equal(out, ref), f"rows={rows}: static-scratch output differs"
    assert _lib.device_error_poll() == 0


def test_static_scratch_need_does_not_grow_with_rows():
    """The split-K scratch holds two slot groups per CTA (one partial per
    consumer warp), so the need is bounded by the SM count, not the rows:
    every call fits the static array, and a many-row call through it equals
    the caller-workspace path."""
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.ensure_device(dev)
    lib = _lib.load_library()
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    static_max = 32 << 20
    for hq, hkv, d in ((32, 4, 128), (16, 2, 128), (16, 1, 128), (64, 4, 64), (8, 8, 128)):
        bound = 256 + 2 * sms * 8 * (hq // hkv) * (d + 1) * 4
        for rows in (1, 64, 1024, 8192, 1 << 20):
            for width, decode in ((2051, 1), (1027, 0), (65539, 1)):
                need = lib.qsa_sparse_attention_workspace_bytes(rows, hq, hkv, d, width, decode)
                assert need <= bound <= static_max, (hq, hkv, d, rows, width, need)
    rows = 3000
    q, k, v, idx, table, t2r, counts, gate = _case(dev, rows, seed=5)
    ref = qsa_sparse_paged_attention(q, k, v, idx, table, t2r, output_gate=gate,
                                     use_decode_kernel=True, indices_are_physical=True,
                                     valid_counts=counts)
    out = torch.full_like(q, float("nan"))
    _lib.check(_static_call(lib, q, k, v, idx, table, t2r, counts, gate, out),
               "static scratch attention")
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert _lib.device_error_poll() == 0
    assert ctypes.sizeof(ctypes.c_size_t) == 8


def test_static_scratch_validates_shapes_before_its_maximum():
    """A malformed call is refused as malformed (invalid / unsupported shape)
    before any scratch check, and launches nothing."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    _lib.ensure_device(dev)
    lib = _lib.load_library()
    rows, width = 4096, 2051
    x = torch.zeros(16, dtype=torch.int32, device=dev)
    n0 = _lib.kernel_launches()
    for hq, hkv, d, expected in ((32, 4, 256, 2),   # head dim 256: QSA_ERR_UNSUPPORTED
                                 (30, 4, 128, 1)):  # 30 query heads over 4 KV: QSA_ERR_INVALID
        status = lib.qsa_sparse_attention_static_scratch(
            x.data_ptr(), hq * d, d, rows, hq, d,
            x.data_ptr(), 0, 0, 0, x.data_ptr(), 0, 0, 0, 1, 64, hkv,
            x.data_ptr(), width, width, x.data_ptr(), 1, 1, 1, x.data_ptr(), x.data_ptr(),
            None, 0, 0, 0, x.data_ptr(), hq * d, d, 1, 1,
            torch.cuda.current_stream().cuda_stream)
        assert status == expected, (hq, hkv, d, status, lib.qsa_last_error().decode())
    assert _lib.kernel_launches() == n0
