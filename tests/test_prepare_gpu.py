"""GPU parity of ``qsa_prepare`` (index queries, compressed keys, ring commit,
main K/V writes) against the CPU oracle, through the C ABI.

Bars: raw-key ring and main K/V caches bit-exact (they are copies); normed +
rotated rows (index queries, compressed keys) within 2e-2 absolute + 1.6e-2
relative (two bf16 ulps), and at least 99% of their elements bit-exact: the
kernel rounds to bf16 at the reference's steps; the inverse RMS (rsqrt) and
the order of the squared sum may move a value across a rounding boundary.
The oracle itself equals the reference kernel bit for bit on the golden
scenarios (``test_oracle_golden.py``).
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from golden_io import load
from oracle import qsa_oracle as O

pytestmark = pytest.mark.gpu

NORM_ATOL, NORM_RTOL, EXACT_FRACTION = 2e-2, 1.6e-2, 0.99


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def golden_scenario(name: str) -> dict:
    d = load("reference_prepare.npz")
    s = {}
    for key, v in d.items():
        if key.startswith(f"{name}_in_"):
            s[key[len(name) + 4:]] = torch.from_numpy(v.copy()) if v.ndim else v.item()
    # the fixture's norm weights (bf16 + 1.0, kept in fp32) are not all
    # bf16-representable; the device path reads bf16, so both sides use that
    for k in ("q_weight", "k_weight"):
        s[k] = s[k].to(torch.bfloat16).float()
    return s


def random_scenario(seed: int, *, heads: int, dim: int, rotary: int, ratio: int,
                    state_size: int, comp_page: int, kv_heads: int, main_dim: int,
                    main_page: int, chunks: list[tuple[int, int]], unmapped: float = 0.03,
                    padding: int = 3, max_position: int = 4096, row_pad: int = 16) -> dict:
    """Requests given as (chunk_start, query_len); each gets its own ring block,
    scattered compressed slots for its boundary tokens and scattered main slots;
    k_work lists max(groups, 1) items per request in shuffled order plus padding."""
    g = torch.Generator().manual_seed(seed)

    def bf16(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).float()

    positions, owner = [], []
    qsl = [0]
    for r, (start, qlen) in enumerate(chunks):
        positions += list(range(start, start + qlen))
        owner += [r] * qlen
        qsl.append(qsl[-1] + qlen)
    tokens = len(positions)
    positions = torch.tensor(positions, dtype=torch.int64)
    nreq = len(chunks)
    ring_blocks = nreq + 2
    state_table = torch.randperm(ring_blocks, generator=g)[:nreq].to(torch.int32)[:, None]
    state_slots = torch.tensor([int(state_table[r, 0]) * state_size + p % state_size
                                for r, p in zip(owner, positions.tolist())], dtype=torch.int64)
    boundary = [t for t, p in enumerate(positions.tolist()) if (p + 1) % ratio == 0]
    comp_blocks = -(-len(boundary) // comp_page) + 2
    comp_perm = torch.randperm(comp_blocks * comp_page, generator=g)
    comp_slots = torch.full((tokens,), -1, dtype=torch.int64)
    for k, t in enumerate(boundary):
        comp_slots[t] = comp_perm[k]
    main_blocks = -(-tokens // main_page) + 2
    main_slots = torch.randperm(main_blocks * main_page, generator=g)[:tokens].to(torch.int64)
    drop = torch.rand(tokens, generator=g) < unmapped
    state_slots[drop] = -1
    comp_slots[torch.rand(tokens, generator=g) < unmapped] = -1
    main_slots[torch.rand(tokens, generator=g) < unmapped] = -1
    work = []
    for r, (start, qlen) in enumerate(chunks):
        end = start + qlen - 1
        groups = (end + 1) // ratio - start // ratio
        work += [[r, w] for w in range(max(groups, 1))]
    work += [[-1, 0]] * padding
    k_work = torch.tensor(work, dtype=torch.int32)[torch.randperm(len(work), generator=g)]
    # main K/V as views of one projection row (strided tokens), caches as the
    # two halves of a [blocks, page, kv_heads, 2 * dim] pool
    proj = bf16(tokens, 2 * kv_heads * main_dim + 8)
    kv_pool = bf16(main_blocks, main_page, kv_heads, 2 * main_dim)
    return dict(
        heads=heads, dim=dim, rotary=rotary, ratio=ratio, state_size=state_size,
        comp_page=comp_page, kv_heads=kv_heads, main_dim=main_dim, main_page=main_page,
        eps=1e-6,
        index_qk=bf16(tokens, (heads + 1) * dim + row_pad)[:, :(heads + 1) * dim],
        positions=positions, q_weight=(bf16(dim, scale=0.5) + 1.0).to(torch.bfloat16).float(),
        k_weight=(bf16(dim, scale=0.5) + 1.0).to(torch.bfloat16).float(),
        cos_sin=bf16(max_position, rotary, scale=0.7).clamp(-1, 1),
        state_cache=bf16(ring_blocks, state_size, dim),
        state_slots=state_slots, state_table=state_table,
        query_start_loc=torch.tensor(qsl, dtype=torch.int32),
        logical_positions=positions.clone(),
        compressed_cache=bf16(comp_blocks, comp_page, dim),
        compressed_slots=comp_slots, k_work=k_work,
        main_key=proj[:, :kv_heads * main_dim].reshape(tokens, kv_heads, main_dim),
        main_value=proj[:, kv_heads * main_dim:2 * kv_heads * main_dim].reshape(
            tokens, kv_heads, main_dim),
        main_key_cache=kv_pool[..., :main_dim], main_value_cache=kv_pool[..., main_dim:],
        main_slots=main_slots,
    )


CACHES = ("state_cache", "compressed_cache", "main_key_cache", "main_value_cache")


def run_oracle(s: dict) -> dict:
    out = {k: s[k].clone() for k in CACHES}
    q = O.qsa_prepare(
        s["index_qk"], s["positions"], s["q_weight"], s["k_weight"], s["cos_sin"], s["eps"],
        out["state_cache"], s["state_slots"], s["state_table"], s["query_start_loc"],
        s["logical_positions"], out["compressed_cache"], s["compressed_slots"], s["k_work"],
        s["main_key"], s["main_value"], out["main_key_cache"], out["main_value_cache"],
        s["main_slots"], num_index_heads=s["heads"], index_head_dim=s["dim"],
        rotary_dim=s["rotary"], compress_ratio=s["ratio"], rounding="nearest")
    out["index_q"] = q
    return out


def _to_dev(t: torch.Tensor, dev) -> torch.Tensor:
    """bf16 (for float) copy on the device that keeps the tensor's strides."""
    dtype = torch.bfloat16 if t.is_floating_point() else t.dtype
    base = torch.empty_strided(t.size(), t.stride(), dtype=dtype, device=dev)
    base.copy_(t)
    return base


def run_gpu(s: dict, dev, *, main_pool_views: bool = True) -> dict:
    from qsa_vllm_b200.prepare import qsa_prepare
    t = {k: _to_dev(v, dev) for k, v in s.items() if isinstance(v, torch.Tensor)}
    if main_pool_views and s["main_key_cache"].data_ptr() + s["main_dim"] * 4 == \
            s["main_value_cache"].data_ptr():
        # keep the caches as the two halves of one pool, as the layer holds them
        pool = _to_dev(torch.cat([s["main_key_cache"], s["main_value_cache"]], -1), dev)
        t["main_key_cache"] = pool[..., :s["main_dim"]]
        t["main_value_cache"] = pool[..., s["main_dim"]:]
    raw = SimpleNamespace(slot_mapping=t["state_slots"], block_table=t["state_table"],
                          query_start_loc=t["query_start_loc"],
                          logical_positions=t["logical_positions"])
    comp = SimpleNamespace(slot_mapping=t["compressed_slots"], k_work_metadata=t["k_work"])
    q = qsa_prepare(t["index_qk"], t["positions"], t["q_weight"], t["k_weight"], t["cos_sin"],
                    s["eps"], raw, comp, t["state_cache"], t["compressed_cache"],
                    t["main_key"], t["main_value"], t["main_key_cache"],
                    t["main_value_cache"], t["main_slots"], num_index_heads=s["heads"],
                    index_head_dim=s["dim"], rotary_dim=s["rotary"],
                    compress_ratio=s["ratio"])
    torch.cuda.synchronize()
    out = {k: t[k].float().cpu() for k in CACHES}
    out["index_q"] = q.float().cpu()
    return out


def check(got: dict, ref: dict) -> None:
    for k in ("state_cache", "main_key_cache", "main_value_cache"):
        assert torch.equal(got[k], ref[k]), f"{k} differs"
    for k in ("index_q", "compressed_cache"):
        torch.testing.assert_close(got[k], ref[k], atol=NORM_ATOL, rtol=NORM_RTOL, msg=k)
        exact = (got[k] == ref[k]).float().mean().item()
        assert exact >= EXACT_FRACTION, f"{k}: only {exact:.4f} of elements bit-exact"


@pytest.mark.parametrize("name", ["rot64", "rot32"])
def test_prepare_golden_scenarios(dev, name):
    """The reference kernel's golden scenarios (decode at a boundary reading the
    ring, a chunk starting mid-group, a sequence start, unmapped slots)."""
    s = golden_scenario(name)
    check(run_gpu(s, dev), run_oracle(s))


BENCH_INDEX = dict(heads=8, dim=64, rotary=64, ratio=4, state_size=128, comp_page=64, kv_heads=4,
                   main_dim=128, main_page=64)


@pytest.mark.parametrize("rotary", [64, 32])
def test_prepare_decode_batch(dev, rotary):
    """64 decode rows at scattered positions (every fourth at a group boundary)."""
    g = torch.Generator().manual_seed(7)
    starts = torch.randint(8, 4000, (64,), generator=g).tolist()
    s = random_scenario(11, chunks=[(p, 1) for p in starts], **{**BENCH_INDEX, "rotary": rotary})
    check(run_gpu(s, dev), run_oracle(s))


@pytest.mark.parametrize("dim,heads,rotary,ratio,state_size", [
    (64, 8, 64, 4, 128), (128, 4, 64, 4, 16), (128, 2, 128, 8, 8), (64, 8, 16, 2, 4)])
def test_prepare_mixed_chunks(dev, dim, heads, rotary, ratio, state_size):
    """Decodes and prefill chunks of assorted starts and lengths: groups split
    across chunks (ring reads), chunks shorter than a group, chunks longer than
    the ring, a sequence start."""
    chunks = [(0, 37), (5, 1), (ratio - 1, 1), (130, 200), (41, ratio - 1), (300, 3), (7, 64),
              (1000, 1), (2 * ratio + 1, 2)]
    s = random_scenario(100 + dim + rotary + ratio, heads=heads, dim=dim, rotary=rotary,
                        ratio=ratio, state_size=state_size, comp_page=16, kv_heads=2,
                        main_dim=dim, main_page=16, chunks=chunks)
    check(run_gpu(s, dev), run_oracle(s))


@pytest.mark.parametrize("rotary,row_pad", [(24, 16), (64, 2)])
def test_prepare_per_head_path(dev, rotary, row_pad):
    """Layouts the 16-byte token path does not take: a rotary width that is not
    a multiple of 16, and index rows that are only 4-byte aligned."""
    chunks = [(0, 21), (9, 1), (3, 1), (50, 30), (17, 2)]
    s = random_scenario(31 + rotary, chunks=chunks, row_pad=row_pad,
                        **{**BENCH_INDEX, "rotary": rotary})
    check(run_gpu(s, dev), run_oracle(s))


def test_prepare_main_scalar_path(dev):
    """Main K/V with a non-unit dim stride (element-wise copies)."""
    s = random_scenario(5, chunks=[(3, 9), (64, 1)], **BENCH_INDEX)
    t = s["main_key"].shape
    s["main_key"] = s["main_key"].transpose(1, 2).contiguous().transpose(1, 2)
    assert s["main_key"].stride(2) != 1 and s["main_key"].shape == t
    check(run_gpu(s, dev, main_pool_views=False), run_oracle(s))


def test_prepare_large_prefill(dev):
    """One 8192-token chunk (2048 groups) + 64 decodes at the bench's index shapes."""
    g = torch.Generator().manual_seed(3)
    starts = torch.randint(8, 60000, (64,), generator=g).tolist()
    s = random_scenario(21, chunks=[(0, 8192)] + [(p, 1) for p in starts],
                        max_position=65536, padding=0, **BENCH_INDEX)
    check(run_gpu(s, dev), run_oracle(s))


def test_prepare_out_of_range_slot_is_skipped_and_reported(dev):
    from qsa_vllm_b200 import _lib
    s = random_scenario(9, chunks=[(0, 8)], unmapped=0.0, **BENCH_INDEX)
    blocks, page = s["main_key_cache"].shape[:2]
    s_bad = dict(s)
    s_bad["main_slots"] = s["main_slots"].clone()
    s_bad["main_slots"][2] = blocks * page + 5    # past the pool: skipped
    _lib.device_error_poll()
    got = run_gpu(s_bad, dev)
    bits = _lib.device_error_poll()
    assert bits & 2
    s_ref = dict(s_bad)
    s_ref["main_slots"] = s_bad["main_slots"].clone()
    s_ref["main_slots"][2] = -1                   # the oracle's view: token 2 unmapped
    check(got, run_oracle(s_ref))


def test_prepare_empty(dev):
    from qsa_vllm_b200.prepare import qsa_prepare
    s = random_scenario(1, chunks=[(0, 4)], **BENCH_INDEX)
    t = {k: _to_dev(v, dev) for k, v in s.items() if isinstance(v, torch.Tensor)}
    raw = SimpleNamespace(slot_mapping=t["state_slots"][:0], block_table=t["state_table"],
                          query_start_loc=t["query_start_loc"][:1],
                          logical_positions=t["logical_positions"][:0])
    comp = SimpleNamespace(slot_mapping=t["compressed_slots"][:0],
                           k_work_metadata=t["k_work"][:0])
    before = t["state_cache"].clone()
    q = qsa_prepare(t["index_qk"][:0], t["positions"][:0], t["q_weight"], t["k_weight"],
                    t["cos_sin"], 1e-6, raw, comp, t["state_cache"], t["compressed_cache"],
                    t["main_key"][:0], t["main_value"][:0], t["main_key_cache"],
                    t["main_value_cache"], t["main_slots"][:0], num_index_heads=8,
                    index_head_dim=64, rotary_dim=64, compress_ratio=4)
    torch.cuda.synchronize()
    assert q.shape == (0, 8, 64)
    assert torch.equal(before, t["state_cache"])
