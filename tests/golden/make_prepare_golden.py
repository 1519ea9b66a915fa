"""Golden vectors of the reference ``qsa_prepare`` kernel (CPU interpreter).

Run in the development container, where the reference package is readable:

    python tests/golden/make_prepare_golden.py REFERENCE_ROOT   (or set QSA_REFERENCE_ROOT)

Copies the reference package ``yulan_qsa_vllm`` to a temporary directory (as
``make_golden.py`` does), sets ``TRITON_INTERPRET=1`` and launches
``_qsa_prepare_kernel`` (ops/prepare.py:49-166) exactly as ``qsa_prepare``
(ops/prepare.py:169-228) does, on a seeded scenario of three requests:

* a decode row at a compression boundary whose group reads three earlier raw
  keys from the request's ring (state) cache;
* a 10-token prefill chunk whose first group starts in the previous chunk
  (two members from the ring) and whose suffix overwrites the ring;
* a 5-token chunk starting a sequence (one group, nothing from the ring);
* unmapped (-1) state, compressed and main slots.

The interpreter mishandles bf16 tensors, so every "bf16" tensor is stored as
fp32 holding bf16-representable values; the kernel's explicit bf16 casts
round correctly under the interpreter.  Its unary minus on a bf16 tensor does
not (it negates the raw bit pattern), so the copy's rotate-half line negates
in fp32 before the same bf16 cast (exact, value-preserving on the GPU).  Output: ``tests/golden/reference_prepare.npz``
with the inputs, the scenario constants and the four outputs (index queries,
compressed cache, state cache, main K/V caches).
"""

from __future__ import annotations

import os
import shutil
import sys
import tempfile
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent



def _reference_root(explicit: str | None) -> Path:
    """The reference checkout (holding ``yulan_qsa_vllm/``): the command-line
    argument, else ``$QSA_REFERENCE_ROOT``; one of them is required."""
    root = explicit or os.environ.get("QSA_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: pass the reference checkout as the first argument "
                         "or set QSA_REFERENCE_ROOT")
    return Path(root)

def _import_reference(ref_root: Path):
    tmp = Path(tempfile.mkdtemp(prefix="qsa_ref_"))
    shutil.copytree(ref_root / "yulan_qsa_vllm", tmp / "yulan_qsa_vllm")
    sys.path.insert(0, str(tmp))
    gd = types.ModuleType("yulan_qsa_vllm.graph_dispatch")
    gd.decode_logits_columns = lambda *a, **k: 0
    tk = types.ModuleType("yulan_qsa_vllm.ops.topk")
    tk.topk_expand = None
    sys.modules["yulan_qsa_vllm.graph_dispatch"] = gd
    sys.modules["yulan_qsa_vllm.ops.topk"] = tk
    # The interpreter negates a bf16 tensor by negating its raw 16-bit
    # pattern (as an integer), which turns -5.0 into -0.875.  On the GPU the
    # negation is exact; the copy negates in fp32 before the same bf16 cast,
    # which changes no value there.
    src = tmp / "yulan_qsa_vllm" / "ops" / "prepare.py"
    text = src.read_text()
    old = "rotated = tl.where(dims[None, :] < half, -partner, partner).to(tl.bfloat16)"
    assert old in text, "reference rotate-half line not found"
    src.write_text(text.replace(old, "rotated = tl.where(dims[None, :] < half, "
                                     "-partner.to(tl.float32), partner.to(tl.float32))"
                                     ".to(tl.bfloat16)"))
    from yulan_qsa_vllm.ops import prepare  # noqa: E402
    return prepare, tmp


def bf16ish(*shape, gen, scale=1.0):
    return (torch.randn(*shape, generator=gen) * scale).to(torch.bfloat16).float()


def scenario(gen: torch.Generator, rotary: int) -> dict:
    """Inputs of one launch (shared by the golden file and the GPU tests)."""
    heads, dim, ratio, state_size, comp_page = 4, 64, 4, 8, 16
    kv_heads, main_dim, main_page = 2, 128, 16
    # request 0: decode at 15; request 1: chunk 6..15; request 2: chunk 0..4
    positions = torch.tensor([15] + list(range(6, 16)) + list(range(0, 5)), dtype=torch.int64)
    qsl = torch.tensor([0, 1, 11, 16], dtype=torch.int32)
    tokens = positions.numel()
    state_table = torch.tensor([[2], [0], [1]], dtype=torch.int32)   # request -> ring block
    state_slots = torch.tensor([int(state_table[r, 0]) * state_size + int(p) % state_size
                                for r, p in zip([0] + [1] * 10 + [2] * 5, positions.tolist())],
                               dtype=torch.int64)
    state_slots[13] = -1                       # an unmapped raw-key slot
    # compressed slot of each boundary token (positions 3, 7, 11, 15), -1 elsewhere
    comp_slots = torch.full((tokens,), -1, dtype=torch.int64)
    for t, p in enumerate(positions.tolist()):
        if (p + 1) % ratio == 0:
            comp_slots[t] = 5 * comp_page + 3 * t        # scattered pages/offsets
    comp_slots[2] = -1                         # request 1's boundary at 7: unmapped
    # k work items: (request, work_in_request); request r has max(groups, 1)
    k_work = torch.tensor([[0, 0], [1, 0], [1, 1], [1, 2], [2, 0], [-1, 0]], dtype=torch.int32)
    main_slots = torch.tensor([3 * main_page + t for t in range(tokens)], dtype=torch.int64)
    main_slots[7] = -1
    return dict(
        heads=heads, dim=dim, rotary=rotary, ratio=ratio, state_size=state_size,
        comp_page=comp_page, kv_heads=kv_heads, main_dim=main_dim, main_page=main_page,
        eps=1e-6,
        index_qk=bf16ish(tokens, (heads + 1) * dim, gen=gen),
        positions=positions, q_weight=bf16ish(dim, gen=gen, scale=0.5) + 1.0,
        k_weight=bf16ish(dim, gen=gen, scale=0.5) + 1.0,
        cos_sin=bf16ish(64, rotary, gen=gen, scale=0.7).clamp(-1, 1).to(torch.bfloat16).float(),
        state_cache=bf16ish(3, state_size, dim, gen=gen),
        state_slots=state_slots, state_table=state_table, query_start_loc=qsl,
        logical_positions=positions.clone(),
        compressed_cache=bf16ish(8, comp_page, dim, gen=gen),
        compressed_slots=comp_slots, k_work=k_work,
        main_key=bf16ish(tokens, kv_heads, main_dim, gen=gen),
        main_value=bf16ish(tokens, kv_heads, main_dim, gen=gen),
        main_key_cache=bf16ish(6, main_page, kv_heads, main_dim, gen=gen),
        main_value_cache=bf16ish(6, main_page, kv_heads, main_dim, gen=gen),
        main_slots=main_slots,
    )


def run_reference(prepare, s: dict) -> dict:
    """The reference launch (ops/prepare.py:202-228) on copies of the caches."""
    out = {k: s[k].clone() for k in ("state_cache", "compressed_cache",
                                     "main_key_cache", "main_value_cache")}
    tokens = s["index_qk"].shape[0]
    query = torch.full((tokens, s["heads"], s["dim"]), float("nan"))
    tile_t, tile_h = 2, 2
    q_work = -(-tokens // tile_t) * -(-s["heads"] // tile_h)
    main_work = tokens * s["kv_heads"]
    mk, mv = s["main_key"], s["main_value"]
    kc, vc = out["main_key_cache"], out["main_value_cache"]
    prepare._qsa_prepare_kernel[(s["k_work"].shape[0] + q_work + main_work,)](
        s["index_qk"], s["positions"], s["q_weight"], s["k_weight"], s["cos_sin"], query,
        out["state_cache"], s["state_slots"], s["state_table"], s["query_start_loc"],
        s["logical_positions"], out["compressed_cache"], s["compressed_slots"], s["k_work"],
        mk, mv, kc, vc, s["main_slots"],
        s["index_qk"].stride(0), s["positions"].stride(0), out["state_cache"].stride(0),
        out["state_cache"].stride(1), s["state_table"].stride(0),
        out["compressed_cache"].stride(0), out["compressed_cache"].stride(1),
        *mk.stride(), *mv.stride(), *kc.stride(), *vc.stride(),
        tokens, s["k_work"].shape[0],
        INDEX_HEADS=s["heads"], INDEX_DIM=s["dim"], ROTARY=s["rotary"], EPS=s["eps"],
        COMPRESS_RATIO=s["ratio"], STATE_SIZE=s["state_size"], COMP_PAGE_SIZE=s["comp_page"],
        MAIN_KV_HEADS=s["kv_heads"], MAIN_DIM=s["main_dim"], MAIN_PAGE_SIZE=s["main_page"],
        TILE_T_Q=tile_t, TILE_H_Q=tile_h, num_warps=1, num_stages=1,
    )
    out["index_q"] = query
    return out


def main(ref_root: str | None = None) -> None:
    ref_root = str(_reference_root(ref_root))
    prepare, tmp = _import_reference(Path(ref_root))
    gen = torch.Generator().manual_seed(4321)
    arrays: dict[str, np.ndarray] = {}
    for name, rotary in (("rot64", 64), ("rot32", 32)):
        s = scenario(gen, rotary)
        res = run_reference(prepare, s)
        for k, v in s.items():
            arrays[f"{name}_in_{k}"] = v.numpy() if isinstance(v, torch.Tensor) else np.array(v)
        for k, v in res.items():
            arrays[f"{name}_out_{k}"] = v.numpy()
    path = HERE / "reference_prepare.npz"
    np.savez_compressed(path, **arrays)
    shutil.rmtree(tmp, ignore_errors=True)
    print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main(*sys.argv[1:])
