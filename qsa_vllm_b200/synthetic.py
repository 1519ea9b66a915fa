"""Seeded synthetic QSA layer inputs with the shapes of the benchmark configurations.

No dataset is involved: every input is drawn from a seeded generator with the
distributions the benchmark specifies (q / K / V / index keys N(0,1) bf16, q
scaled by head_dim^-0.5, head weights U(0,1)), on paged caches whose block
tables are seeded random permutations of the physical pool (so consecutive
logical pages land on scattered physical pages, as in a fragmented cache).

Layouts match what the reference plugin receives from vLLM:
  * main cache ``kv``: bf16 ``[num_blocks, page, H_kv, 2*d]``; ``k_cache`` /
    ``v_cache`` are the two halves of the last dim (backend.py:148-153);
  * index-key cache: bf16 ``[num_index_blocks, index_page, 1, d_i]`` (one
    compressed key per ``ratio`` tokens) with its own block table;
  * decode rows are the last token of each request: position = seq_len - 1
    (the last ``dql`` tokens for multi-token decode).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

# name -> configuration ("cfg2_32k" is the headline decode point)
CONFIGS: dict[str, dict] = {
    "cfg0": dict(batch=4, seq_len=2048, hq=16, hkv=2, d=128, hi=4, di=64, page=16,
                 num_blocks=512, token_topk=512, ratio=4),
    "cfg1": dict(batch=2, seq_len=8192, new_tokens=4096, hq=16, hkv=2, d=128, hi=4, di=64,
                 page=16, token_topk=1024, ratio=4),
    "cfg2": dict(batch=64, seq_len=(8192, 32768), hq=32, hkv=4, d=128, hi=8, di=64, page=64,
                 token_topk=2048, ratio=4),
    "cfg2_32k": dict(batch=64, seq_len=32768, hq=32, hkv=4, d=128, hi=8, di=64, page=64,
                     token_topk=2048, ratio=4),
    "cfg3": dict(batch=8, seq_len=131072, hq=32, hkv=4, d=128, hi=8, di=64, page=64,
                 token_topk=2048, ratio=4),
    # variants of the headline decode point: per-token index keys (ratio 1), and
    # multi-token (MTP) decode with two query rows per request
    "cfg2_32k_r1": dict(batch=64, seq_len=32768, hq=32, hkv=4, d=128, hi=8, di=64, page=64,
                        token_topk=2048, ratio=1),
    "cfg2_32k_mtp2": dict(batch=64, seq_len=32768, hq=32, hkv=4, d=128, hi=8, di=64, page=64,
                          token_topk=2048, ratio=4, dql=2),
}


@dataclass
class SyntheticQSA:
    """One QSA layer's inputs for a decode or chunked-prefill step."""
    name: str
    ratio: int
    token_topk: int
    page_size: int
    seq_lens: torch.Tensor          # int32 [B]
    positions: torch.Tensor         # int64 [rows]
    token_to_req: torch.Tensor      # int32 [rows]
    query_start_loc: torch.Tensor   # int32 [B+1]
    q: torch.Tensor                 # bf16 [rows, H_q, d]
    gate: torch.Tensor              # bf16 [rows, H_q, d]
    kv: torch.Tensor                # bf16 [blocks, page, H_kv, 2d]
    block_table: torch.Tensor       # int32 [B, width]
    index_q: torch.Tensor           # bf16 [rows, H_i, d_i]
    index_weights: torch.Tensor | None  # fp32 [rows, H_i]
    index_scale: float
    index_cache: torch.Tensor       # bf16 [index_blocks, page, 1, d_i]
    index_table: torch.Tensor       # int32 [B, index_width]
    is_decode: bool = True
    extra: dict = field(default_factory=dict)

    @property
    def d(self) -> int:
        return self.q.shape[2]

    @property
    def k_cache(self) -> torch.Tensor:
        return self.kv[..., : self.d]

    @property
    def v_cache(self) -> torch.Tensor:
        return self.kv[..., self.d:]

    @property
    def rows(self) -> int:
        return self.q.shape[0]

    @property
    def max_seq_len(self) -> int:
        """Host-side value (no device sync: safe inside CUDA-graph capture)."""
        return self.extra["max_seq_len"]

    @property
    def max_query_len(self) -> int:
        return self.extra["max_query_len"]

    @property
    def decode_query_len(self) -> int:
        return self.extra.get("decode_query_len", 1)

    def select_kwargs(self) -> dict:
        """Batch-shape keywords of ``select_paged_tokens`` for this step: every
        row a decode row (``decode_query_len`` per request), or every row a
        packed prefill row."""
        if self.is_decode:
            dql = self.decode_query_len
            return dict(query_start_loc=self.query_start_loc, max_query_len=dql,
                        max_seq_len=self.max_seq_len, num_decodes=self.rows // dql,
                        num_decode_tokens=self.rows, decode_query_len=dql)
        return dict(query_start_loc=self.query_start_loc, max_query_len=self.max_query_len,
                    max_seq_len=self.max_seq_len)

    def shard_heads(self, tp_size: int, tp_rank: int) -> "SyntheticQSA":
        """This rank's view under head (tensor-parallel) sharding: query heads and
        KV heads split ``//tp`` (attention.py:148-150); when tp exceeds the KV
        head count each rank keeps the one KV head its query heads use.  The
        indexer and its caches are replicated on every rank (cache.py:6-7)."""
        from .sharding import head_shard
        qs, ks = head_shard(self.q.shape[1], self.kv.shape[2], tp_size, tp_rank)
        kv = self.kv[:, :, ks].contiguous()
        return SyntheticQSA(
            name=f"{self.name}/tp{tp_size}r{tp_rank}", ratio=self.ratio,
            token_topk=self.token_topk, page_size=self.page_size, seq_lens=self.seq_lens,
            positions=self.positions, token_to_req=self.token_to_req,
            query_start_loc=self.query_start_loc, q=self.q[:, qs].contiguous(),
            gate=self.gate[:, qs].contiguous(), kv=kv, block_table=self.block_table,
            index_q=self.index_q, index_weights=self.index_weights,
            index_scale=self.index_scale, index_cache=self.index_cache,
            index_table=self.index_table, is_decode=self.is_decode, extra=dict(self.extra))


def _tables(gen: torch.Generator, pages_per_req: list[int], device) -> tuple[torch.Tensor, int]:
    total = sum(pages_per_req)
    perm = torch.randperm(total, generator=gen).to(torch.int32)
    width = max(pages_per_req)
    table = torch.full((len(pages_per_req), width), -1, dtype=torch.int32)
    off = 0
    for r, n in enumerate(pages_per_req):
        table[r, :n] = perm[off:off + n]
        off += n
    return table.to(device), total


def make_workload(name: str = "cfg2_32k", *, device="cuda", seed: int = 0,
                  batch: int | None = None, seq_len: int | tuple | None = None,
                  head_weights: bool = True, **overrides) -> SyntheticQSA:
    """Build the inputs of configuration ``name`` (see ``CONFIGS``).

    ``batch`` / ``seq_len`` / other keys override the configuration (tests use
    small versions of the same shapes).  Random tensors are drawn on
    ``device`` with a generator seeded by ``seed``; metadata is built on the CPU.
    ``head_weights=False`` gives the reference's unit head weights.
    """
    cfg = dict(CONFIGS[name])
    if batch is not None:
        cfg["batch"] = batch
    if seq_len is not None:
        cfg["seq_len"] = seq_len
    cfg.update(overrides)
    device = torch.device(device)
    cpu = torch.Generator().manual_seed(seed)
    B, ratio, page = cfg["batch"], cfg["ratio"], cfg["page"]
    sl = cfg["seq_len"]
    if isinstance(sl, tuple):
        seq_lens = torch.randint(sl[0], sl[1] + 1, (B,), generator=cpu).to(torch.int32)
    else:
        seq_lens = torch.full((B,), int(sl), dtype=torch.int32)
    new = cfg.get("new_tokens")
    is_decode = new is None
    dql = int(cfg.get("dql", 1))
    if is_decode:
        q_lens = torch.full((B,), dql, dtype=torch.int32)
    else:
        q_lens = torch.full((B,), int(new), dtype=torch.int32)
    qsl = torch.zeros(B + 1, dtype=torch.int32)
    qsl[1:] = torch.cumsum(q_lens, 0)
    rows = int(qsl[-1])
    token_to_req = torch.repeat_interleave(torch.arange(B, dtype=torch.int32), q_lens.long())
    positions = torch.cat([torch.arange(int(L) - int(n), int(L), dtype=torch.int64)
                           for L, n in zip(seq_lens, q_lens)])

    main_pages = [-(-int(L) // page) for L in seq_lens]
    if "num_blocks" in cfg and sum(main_pages) <= cfg["num_blocks"]:
        main_pages_pool = cfg["num_blocks"]
    else:
        main_pages_pool = sum(main_pages)
    perm = torch.randperm(main_pages_pool, generator=cpu).to(torch.int32)
    width = max(main_pages)
    block_table = torch.full((B, width), -1, dtype=torch.int32)
    off = 0
    for r, n in enumerate(main_pages):
        block_table[r, :n] = perm[off:off + n]
        off += n
    index_pages = [max(1, -(-(int(L) // ratio) // page)) for L in seq_lens]
    index_table, index_pool = _tables(cpu, index_pages, "cpu")

    gdev = torch.Generator(device=device).manual_seed(seed + 1)
    hq, hkv, d, hi, di = cfg["hq"], cfg["hkv"], cfg["d"], cfg["hi"], cfg["di"]

    def randn(*shape, scale=1.0):
        x = torch.randn(*shape, generator=gdev, device=device, dtype=torch.bfloat16)
        return x if scale == 1.0 else (x.float() * scale).to(torch.bfloat16)

    kv = randn(main_pages_pool, page, hkv, 2 * d)
    q = randn(rows, hq, d, scale=d ** -0.5)
    gate = randn(rows, hq, d)
    index_cache = randn(index_pool, page, 1, di)
    index_q = randn(rows, hi, di, scale=di ** -0.5)
    weights = (torch.rand(rows, hi, generator=gdev, device=device, dtype=torch.float32)
               if head_weights else None)
    return SyntheticQSA(
        name=name, ratio=ratio, token_topk=cfg["token_topk"], page_size=page,
        seq_lens=seq_lens.to(device), positions=positions.to(device),
        token_to_req=token_to_req.to(device), query_start_loc=qsl.to(device), q=q, gate=gate,
        kv=kv, block_table=block_table.to(device), index_q=index_q, index_weights=weights,
        index_scale=di ** -0.5, index_cache=index_cache, index_table=index_table.to(device),
        is_decode=is_decode,
        extra={"config": cfg, "max_seq_len": int(seq_lens.max()),
               "max_query_len": int(q_lens.max()), "decode_query_len": dql})


def rope_cache(max_position: int, rotary_dim: int, theta: float, device) -> torch.Tensor:
    """bf16 [max_position, rotary_dim]: cos(p * theta^(-2i/rotary)) for the
    rotary_dim/2 channels, then the sines (the layout ops/normalization.py:18-23
    builds)."""
    inv = theta ** (-torch.arange(0, rotary_dim, 2, dtype=torch.float32) / rotary_dim)
    phase = torch.outer(torch.arange(max_position, dtype=torch.float32), inv)
    return torch.cat((phase.cos(), phase.sin()), -1).to(torch.bfloat16).to(device)


def make_prepare_inputs(w: SyntheticQSA, *, seed: int = 0, state_size: int = 64,
                        rotary_dim: int | None = None, theta: float = 1e7) -> dict:
    """Keyword arguments of ``qsa_vllm_b200.prepare.qsa_prepare`` for the step of
    ``w``: a fresh index projection (bf16 N(0,1), ``[rows, (H_i + 1) * d_i]``),
    main K/V rows written into ``w``'s paged pool at each token's slot, the
    compressed key of every group that ends in this step written into ``w``'s
    index-key cache (slot from its index table), and one raw-key ring of
    ``state_size`` rows per request.  Metadata is built on the host, as a
    scheduler does, then moved to the device."""
    dev = w.q.device
    hi, di = w.index_q.shape[1], w.index_q.shape[2]
    hkv, d = w.kv.shape[2], w.d
    r, page = w.ratio, w.page_size
    rows = w.rows
    rotary_dim = di if rotary_dim is None else rotary_dim
    pos = w.positions.cpu()
    req = w.token_to_req.cpu().long()
    qsl = w.query_start_loc.cpu()
    table = w.block_table.cpu().long()
    itable = w.index_table.cpu().long()
    ipage = w.index_cache.shape[1]
    B = qsl.numel() - 1
    main_slots = table[req, pos // page] * page + pos % page
    blk = pos // r
    comp_slots = torch.where((pos + 1) % r == 0,
                             itable[req, (blk // ipage).clamp(max=itable.shape[1] - 1)] * ipage
                             + blk % ipage, torch.full_like(pos, -1))
    state_slots = req * state_size + pos % state_size
    work = []
    for b in range(B):
        q0, q1 = int(qsl[b]), int(qsl[b + 1])
        if q1 <= q0:
            continue
        end = int(pos[q1 - 1])
        start = end - (q1 - q0) + 1
        groups = (end + 1) // r - start // r
        work += [[b, i] for i in range(max(groups, 1))]
    g = torch.Generator(device=dev).manual_seed(seed + 7)

    def randn(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(torch.bfloat16)

    from types import SimpleNamespace
    raw = SimpleNamespace(slot_mapping=state_slots.to(dev),
                          block_table=torch.arange(B, dtype=torch.int32, device=dev)[:, None],
                          query_start_loc=w.query_start_loc, logical_positions=w.positions)
    comp = SimpleNamespace(slot_mapping=comp_slots.to(dev),
                           k_work_metadata=torch.tensor(work, dtype=torch.int32,
                                                        device=dev).reshape(-1, 2))
    return dict(
        index_qk=randn(rows, (hi + 1) * di), positions=w.positions,
        q_norm_weight=randn(di, scale=0.1) + 1, k_norm_weight=randn(di, scale=0.1) + 1,
        cos_sin_cache=rope_cache(w.max_seq_len + 1, rotary_dim, theta, dev), eps=1e-6,
        raw_metadata=raw, compressed_metadata=comp,
        state_cache=randn(B, state_size, di), compressed_cache=w.index_cache,
        main_key=randn(rows, hkv, d), main_value=randn(rows, hkv, d),
        main_key_cache=w.k_cache, main_value_cache=w.v_cache,
        main_slots=main_slots.to(dev), num_index_heads=hi, index_head_dim=di,
        rotary_dim=rotary_dim, compress_ratio=r)


__all__ = ["CONFIGS", "SyntheticQSA", "make_prepare_inputs", "make_workload", "rope_cache"]
