"""Benchmark: one QSA layer decode step (indexer -> top-k -> sparse attention).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2_32k] [--impl ours|reference]

Workload (``--config``, default the headline ``cfg2_32k``): batch 64 decode
rows at 32768 tokens of context, 32 query / 4 KV heads of dim 128 (bf16),
indexer 8 heads x 64 with U(0,1) head weights, compress ratio 4, top-k 2048
tokens (512 blocks), page 64, seeded random block tables.  A step is the whole
QSA path of one layer for those 64 rows, run as vLLM runs decode: through the
drop-in operators (``select_paged_tokens`` + ``qsa_sparse_paged_attention``)
captured in a CUDA graph, with the per-step metadata the reference layer
receives (block tables, positions, sequence lengths and visible block counts,
reference attention.py:128-142).  Inputs are synthetic (seeded N(0,1) / U(0,1)).

Timing: W untimed warm-up steps, then K steps each bracketed by CUDA events on
the launching stream, with the L2 flushed before every step outside the
events (a 256 MiB write, then a 256 MiB read of another buffer so the timed
step does not pay for writing the flush's dirty lines back); max over ranks.  With ``--gpus N`` (torchrun, NCCL) the
heads are sharded across ranks as vLLM tensor parallelism does (no
collective inside the path; the indexer is replicated), so the total work is
fixed: ``value`` = rows / (max-over-ranks step time).

``e2e`` re-times the same step through the public Python API (captured in a
CUDA graph, as vLLM runs decode; the eager time is reported beside it) with the
step's inputs copied host->device from pinned memory and the attention output
copied back, inside the timed region.  ``roofline`` times the dominant kernel
(the main sparse-attention kernel) alone, through CUDA events the library
records on its stream right around that launch; the whole attention op (with
its split merge) is reported beside it.  ``cpu_baseline`` times the CPU oracle on a bounded
sample of rows on this host.  ``--impl reference`` runs the reference math
(the CPU oracle port, the only form of the reference's path that runs without
its vLLM 0.30 / SM80 stack) with all host threads.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "QSA decode tokens/s/GPU @32k ctx, top-k 2048; % HBM and tensor-pipe roofline"
UNIT = "tokens/s"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


def workload_desc(cfg: str, w) -> dict:
    c = w.extra["config"]
    return {
        "workload": (f"{cfg}: one QSA layer decode step (indexer + top-k + sparse attention), "
                     f"B={w.rows}, ctx {c['seq_len']}, H_q {c['hq']} / H_kv {c['hkv']} x d "
                     f"{c['d']} bf16, indexer {c['hi']}x{c['di']} (U(0,1) head weights), "
                     f"ratio {w.ratio}, top-k {w.token_topk} tokens, page {w.page_size}"),
        "global_batch": w.rows,
        "seq_len": c["seq_len"] if not isinstance(c["seq_len"], tuple) else list(c["seq_len"]),
        "l2": "flushed before every timed step (256 MiB write + 256 MiB read, outside the events)",
        "cuda_graph": True,
    }


def algorithmic_bytes(w) -> dict:
    """Bytes each stage must move at least once (no credit for cache reuse).

    attention: every selected token's K and V row of every KV head (2*d bf16
    each), its index, plus q, gate and out; indexer: every visible compressed
    key (d_i bf16) + the fp32 score written; top-k: scores read + ids written.
    """
    rows, hq, d = w.q.shape
    hkv = w.kv.shape[2]
    r = w.ratio
    k_blk = w.token_topk // r
    width = w.token_topk + r - 1
    pos1 = w.positions.long().cpu() + 1
    seq = w.seq_lens.long().cpu()[w.token_to_req.long().cpu()]
    vis = torch.minimum(pos1 // r, seq // r)
    complete = torch.clamp(vis, max=k_blk)
    count = torch.minimum(complete * r + (pos1 - (pos1 // r) * r), seq)
    sel = int(count.sum())
    vis_total = int(vis.sum())
    hi, di = w.index_q.shape[1], w.index_q.shape[2]
    att = sel * hkv * 2 * d * 2 + sel * 4 + 3 * rows * hq * d * 2
    idx = vis_total * di * 2 + rows * hi * di * 2 + vis_total * 4
    topk = vis_total * 4 + rows * width * 4
    return {"attention": att, "indexer": idx, "topk": topk, "rows": rows,
            "attention_flops": sel * hq * d * 4, "indexer_flops": vis_total * hi * di * 2}


class ClockSampler:
    """SM clock and clock-event (throttle) reasons of one GPU, sampled through
    NVML every ~2 ms on a background thread while the timed region runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device: torch.device, period_s: float = 0.002):
        self.device = device
        self.period = period_s
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self._stop = None
        self._thread = None
        self._nvml = None
        self._handle = None

    def _open(self):
        import pynvml as N
        N.nvmlInit()
        props = torch.cuda.get_device_properties(self.device)
        try:
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            h = N.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            h = N.nvmlDeviceGetHandleByIndex(self.device.index or 0)
        self._nvml, self._handle = N, h
        self.max_mhz = float(N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM))

    def _reasons(self) -> int:
        N, h = self._nvml, self._handle
        fn = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
            N.nvmlDeviceGetCurrentClocksThrottleReasons
        return int(fn(h))

    def _run(self):
        import time as _t
        N, h = self._nvml, self._handle
        while not self._stop.is_set():
            try:
                self.samples.append((float(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)),
                                     self._reasons()))
            except Exception:
                pass
            _t.sleep(self.period)

    def __enter__(self):
        import threading
        try:
            self._open()
        except Exception:
            self._nvml = None
            return self
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._thread is not None:
            self._stop.set()
            self._thread.join(timeout=5)

    def summary(self) -> dict | None:
        if not self.samples:
            return None
        reasons = sorted({name for _, bits in self.samples for b, name in self.REASONS.items()
                          if bits & b})
        return {"sm_mhz": statistics.median(c for c, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples),
                "source": "NVML, every 2 ms during the timed region"}


def oracle_sample(cfg: str, rows: int):
    """A CPU workload with ``rows`` rows of ``cfg``'s per-row shapes and the
    oracle step that runs it: decode rows are ``rows`` requests; prefill rows
    are the last ``rows`` new tokens of one request (same context and causal
    visibility as the configuration's chunk ends)."""
    from oracle import qsa_oracle as O
    from qsa_vllm_b200.synthetic import CONFIGS, make_workload
    if CONFIGS[cfg].get("new_tokens") is None:
        return make_workload(cfg, device="cpu", seed=0, batch=rows), O.decode_step, "decode_step"
    w = make_workload(cfg, device="cpu", seed=0, batch=1, new_tokens=rows)
    return w, O.prefill_step, "prefill_step"


def cpu_baseline(cfg: str, rows: int = 4, min_seconds: float = 10.0) -> dict:
    """The CPU oracle on a bounded sample: ``rows`` rows of the same workload."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w, step, name = oracle_sample(cfg, rows)
    step(w)
    n, t0 = 0, time.perf_counter()
    while True:
        step(w)
        n += 1
        el = time.perf_counter() - t0
        if el >= min_seconds or n >= 5000:
            break
    return {"value": rows * n / el, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{rows} of the workload's rows ({cfg} per-row shapes) x {n} passes "
                      f"of oracle.{name}, {el:.1f} s"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    rows = args.ref_rows
    w, step, name = oracle_sample(args.config, rows)
    for _ in range(args.warmup):
        step(w)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        step(w)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = rows * args.steps / total
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": f"{args.config} per-row shapes, {rows} rows per step "
                               "(bounded CPU sample)", "global_batch": rows},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{rows} rows per step of {args.config} through the CPU "
                                   "oracle (reference math restated in PyTorch eager)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg2_32k")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ref-rows", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        run_reference(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)

    from qsa_vllm_b200 import _lib
    from qsa_vllm_b200.indexer import compute_visible_blocks, select_paged_tokens
    from qsa_vllm_b200.qsa import qsa_sparse_paged_attention
    from qsa_vllm_b200.synthetic import make_workload

    full = make_workload(args.config, device=dev, seed=args.seed)
    w = full.shard_heads(world, rank) if world > 1 else full
    del full
    rows = w.rows
    width = w.token_topk + w.ratio - 1
    idx_buf = torch.empty(rows, width, dtype=torch.int32, device=dev)
    cnt_buf = torch.empty(rows, dtype=torch.int32, device=dev)
    out = torch.empty_like(w.q)
    flush_w = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    flush_r = torch.ones(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def flush_l2():
        flush_w.zero_()   # evicts the previous step's lines (leaves dirty flush lines) ...
        flush_r.sum()     # ... which a clean read then writes back, outside the timed region

    # Per-step metadata, as the reference layer receives it: visible_blocks
    # comes with vLLM's compressed-cache metadata (reference attention.py:139),
    # built once per step for every QSA layer, like the block tables.
    w.visible_blocks = compute_visible_blocks(w.positions, w.seq_lens, w.token_to_req, w.ratio)

    def step():
        select_paged_tokens(
            w.index_q, w.index_cache, w.index_table, w.token_to_req, w.positions, w.seq_lens,
            w.token_topk, w.ratio, idx_buf, **w.select_kwargs(),
            visible_blocks=w.visible_blocks,
            main_block_table=w.block_table, main_page_size=w.page_size, valid_counts_out=cnt_buf,
            weights=w.index_weights, scale=w.index_scale)
        qsa_sparse_paged_attention(w.q, w.k_cache, w.v_cache, idx_buf, w.block_table,
                                   w.token_to_req, out, output_gate=w.gate,
                                   use_decode_kernel=True, indices_are_physical=True,
                                   valid_counts=cnt_buf)

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    # kernels of one step, counted by the library at each launch (the graph
    # replays exactly these)
    n0 = _lib.kernel_launches()
    step()
    launches_per_step = _lib.kernel_launches() - n0
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(dev)

    def timed(fn, k):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(k)]
        for a, b in evs:
            flush_l2()
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize(dev)
        return sum(a.elapsed_time(b) for a, b in evs) / k   # ms per step

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---- device-timed step (CUDA graph replay)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(dev) as clocks:
        ms = timed(graph.replay, args.steps)
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    ms = max_over_ranks(ms)
    value = rows / (ms * 1e-3)

    # ---- dominant kernel alone: the main sparse-attention kernel (and the op with its merge)
    def attn():
        qsa_sparse_paged_attention(w.q, w.k_cache, w.v_cache, idx_buf, w.block_table,
                                   w.token_to_req, out, output_gate=w.gate,
                                   use_decode_kernel=True, indices_are_physical=True,
                                   valid_counts=cnt_buf)
    attn()
    # the op (main kernel + split merge) as the library runs it: a graph with
    # no timing nodes, so the merge still launches early behind the main
    # kernel (programmatic dependent launch)
    op_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(op_graph):
        attn()
    op_graph.replay()
    ms_attn_op = max_over_ranks(timed(op_graph.replay, args.steps))
    del op_graph
    # the library records ev_kernel[0] / [1] on the stream right around the
    # main attention kernel (before the split merge); the graph keeps them
    ev_kernel = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
    _lib.set_attention_timing_events(*ev_kernel)
    attn_graph = torch.cuda.CUDAGraph()   # replayed: no host launch gaps inside the events
    try:
        with torch.cuda.graph(attn_graph):
            attn()
    finally:
        _lib.set_attention_timing_events(None, None)
    attn_graph.replay()
    kernel_ms = []
    for _ in range(args.steps):
        flush_l2()
        attn_graph.replay()
        torch.cuda.synchronize(dev)
        kernel_ms.append(ev_kernel[0].elapsed_time(ev_kernel[1]))
    ms_attn = max_over_ranks(sum(kernel_ms) / len(kernel_ms))

    # ---- end to end through the public API with host buffers
    # The step's inputs live in persistent device buffers (typed views,
    # 256-byte aligned) mirrored by pinned host buffers, as vLLM stages its
    # per-step inputs.  Two staging groups copied concurrently at the step's
    # start: the indexer's inputs (metadata, index queries) on the main
    # stream, the attention-only inputs (q, gate) on a second stream while the
    # indexer and top-k run; attention waits for them.  One device->host copy
    # of the output.
    def stage(names):
        names = [n for n in names if getattr(w, n) is not None]
        offs, total = [], 0
        for n in names:
            t = getattr(w, n)
            offs.append(total)
            total += (t.numel() * t.element_size() + 255) // 256 * 256
        d = torch.empty(total, dtype=torch.uint8, device=dev)
        h = torch.empty(total, dtype=torch.uint8).pin_memory()
        for n, o in zip(names, offs):
            t = getattr(w, n)
            nbytes = t.numel() * t.element_size()
            view = d[o:o + nbytes].view(t.dtype).view(t.shape)
            view.copy_(t)
            h[o:o + nbytes].copy_(view.view(torch.uint8).view(-1).cpu())
            setattr(w, n, view)   # the step now reads its inputs from the staged buffer
        return d, h
    dev_meta, host_meta = stage(("index_q", "index_weights", "positions", "seq_lens",
                                 "token_to_req", "visible_blocks", "block_table",
                                 "index_table"))
    dev_qg, host_qg = stage(("q", "gate"))
    host_out = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    h2d = dev_meta.numel() + dev_qg.numel()
    d2h = host_out.numel() * host_out.element_size()
    side = torch.cuda.Stream(dev)
    step_start = torch.cuda.Event()
    qg_ready = torch.cuda.Event()

    def e2e_step():
        main = torch.cuda.current_stream(dev)
        # both host->device copies start at once, on two streams: the
        # indexer's inputs on the main stream, q and gate on the side stream
        # (after the previous step's attention, which step_start orders),
        # overlapped with the indexer and top-k
        step_start.record(main)
        side.wait_event(step_start)
        with torch.cuda.stream(side):
            dev_qg.copy_(host_qg, non_blocking=True)
            qg_ready.record(side)
        dev_meta.copy_(host_meta, non_blocking=True)
        select_paged_tokens(
            w.index_q, w.index_cache, w.index_table, w.token_to_req, w.positions, w.seq_lens,
            w.token_topk, w.ratio, idx_buf, **w.select_kwargs(),
            visible_blocks=w.visible_blocks,
            main_block_table=w.block_table, main_page_size=w.page_size, valid_counts_out=cnt_buf,
            weights=w.index_weights, scale=w.index_scale)
        main.wait_event(qg_ready)
        qsa_sparse_paged_attention(w.q, w.k_cache, w.v_cache, idx_buf, w.block_table,
                                   w.token_to_req, out, output_gate=w.gate,
                                   use_decode_kernel=True, indices_are_physical=True,
                                   valid_counts=cnt_buf)
        host_out.copy_(out, non_blocking=True)
    e2e_step()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    ms_e2e_eager = max_over_ranks(timed(e2e_step, args.steps))
    # as vLLM runs decode: the step's copies and kernels captured in one graph
    e2e_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(e2e_graph):
        e2e_step()
    e2e_graph.replay()
    torch.cuda.synchronize(dev)
    if dist is not None:
        dist.barrier()
    ms_e2e = max_over_ranks(timed(e2e_graph.replay, args.steps))
    e2e_value = rows / (ms_e2e * 1e-3)

    ab = algorithmic_bytes(w)
    pk, pk_kind = peaks()
    achieved = ab["attention"] / (ms_attn * 1e-3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "attention_cfg2_32k_traffic.json"
    if tf.exists() and world == 1 and args.config == "cfg2_32k":
        traffic = json.loads(tf.read_text()).get("dram_bytes_per_launch")

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.config)
    if dist is not None:
        del graph, attn_graph, e2e_graph
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "value_note": "value = all ranks' rows / max-over-ranks step time (whole job)",
        "per_gpu": {"value": value / world, "unit": "tokens/s per GPU"},
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {**workload_desc(args.config, w),
                   "parallelism": f"tp{world} head-sharded (indexer replicated)"},
        "roofline": {
            "kernel": "attention_kernel (paged K/V gather + online softmax, stream-K split)",
            "bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"], "peak_kind": pk_kind,
            "algorithmic_bytes_per_launch": ab["attention"], "ms_per_launch": ms_attn,
            "timing": "CUDA events the library records on the launching stream right "
                      "around the main kernel, inside a replayed graph, L2 flushed before "
                      "each replay",
            "op_ms_per_launch": ms_attn_op,
            "op_timing": "replay of a graph of the op alone (main kernel + split merge, no "
                         "timing nodes), L2 flushed before each replay",
            "op_frac": ab["attention"] / (ms_attn_op * 1e-3) / 1e9 / pk["hbm_gbs"],
            "traffic": traffic},
        "stage_bytes": {k: ab[k] for k in ("attention", "indexer", "topk")},
        "step_hbm_frac": (ab["attention"] + ab["indexer"] + ab["topk"]) / (ms * 1e-3) / 1e9
        / pk["hbm_gbs"],
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e,
                "api": "select_paged_tokens + qsa_sparse_paged_attention with the step's "
                       "pinned-host -> device input copies (indexer inputs on the main "
                       "stream and q and gate on a second stream, both from the step's "
                       "start, overlapped with the indexer and top-k) and "
                       "the device -> host output copy, captured in one CUDA graph as vLLM "
                       "runs decode",
                "eager_ms_per_step": ms_e2e_eager},
        "gpu_launches": launches_per_step * args.steps,
        "gpu_launches_per_step": launches_per_step,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
