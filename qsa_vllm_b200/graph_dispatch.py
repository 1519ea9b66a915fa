"""Context-length CUDA-graph buckets for QSA decode (drop-in for graph_dispatch.py).

The decode indexer writes ``columns`` fp32 logits per row, and the decode
launch grid depends on that width, so a captured decode graph is specific to
it.  As in the reference (graph_dispatch.py:16-100), every FULL decode graph
is captured twice: once for ``SHORT_DECODE_COLUMNS`` (32768 compressed
columns = 131072 tokens at ratio 4) and once for the page-table capacity
(``0``).  At run time the bucket is chosen from the batch's longest sequence.

``decode_logits_columns`` is what the indexer host code calls; the
``install_short_decode_dispatch`` patch wires the buckets into vLLM's graph
manager.  The patch targets are vLLM 0.30 internals
(``vllm.v1.worker.gpu.cudagraph_utils``, ``GPUModelRunner``); they can also be
passed explicitly, which is how the patch logic is tested without vLLM.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import asdict, make_dataclass

SHORT_DECODE_COLUMNS = 32768

_state = {"runtime_columns": 0, "capture_columns": None}


def decode_column_bucket(max_seq_len: int, compress_ratio: int = 4) -> int:
    """32768 when the longest row fits the short bucket, else 0 (= full capacity)."""
    return SHORT_DECODE_COLUMNS if max_seq_len // compress_ratio <= SHORT_DECODE_COLUMNS else 0


def decode_logits_columns(max_seq_len: int, compress_ratio: int, capacity: int) -> int:
    """Logits width of a decode step: the capture bucket while capturing, else
    the run-time bucket of ``max_seq_len``; 0 means the full ``capacity``."""
    cap_cols = _state["capture_columns"]
    columns = cap_cols if cap_cols is not None else decode_column_bucket(max_seq_len,
                                                                          compress_ratio)
    return min(columns, capacity) if columns else capacity


@contextmanager
def capture_column_scope(columns):
    """Pin the decode logits width for the forward passes run inside the scope."""
    previous = _state["capture_columns"]
    _state["capture_columns"] = columns
    try:
        yield
    finally:
        _state["capture_columns"] = previous


def runtime_columns() -> int:
    return _state["runtime_columns"]


def set_runtime_columns(max_seq_len: int | None) -> int:
    """Record the bucket of the batch about to run (0 when there is no batch)."""
    _state["runtime_columns"] = 0 if max_seq_len is None else decode_column_bucket(max_seq_len)
    return _state["runtime_columns"]


def install_short_decode_dispatch(model_graph_manager=None, graph_manager=None,
                                  model_runner=None, full_mode=None, descriptor_cls=None):
    """Patch vLLM's CUDA-graph manager so FULL decode graphs exist per column bucket.

    Patched: ``ModelCudaGraphManager._init_candidates`` (duplicate every FULL
    descriptor per bucket), ``.dispatch`` (pick the bucket's descriptor),
    ``CudaGraphManager.capture`` (run capture forwards inside
    ``capture_column_scope``) and ``GPUModelRunner.gather_batch_req_state``
    (record the bucket of the scheduled batch).
    """
    if model_graph_manager is None:
        from vllm.config.compilation import CUDAGraphMode
        from vllm.v1.worker.gpu.cudagraph_utils import (
            BatchExecutionDescriptor, CudaGraphManager, ModelCudaGraphManager)
        from vllm.v1.worker.gpu.model_runner import GPUModelRunner
        model_graph_manager, graph_manager, model_runner = (
            ModelCudaGraphManager, CudaGraphManager, GPUModelRunner)
        full_mode, descriptor_cls = CUDAGraphMode.FULL, BatchExecutionDescriptor

    bucket_desc = make_dataclass(
        "QSABatchExecutionDescriptor", [("qsa_columns", int, 0)], bases=(descriptor_cls,),
        frozen=True)

    original_init = model_graph_manager._init_candidates
    original_dispatch = model_graph_manager.dispatch
    original_capture = graph_manager.capture
    original_gather = model_runner.gather_batch_req_state

    def init_candidates(manager):
        original_init(manager)
        if full_mode in manager._capture_descs:
            manager._qsa_full_descs = {
                (desc, cols): bucket_desc(**asdict(desc), qsa_columns=cols)
                for desc in manager._capture_descs[full_mode]
                for cols in (0, SHORT_DECODE_COLUMNS)
            }
            manager._capture_descs[full_mode] = list(manager._qsa_full_descs.values())

    def dispatch(manager, *args, **kwargs):
        desc = original_dispatch(manager, *args, **kwargs)
        if desc.cg_mode == full_mode:
            desc = manager._qsa_full_descs[(desc, _state["runtime_columns"])]
        return desc

    def capture(manager, create_forward_fn, progress_bar_desc="Capturing CUDA graphs"):
        if not isinstance(manager, model_graph_manager):
            return original_capture(manager, create_forward_fn, progress_bar_desc)

        def create_bucket_forward(desc, warmup):
            cols = desc.qsa_columns if desc.cg_mode == full_mode else None
            with capture_column_scope(cols):
                forward = create_forward_fn(desc, warmup)

            def bucket_forward(mode):
                with capture_column_scope(cols):
                    return forward(mode)
            return bucket_forward

        return original_capture(manager, create_bucket_forward, progress_bar_desc)

    def gather(runner, scheduler_output, dummy_run):
        batch, uniform = original_gather(runner, scheduler_output, dummy_run)
        longest = None
        if batch is not None:
            lengths = (runner.req_states.num_computed_tokens_np[batch.idx_mapping_np]
                       + batch.num_scheduled_tokens)
            longest = int(lengths.max())
        set_runtime_columns(longest)
        return batch, uniform

    model_graph_manager._init_candidates = init_candidates
    model_graph_manager.dispatch = dispatch
    graph_manager.capture = capture
    model_runner.gather_batch_req_state = gather
    return bucket_desc


__all__ = [
    "SHORT_DECODE_COLUMNS", "decode_column_bucket", "decode_logits_columns",
    "capture_column_scope", "install_short_decode_dispatch", "runtime_columns",
    "set_runtime_columns",
]

