"""Decode logits-width buckets for CUDA-graph capture (drop-in for the plugin's
graph_dispatch.py, reference graph_dispatch.py:16-100).

Why buckets exist.  The decode indexer writes one fp32 score per visible
compressed block and row, into a logits buffer ``columns`` wide; its launch
grid is derived from that width.  A captured decode graph therefore bakes in
one width.  Two widths cover every batch:

* ``SHORT_DECODE_COLUMNS`` (32768 compressed blocks, 131072 tokens at ratio 4)
  for batches whose longest sequence fits it, and
* the page-table capacity (bucket value ``0``) for everything longer.

This module keeps the bucket bookkeeping in one ``_Buckets`` object owned by
the module (never on vLLM's objects):

* ``pinned`` -- the width forced while a graph for a given bucket is captured
  (``None`` outside capture);
* ``current`` -- the bucket of the batch about to run, recorded when the runner
  gathers the batch's request state;
* ``variants`` -- per graph manager (weakly keyed), the bucketed copy of each
  FULL-graph descriptor.

``decode_logits_columns`` is what the indexer host code calls.
``install_short_decode_dispatch`` attaches the buckets to vLLM's graph
machinery.  Its targets are vLLM 0.30 internals (``ModelCudaGraphManager``,
``CudaGraphManager`` in ``vllm.v1.worker.gpu.cudagraph_utils`` and
``GPUModelRunner``); they can be passed in explicitly, which is how the logic
is tested without vLLM.
"""

from __future__ import annotations

import dataclasses
import weakref
from contextlib import contextmanager

# Width of the short-context bucket, in compressed blocks (the reference's
# constant: captured graphs must agree with the plugin's).
SHORT_DECODE_COLUMNS = 32768
# Every FULL decode graph is captured once per bucket value (0 = capacity).
BUCKET_VALUES = (0, SHORT_DECODE_COLUMNS)


class _Buckets:
    def __init__(self) -> None:
        self.pinned: int | None = None
        self.current: int = 0
        self.variants: "weakref.WeakKeyDictionary[object, dict]" = weakref.WeakKeyDictionary()


_BUCKETS = _Buckets()


def decode_column_bucket(max_seq_len: int, compress_ratio: int = 4) -> int:
    """Bucket of a batch: the short bucket when its longest row's compressed
    length fits it, else 0 (the page-table capacity)."""
    if max_seq_len // compress_ratio <= SHORT_DECODE_COLUMNS:
        return SHORT_DECODE_COLUMNS
    return 0


def decode_logits_columns(max_seq_len: int, compress_ratio: int, capacity: int) -> int:
    """Logits width for a decode step.

    While a graph is captured for a bucket, that bucket decides; otherwise the
    bucket of ``max_seq_len``.  Bucket 0, or a bucket wider than the table,
    gives ``capacity``."""
    bucket = _BUCKETS.pinned
    if bucket is None:
        bucket = decode_column_bucket(max_seq_len, compress_ratio)
    if bucket == 0:
        return capacity
    return min(bucket, capacity)


@contextmanager
def capture_column_scope(columns):
    """Forward passes run inside the scope use bucket ``columns`` (``None``
    restores the run-time choice)."""
    saved = _BUCKETS.pinned
    _BUCKETS.pinned = columns
    try:
        yield
    finally:
        _BUCKETS.pinned = saved


def runtime_columns() -> int:
    """Bucket recorded for the batch about to run."""
    return _BUCKETS.current


def set_runtime_columns(max_seq_len: int | None) -> int:
    """Record the bucket of the batch about to run (0 when there is no batch)."""
    _BUCKETS.current = 0 if max_seq_len is None else decode_column_bucket(max_seq_len)
    return _BUCKETS.current


def batch_longest_sequence(runner, batch) -> int | None:
    """Longest sequence of a scheduled batch once its new tokens are counted.

    Length source (vLLM 0.30 runner state): per request, the tokens already
    computed (``runner.req_states.num_computed_tokens_np``, indexed through the
    batch's ``idx_mapping_np``) plus the tokens scheduled this step
    (``batch.num_scheduled_tokens``)."""
    if batch is None:
        return None
    computed = runner.req_states.num_computed_tokens_np[batch.idx_mapping_np]
    return int((computed + batch.num_scheduled_tokens).max())


class _PinnedForward:
    """A capture forward that runs with its graph's bucket pinned."""

    def __init__(self, forward, columns):
        self._forward = forward
        self._columns = columns

    def __call__(self, *args, **kwargs):
        with capture_column_scope(self._columns):
            return self._forward(*args, **kwargs)


class _BucketedFactory:
    """Wraps vLLM's ``create_forward_fn(desc, warmup)``: FULL descriptors carry
    their bucket, and both building the forward and every call of it see that
    bucket (other modes keep the run-time choice)."""

    def __init__(self, create_forward_fn, full_mode):
        self._create = create_forward_fn
        self._full = full_mode

    def __call__(self, desc, warmup):
        columns = desc.logits_columns if desc.cg_mode == self._full else None
        with capture_column_scope(columns):
            forward = self._create(desc, warmup)
        return _PinnedForward(forward, columns)


def _bucketed_descriptor_type(descriptor_cls):
    """Subclass of vLLM's (frozen dataclass) batch descriptor with one more
    field, so the two buckets' graphs are keyed apart."""
    return dataclasses.make_dataclass(
        "QSABucketedDescriptor", [("logits_columns", int, 0)], bases=(descriptor_cls,),
        frozen=True)


def install_short_decode_dispatch(model_graph_manager=None, graph_manager=None,
                                  model_runner=None, full_mode=None, descriptor_cls=None):
    """Make vLLM capture and replay one FULL decode graph per logits bucket.

    Four methods are wrapped (the names and signatures are vLLM 0.30's):

    * ``ModelCudaGraphManager._init_candidates(self)``: each FULL capture
      descriptor is replaced by one bucketed copy per ``BUCKET_VALUES`` entry;
    * ``ModelCudaGraphManager.dispatch(self, *a, **kw)``: a FULL result is
      swapped for its copy in the recorded run-time bucket;
    * ``CudaGraphManager.capture(self, create_forward_fn, progress_bar_desc)``:
      for the model manager, forwards are created and run with their bucket
      pinned (``_BucketedFactory``);
    * ``GPUModelRunner.gather_batch_req_state(self, scheduler_output,
      dummy_run)``: records the bucket of the gathered batch.

    Returns the bucketed descriptor type.
    """
    if model_graph_manager is None:
        from vllm.config.compilation import CUDAGraphMode
        from vllm.v1.worker.gpu.cudagraph_utils import (
            BatchExecutionDescriptor, CudaGraphManager, ModelCudaGraphManager)
        from vllm.v1.worker.gpu.model_runner import GPUModelRunner
        model_graph_manager, graph_manager = ModelCudaGraphManager, CudaGraphManager
        model_runner, full_mode = GPUModelRunner, CUDAGraphMode.FULL
        descriptor_cls = BatchExecutionDescriptor
    bucketed = _bucketed_descriptor_type(descriptor_cls)
    base = {
        "init": model_graph_manager._init_candidates,
        "dispatch": model_graph_manager.dispatch,
        "capture": graph_manager.capture,
        "gather": model_runner.gather_batch_req_state,
    }

    def _init_candidates(manager):
        base["init"](manager)
        descs = manager._capture_descs
        if full_mode not in descs:
            return
        table: dict = {}
        expanded = []
        for desc in descs[full_mode]:
            fields = {f.name: getattr(desc, f.name) for f in dataclasses.fields(desc)}
            per_bucket = {cols: bucketed(**fields, logits_columns=cols) for cols in BUCKET_VALUES}
            table[desc] = per_bucket
            expanded.extend(per_bucket.values())
        _BUCKETS.variants[manager] = table
        descs[full_mode] = expanded

    def _dispatch(manager, *args, **kwargs):
        desc = base["dispatch"](manager, *args, **kwargs)
        if desc.cg_mode != full_mode:
            return desc
        return _BUCKETS.variants[manager][desc][_BUCKETS.current]

    def _capture(manager, create_forward_fn, progress_bar_desc="Capturing CUDA graphs"):
        if isinstance(manager, model_graph_manager):
            create_forward_fn = _BucketedFactory(create_forward_fn, full_mode)
        return base["capture"](manager, create_forward_fn, progress_bar_desc)

    def _gather(runner, scheduler_output, dummy_run):
        batch, uniform = base["gather"](runner, scheduler_output, dummy_run)
        set_runtime_columns(batch_longest_sequence(runner, batch))
        return batch, uniform

    model_graph_manager._init_candidates = _init_candidates
    model_graph_manager.dispatch = _dispatch
    graph_manager.capture = _capture
    model_runner.gather_batch_req_state = _gather
    return bucketed


__all__ = [
    "BUCKET_VALUES", "SHORT_DECODE_COLUMNS", "batch_longest_sequence", "capture_column_scope",
    "decode_column_bucket", "decode_logits_columns", "install_short_decode_dispatch",
    "runtime_columns", "set_runtime_columns",
]
