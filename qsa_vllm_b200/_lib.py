"""ctypes binding of the sm_100a C-ABI library ``libqsa_b200.so``.

The library is built in-tree by ``python -m qsa_vllm_b200.build`` (also run by
``__graft_entry__.build()``).  There is no fallback: if the library is missing
or the device is not an sm_100 GPU, every operator raises ``QSAError``.
"""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libqsa_b200.so")


class QSAError(RuntimeError):
    """A C-ABI call returned a non-zero status (or the library is unavailable)."""


_vp, _i32, _i64, _f32, _sz = C.c_void_p, C.c_int32, C.c_int64, C.c_float, C.c_size_t

# Exported symbols of include/qsa_b200.h: name -> (restype, argtypes)
SIGNATURES: dict[str, tuple] = {
    "qsa_status_string": (C.c_char_p, [C.c_int]),
    "qsa_last_error": (C.c_char_p, []),
    "qsa_version": (C.c_char_p, []),
    "qsa_kernel_launches": (C.c_uint64, []),
    "qsa_set_attention_timing_events": (C.c_int, [_vp, _vp]),
    "qsa_device_check": (C.c_int, []),
    "qsa_device_error_poll": (C.c_int, [C.POINTER(_i32)]),
    "qsa_selftest_wait_timeout": (C.c_int, [C.c_void_p]),
    "qsa_topk_expand": (C.c_int, [
        _vp, _i64, _i32, _i32, _vp, _vp, _vp, _i32, _vp, _vp, _i64, _i32,
        _vp, _i64, _i64, _i32, _vp, _i32, _i32, _i32, _vp]),
    "qsa_topk": (C.c_int, [_vp, _i64, _i32, _i32, _vp, _vp, _i64, _i32, _vp]),
    "qsa_indexer_scores": (C.c_int, [
        _vp, _i64, _i64, _i32, _i32, _vp, _i64, _i64, _i32, _i32, _vp, _i64, _i32, _i32,
        _vp, _vp, _vp, _i32, _vp, _i32,
        _vp, _i32, _i32, _i32, _i32, _vp, _i64, _i64, _f32, _vp, _i64, _i32, _vp]),
    "qsa_select_decode": (C.c_int, [
        _vp, _i64, _i64, _i32, _i32, _vp, _i64, _i64, _i32, _i32, _vp, _i64, _i32, _i32,
        _vp, _vp, _vp, _i32, _vp, _i32, _i32, _i32, _vp, _i64, _i64, _f32, _i32,
        _vp, _i64, _i32, _i32, _i32, _vp, _i64, _i64, _i32, _vp, _vp, _i64, _vp]),
    "qsa_visible_blocks": (C.c_int, [_vp, _vp, _i32, _vp, _i32, _i32, _vp, _vp]),
    "qsa_sparse_attention_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32, _i32]),
    "qsa_sparse_attention": (C.c_int, [
        _vp, _i64, _i64, _i32, _i32, _i32,
        _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _i32, _i32,
        _vp, _i64, _i32, _vp, _i64, _i32, _i32, _vp, _vp,
        _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i32, _i32, _vp, _sz, _vp]),
    "qsa_prepare": (C.c_int, [
        _vp, _i64, _i32, _i32, _i32, _vp, _i64,
        _vp, _vp, _vp, _i64, _i32, _f32, _vp,
        _vp, _i64, _i64, _i64, _i32, _vp, _vp, _i64, _vp, _i32, _vp,
        _vp, _i64, _i64, _i64, _i32, _vp, _vp, _i32, _i32,
        _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64,
        _vp, _i64, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i64,
        _i64, _i32, _vp, _i32, _i32, _vp]),
    "qsa_sparse_attention_static_scratch": (C.c_int, [
        _vp, _i64, _i64, _i32, _i32, _i32,
        _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i64, _i32, _i32, _i32,
        _vp, _i64, _i32, _vp, _i64, _i32, _i32, _vp, _vp,
        _vp, _i64, _i64, _i64, _vp, _i64, _i64, _i32, _i32, _vp]),
}

_lib: C.CDLL | None = None
_checked_devices: set[int] = set()


def load_library() -> C.CDLL:
    """Load (once) and return the C-ABI library, with argument types declared."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise QSAError(
                f"{LIB_PATH.name} is not built; run `python -m qsa_vllm_b200.build` "
                "(there is no CPU or Triton fallback)")
        lib = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(status: int, what: str = "") -> None:
    if status != 0:
        lib = load_library()
        msg = lib.qsa_last_error().decode(errors="replace")
        name = lib.qsa_status_string(status).decode()
        raise QSAError(f"{what or 'qsa'}: {name} ({status}): {msg}")


def ensure_device(device: torch.device) -> None:
    """Fail loudly unless ``device`` is an sm_100 CUDA device."""
    if device.type != "cuda":
        raise QSAError(f"QSA operators run on sm_100 CUDA devices only, got {device}")
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx in _checked_devices:
        return
    lib = load_library()
    with torch.cuda.device(idx):
        check(lib.qsa_device_check(), "device check")
    _checked_devices.add(idx)


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def device_error_poll() -> int:
    """Read-and-clear the device error word (synchronous).  0 means no error."""
    lib = load_library()
    v = _i32(0)
    check(lib.qsa_device_error_poll(C.byref(v)), "device error poll")
    return int(v.value)


def version() -> str:
    return load_library().qsa_version().decode()


def set_attention_timing_events(before, after) -> None:
    """Have the library record two ``torch.cuda.Event``s around the main
    attention kernel of later attention calls on this thread (None, None
    clears)."""
    lib = load_library()

    def handle(e):
        if e is None:
            return None
        if not e.cuda_event:   # torch creates the CUDA event at its first record
            e.record()
        return e.cuda_event
    check(lib.qsa_set_attention_timing_events(handle(before), handle(after)), "timing events")


def kernel_launches() -> int:
    """Kernels launched (or recorded into CUDA graphs) by the library so far."""
    return int(load_library().qsa_kernel_launches())
