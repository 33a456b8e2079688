"""Asynchronous host/device byte-copy batch for LMCache direct transfers.

Public contract of the reference (musa_aiter/ops/lmcache_musa_batch_copy.py:121-247):
validate, split at host registration boundaries, submit on the current stream in
order, return True when submitted.  The reference submits through the MUSA
batched-copy runtime call; here ``mak_memcpy_batch`` submits large entries to
the copy engines and batches small entries into one zero-copy kernel launch per
128 entries (pinned host memory is addressed directly).  ``prefer_overlap_with_compute``
keeps every entry on the copy engines so no SM time is taken.
"""

from __future__ import annotations

import ctypes
import os
from typing import Sequence

import torch

from .. import _native
from ..dispatch import emit_native
from .kv_backend import KVBackendCapabilities, KVBackendDecision, select_kv_backend
from .kv_transfer_plan import KVTransferPlan
from .lmcache_musa_batch_copy_plan import build_batch_copy_plan, chunk_batch_copy_plan

_ABI_VERSION = 1
_DEFAULT_MAX_BATCH_ENTRIES = 1024


def native_lmcache_musa_batch_copy_abi_version() -> int:
    return _ABI_VERSION


def native_lmcache_musa_batch_copy_runtime_versions() -> tuple[int, int] | None:
    """(runtime, driver) CUDA versions seen by the kernel library."""
    try:
        rt, drv = ctypes.c_int32(0), ctypes.c_int32(0)
        if _native.load().mak_runtime_versions(ctypes.byref(rt), ctypes.byref(drv)) != 0:
            return None
        return int(rt.value), int(drv.value)
    except Exception:
        return None


def is_native_lmcache_musa_batch_copy_available() -> bool:
    return _native.is_available() and torch.cuda.is_available()


def select_lmcache_batch_copy_backend(plan: KVTransferPlan, *, native_available: bool | None = None,
                                      require_native: bool = False) -> KVBackendDecision:
    """Classify an LMCache plan before submitting byte copies (reference :74-97)."""
    if native_available is None:
        native_available = is_native_lmcache_musa_batch_copy_available()
    return select_kv_backend(plan, capabilities=KVBackendCapabilities(direct_batch=bool(native_available), reference=True),
                             require_native=require_native)


def _kind(t: torch.Tensor) -> str:
    if t.device.type == "cpu":
        return "cpu"
    if t.device.type == "cuda":
        return "cuda"
    return "unsupported"


def _resolve_max_batch_entries(value: int | None) -> int:
    if value is not None:
        if isinstance(value, bool) or not isinstance(value, int) or value <= 0:
            raise ValueError("max_batch_entries must be a positive integer")
        return value
    configured = os.environ.get("MUSA_AITER_LMCACHE_BATCH_MAX_ENTRIES", str(_DEFAULT_MAX_BATCH_ENTRIES))
    try:
        v = int(configured)
    except ValueError as exc:
        raise ValueError("MUSA_AITER_LMCACHE_BATCH_MAX_ENTRIES must be an integer") from exc
    if v <= 0:
        raise ValueError("MUSA_AITER_LMCACHE_BATCH_MAX_ENTRIES must be positive")
    return v


def lmcache_musa_memcpy_batch_async(
    destinations: Sequence[torch.Tensor],
    sources: Sequence[torch.Tensor],
    sizes: Sequence[int],
    *,
    destination_offsets: Sequence[int] | None = None,
    source_offsets: Sequence[int] | None = None,
    host_registration_offsets: Sequence[int] | None = None,
    pin_chunk_size: int | None = None,
    require_pinned_host: bool = True,
    prefer_overlap_with_compute: bool = False,
    max_batch_entries: int | None = None,
) -> bool:
    """Submit host->device or device->host byte copies on the current CUDA stream.

    Returns True when submitted (or empty) and False for a device pairing this
    path does not serve (device<->device, host<->host), so the caller can use its
    own path, as in the reference.  Validation errors raise ValueError/TypeError.
    """
    destinations, sources, sizes = tuple(destinations), tuple(sources), tuple(sizes)
    n = len(sizes)
    if not destinations and not sources and not sizes:
        return True
    if len(destinations) != n or len(sources) != n:
        raise ValueError("destinations, sources, and sizes must have the same length")
    directions, devices = [], set()
    for i, (dst, src) in enumerate(zip(destinations, sources)):
        if not isinstance(dst, torch.Tensor) or not isinstance(src, torch.Tensor):
            raise TypeError("destinations and sources must contain torch.Tensor values")
        if not dst.is_contiguous() or not src.is_contiguous():
            raise ValueError("batch-copy tensors must be contiguous")
        pair = (_kind(src), _kind(dst))
        if pair == ("cpu", "cuda"):
            direction, host, dev = "h2d", src, dst
        elif pair == ("cuda", "cpu"):
            direction, host, dev = "d2h", dst, src
        else:
            return False
        if require_pinned_host and not host.is_pinned():
            raise ValueError(f"host tensor at index {i} must use pinned memory")
        directions.append(direction)
        devices.add((dev.device.type, dev.device.index))
    if len(set(directions)) != 1:
        raise ValueError("one batch cannot mix h2d and d2h copies")
    if len(devices) != 1:
        raise ValueError("all batch entries must use the same CUDA device")
    plan = build_batch_copy_plan(
        direction=directions[0], sizes=sizes,
        source_capacities=[t.numel() * t.element_size() for t in sources],
        destination_capacities=[t.numel() * t.element_size() for t in destinations],
        source_offsets=source_offsets, destination_offsets=destination_offsets,
        host_registration_offsets=host_registration_offsets, pin_chunk_size=pin_chunk_size,
        destination_keys=[id(t) for t in destinations],
    )
    lib = _native.load()
    dev_t = destinations[0] if directions[0] == "h2d" else sources[0]
    stream = _native.stream_ptr(dev_t.device)
    mode = _native.MAK_COPY_ENGINE if prefer_overlap_with_compute else _native.MAK_COPY_AUTO
    pageable = any(not (t.is_pinned() if t.device.type == "cpu" else True) for t in destinations + sources)
    if pageable:
        mode = _native.MAK_COPY_ENGINE  # the GPU cannot address pageable host memory; the copy engines stage it
    for chunk in chunk_batch_copy_plan(plan, _resolve_max_batch_entries(max_batch_entries)):
        arr = (_native.CopyEntry * len(chunk))()
        for k, e in enumerate(chunk):
            arr[k].dst = destinations[e.input_index].data_ptr() + e.destination_offset
            arr[k].src = sources[e.input_index].data_ptr() + e.source_offset
            arr[k].size = e.size
        _native.check(lib.mak_memcpy_batch(arr, len(chunk), mode, 0, stream), "lmcache_musa_memcpy_batch_async")
    emit_native("lmcache_musa_memcpy_batch_async", dev_t, f"{directions[0]} batch of {len(plan.entries)} entries")
    return True


def lmcache_musa_memcpy_batch_async_internal(destinations, sources, sizes, *, host_registration_offsets,
                                             pin_chunk_size, destination_offsets=None, source_offsets=None,
                                             require_pinned_host: bool = True, prefer_overlap_with_compute: bool = False,
                                             max_batch_entries: int | None = None) -> bool:
    """LMCache-only facade requiring an explicit host registration boundary (reference :207-240)."""
    if host_registration_offsets is None or pin_chunk_size is None:
        raise ValueError("LMCache internal API requires a host registration boundary")
    return lmcache_musa_memcpy_batch_async(
        destinations, sources, sizes, destination_offsets=destination_offsets, source_offsets=source_offsets,
        host_registration_offsets=host_registration_offsets, pin_chunk_size=pin_chunk_size,
        require_pinned_host=require_pinned_host, prefer_overlap_with_compute=prefer_overlap_with_compute,
        max_batch_entries=max_batch_entries,
    )
