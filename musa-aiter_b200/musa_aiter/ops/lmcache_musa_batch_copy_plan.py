"""Validation and splitting of a host/device byte-copy batch (no torch dependency).

Same contract as the reference planner (musa_aiter/ops/lmcache_musa_batch_copy_plan.py:12-178):
sizes positive, offsets non-negative and inside each tensor, no two entries writing
overlapping bytes of one destination (the batch is unordered), and entries split
at host registration boundaries of ``pin_chunk_size`` bytes.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Hashable, Sequence


@dataclass(frozen=True)
class BatchCopyEntry:
    input_index: int
    source_offset: int
    destination_offset: int
    size: int
    host_registration_offset: int


@dataclass(frozen=True)
class BatchCopyPlan:
    direction: str
    entries: tuple[BatchCopyEntry, ...]
    total_bytes: int
    input_entry_count: int


def _ints(name: str, values: Sequence[int], n: int) -> tuple[int, ...]:
    if len(values) != n:
        raise ValueError(f"{name} must have the same length as sizes")
    out = []
    for v in values:
        if isinstance(v, bool) or not isinstance(v, int):
            raise ValueError(f"{name} must contain integers")
        out.append(v)
    return tuple(out)


def _keys(name: str, values: Sequence[Hashable] | None, n: int) -> tuple[Hashable, ...]:
    keys = tuple(range(n)) if values is None else tuple(values)
    if len(keys) != n:
        raise ValueError(f"{name} must have the same length as sizes")
    for k in keys:
        try:
            hash(k)
        except TypeError as exc:
            raise ValueError(f"{name} must contain hashable values") from exc
    return keys


def _reject_overlaps(dst_offsets: Sequence[int], sizes: Sequence[int], keys: Sequence[Hashable]) -> None:
    spans: dict[Hashable, list[tuple[int, int]]] = {}
    for off, size, key in zip(dst_offsets, sizes, keys):
        spans.setdefault(key, []).append((off, off + size))
    for ranges in spans.values():
        ranges.sort()
        for (_, end), (start, _) in zip(ranges, ranges[1:]):
            if start < end:
                raise ValueError("overlapping destination ranges are invalid in an unordered batch")


def build_batch_copy_plan(*, direction: str, sizes: Sequence[int], source_capacities: Sequence[int],
                          destination_capacities: Sequence[int], source_offsets: Sequence[int] | None = None,
                          destination_offsets: Sequence[int] | None = None,
                          host_registration_offsets: Sequence[int] | None = None, pin_chunk_size: int | None = None,
                          destination_keys: Sequence[Hashable] | None = None) -> BatchCopyPlan:
    if direction not in {"h2d", "d2h"}:
        raise ValueError("direction must be 'h2d' or 'd2h'")
    if pin_chunk_size is not None and (isinstance(pin_chunk_size, bool) or not isinstance(pin_chunk_size, int)
                                       or pin_chunk_size <= 0):
        raise ValueError("pin_chunk_size must be a positive integer")
    n = len(sizes)
    sz = _ints("sizes", sizes, n)
    scap = _ints("source_capacities", source_capacities, n)
    dcap = _ints("destination_capacities", destination_capacities, n)
    soff = _ints("source_offsets", [0] * n if source_offsets is None else source_offsets, n)
    doff = _ints("destination_offsets", [0] * n if destination_offsets is None else destination_offsets, n)
    hdefault = soff if direction == "h2d" else doff
    hoff = _ints("host_registration_offsets", hdefault if host_registration_offsets is None else host_registration_offsets, n)
    keys = _keys("destination_keys", destination_keys, n)
    for i in range(n):
        if sz[i] <= 0:
            raise ValueError(f"sizes[{i}] must be positive")
        if soff[i] < 0 or doff[i] < 0 or hoff[i] < 0:
            raise ValueError("copy offsets must be non-negative")
        if dcap[i] < 0 or doff[i] + sz[i] > dcap[i]:
            raise ValueError(f"destination range at index {i} exceeds tensor capacity")
        if scap[i] < 0 or soff[i] + sz[i] > scap[i]:
            raise ValueError(f"source range at index {i} exceeds tensor capacity")
    _reject_overlaps(doff, sz, keys)
    entries: list[BatchCopyEntry] = []
    for i in range(n):
        left, so, do, ho = sz[i], soff[i], doff[i], hoff[i]
        while left:
            take = left if pin_chunk_size is None else min(left, pin_chunk_size - ho % pin_chunk_size)
            entries.append(BatchCopyEntry(i, so, do, take, ho))
            left -= take
            so += take
            do += take
            ho += take
    return BatchCopyPlan(direction, tuple(entries), sum(sz), n)


def chunk_batch_copy_plan(plan: BatchCopyPlan, max_batch_entries: int) -> tuple[tuple[BatchCopyEntry, ...], ...]:
    """Split a validated plan into stream-ordered submissions of at most ``max_batch_entries``."""
    if isinstance(max_batch_entries, bool) or not isinstance(max_batch_entries, int) or max_batch_entries <= 0:
        raise ValueError("max_batch_entries must be a positive integer")
    return tuple(plan.entries[i: i + max_batch_entries] for i in range(0, len(plan.entries), max_batch_entries))
