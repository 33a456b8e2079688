"""Transfer plans: byte-range entries between two KV layouts, plus the slot-mapping
plan builder.

``KVTransferEntry`` / ``KVTransferPlan`` / ``validate_transfer_plan`` /
``assess_direct_eligibility`` keep the reference contract
(musa_aiter/ops/kv_transfer_plan.py:11-90).  The builders below are this
backend's plan builder: slot mappings come from block tables on the device
(``mak_build_slot_mapping``), and ``plan_slot_runs`` coalesces a slot mapping
into maximal contiguous runs (the byte ranges a direct batch copy needs).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal

import torch

from .kv_layout import KVLayoutKind, KVLayoutSpec, KVScaleKind

TransferDirection = Literal["h2d", "d2h", "d2d"]


@dataclass(frozen=True)
class KVTransferEntry:
    src_offset_bytes: int
    dst_offset_bytes: int
    nbytes: int
    layer: int = 0
    block: int = 0
    kv_plane: int = 0


@dataclass(frozen=True)
class KVTransferPlan:
    source: KVLayoutSpec
    destination: KVLayoutSpec
    direction: TransferDirection
    num_tokens: int
    skip_prefix_n_tokens: int
    entries: tuple[KVTransferEntry, ...]
    stream_id: int | None
    direct_eligible: bool
    direct_reject_reason: str | None


def validate_transfer_plan(plan: KVTransferPlan) -> KVTransferPlan:
    """Field checks plus: no two entries may write overlapping destination bytes."""
    if plan.direction not in {"h2d", "d2h", "d2d"}:
        raise ValueError(f"unsupported transfer direction={plan.direction!r}")
    if plan.num_tokens < 0:
        raise ValueError("num_tokens must be non-negative")
    if not 0 <= plan.skip_prefix_n_tokens <= plan.num_tokens:
        raise ValueError("skip_prefix_n_tokens must be within num_tokens")
    if plan.stream_id is not None and plan.stream_id < 0:
        raise ValueError("stream_id must be non-negative")
    spans = []
    for e in plan.entries:
        if e.src_offset_bytes < 0 or e.dst_offset_bytes < 0:
            raise ValueError("transfer offsets must be non-negative")
        if e.nbytes <= 0:
            raise ValueError("transfer nbytes must be positive")
        if e.layer < 0 or e.block < 0 or e.kv_plane < 0:
            raise ValueError("transfer indices must be non-negative")
        spans.append((e.dst_offset_bytes, e.dst_offset_bytes + e.nbytes))
    spans.sort()
    for (_, end_prev), (start, _) in zip(spans, spans[1:]):
        if start < end_prev:
            raise ValueError("destination transfer ranges overlap")
    return plan


_PAGE_KINDS = {KVLayoutKind.PAGE_FIRST, KVLayoutKind.PAGE_FIRST_DIRECT, KVLayoutKind.PAGE_HEAD}


def assess_direct_eligibility(source: KVLayoutSpec, destination: KVLayoutSpec) -> tuple[bool, str | None]:
    """Whether a plain byte-range copy can move data between the two layouts (and why not)."""
    if source.requires_layout_transform or destination.requires_layout_transform:
        return False, "layout transform is required"
    if not source.is_contiguous or not destination.is_contiguous:
        return False, "layout is not contiguous"
    if source.dtype_name != destination.dtype_name:
        return False, "dtype transform is required"
    if source.organization != destination.organization:
        return False, "K/V organization transform is required"
    if source.scale_kind is not KVScaleKind.NONE or destination.scale_kind is not KVScaleKind.NONE:
        return False, "scale transform is required"
    if source.kind in _PAGE_KINDS or destination.kind in _PAGE_KINDS:
        return False, "page layout transform is required"
    return True, None


# ---------------------------------------------------------------------------
# plan builder
# ---------------------------------------------------------------------------


def build_slot_mapping(block_tables: torch.Tensor, seq_lens: torch.Tensor, block_size: int,
                       max_seq_len: int | None = None) -> torch.Tensor:
    """Dense ``[B * S]`` int64 slot mapping from block tables (``-1`` past each sequence).

    Runs ``mak_build_slot_mapping`` on the block tables' CUDA device (one kernel,
    no host loop); ``max_seq_len`` defaults to ``max(seq_lens)`` (one host read).
    """
    import ctypes  # noqa: F401

    from .. import _native
    from ._common import require_cuda

    if block_tables.dim() != 2 or seq_lens.dim() != 1 or seq_lens.shape[0] != block_tables.shape[0]:
        raise ValueError("build_slot_mapping: block_tables must be [batch, max_blocks] and seq_lens [batch]")
    require_cuda("build_slot_mapping", block_tables, seq_lens)
    bt = block_tables if block_tables.dtype in (torch.int32, torch.int64) else block_tables.to(torch.int32)
    sl = seq_lens if seq_lens.dtype in (torch.int32, torch.int64) else seq_lens.to(torch.int32)
    bt = bt.contiguous()
    sl = sl.contiguous()
    batch = int(bt.shape[0])
    if max_seq_len is None:
        max_seq_len = int(sl.max().item()) if batch else 0
    out = torch.empty(batch * int(max_seq_len), dtype=torch.int64, device=bt.device)
    rc = _native.load().mak_build_slot_mapping(
        _native.ptr(bt), _native.dtype_code(bt.dtype), int(bt.stride(0)), _native.ptr(sl), _native.dtype_code(sl.dtype),
        batch, int(max_seq_len), int(block_size), _native.ptr(out), _native.stream_ptr(bt.device),
    )
    _native.check(rc, "build_slot_mapping")
    return out


def plan_slot_runs(slot_mapping: torch.Tensor) -> list[tuple[int, int, int]]:
    """Coalesce a slot mapping into ``(token_start, slot_start, length)`` runs of consecutive slots.

    Negative slots end a run and are dropped.  Host-side (one copy of the slots).
    """
    s = slot_mapping.detach().to("cpu", torch.int64).reshape(-1)
    n = int(s.numel())
    if n == 0:
        return []
    valid = s >= 0
    cont = torch.zeros(n, dtype=torch.bool)
    cont[1:] = (s[1:] == s[:-1] + 1) & valid[1:] & valid[:-1]
    heads = valid & ~cont
    starts = torch.nonzero(heads).flatten()
    run_id = torch.cumsum(heads.to(torch.int64), 0) - 1
    lengths = torch.bincount(run_id[valid], minlength=int(starts.numel()))
    return [(int(t), int(s[t]), int(k)) for t, k in zip(starts.tolist(), lengths.tolist())]


def build_transfer_plan(source: KVLayoutSpec, destination: KVLayoutSpec, slot_mapping: torch.Tensor, *,
                        direction: TransferDirection = "d2d", skip_prefix_n_tokens: int = 0,
                        stream_id: int | None = None, paged_is_source: bool = True) -> KVTransferPlan:
    """Byte-range plan for moving ``slot_mapping``'s tokens between a paged and a linear layout.

    One entry per (layer, contiguous slot run) of row-contiguous layouts; the
    direct-eligibility verdict comes from ``assess_direct_eligibility``.
    """
    eligible, reason = assess_direct_eligibility(source, destination)
    paged, linear = (source, destination) if paged_is_source else (destination, source)
    entries: list[KVTransferEntry] = []
    row = paged.row_bytes
    for layer in range(min(source.num_layers, destination.num_layers)):
        for t0, s0, length in plan_slot_runs(slot_mapping):
            remaining, tok, slot = length, t0, s0
            while remaining:
                off = slot % max(paged.block_size, 1)
                take = min(remaining, paged.block_size - off) if paged.block_size else remaining
                paged_off = (slot // max(paged.block_size, 1)) * paged.block_stride_bytes + off * row
                linear_off = (skip_prefix_n_tokens + tok) * linear.row_bytes
                src, dst = (paged_off, linear_off) if paged_is_source else (linear_off, paged_off)
                entries.append(KVTransferEntry(src, dst, take * row, layer=layer, block=slot // max(paged.block_size, 1)))
                remaining -= take
                tok += take
                slot += take
    plan = KVTransferPlan(source, destination, direction, int(slot_mapping.numel()) + skip_prefix_n_tokens,
                          skip_prefix_n_tokens, tuple(entries), stream_id, eligible, reason)
    return plan
