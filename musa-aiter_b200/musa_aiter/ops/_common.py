"""Validation and descriptor helpers shared by the kvcache ops.

Validation messages follow the reference word for word where its tests assert
them (musa_aiter/ops/kv_transfer.py:2987-3044, ops/lmcache_kv_transfer.py:323-528).
Shape and slot checks run before the device check, so the host-side rules are
testable with CPU tensors; the data movement itself only exists on CUDA.
"""

from __future__ import annotations

import os

import torch

from .. import _native

_INDEX_DTYPES = (torch.int16, torch.int32, torch.int64)


def require_cuda(name: str, *tensors: torch.Tensor) -> torch.device:
    """All tensors must be CUDA tensors on one device: this backend has no CPU path."""
    dev = None
    idx = -2
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(
                f"{name}: the B200 kvcache backend runs on CUDA tensors only (got a {t.device} tensor); "
                "there is no CPU fallback"
            )
        if dev is None:
            dev = t.device
            idx = t.get_device()
        elif t.get_device() != idx:
            raise ValueError(f"{name}: all tensors must be on the same device")
    _native.load()
    return dev


def ensure_slotmapping_vector(slot_mapping: torch.Tensor, *, expected_len: int, name: str) -> torch.Tensor:
    """musa_aiter/ops/kv_transfer.py:3003-3017 (same checks and messages)."""
    if slot_mapping.dim() != 1:
        raise ValueError(f"{name}: slot_mapping must be a 1-D tensor")
    if slot_mapping.numel() != expected_len:
        raise ValueError(f"{name}: slot_mapping length {slot_mapping.numel()} does not match num_tokens={expected_len}")
    if slot_mapping.dtype not in _INDEX_DTYPES:
        raise ValueError(f"{name}: slot_mapping must be integer-valued (int16/int32/int64)")
    return slot_mapping


def kernel_slots(slots: torch.Tensor) -> tuple[torch.Tensor, int]:
    """Slots as a contiguous int32/int64 vector plus its dtype code (int16 widens to int32)."""
    if slots.dtype == torch.int16:
        slots = slots.to(torch.int32)
    if not slots.is_contiguous():
        slots = slots.contiguous()
    return slots, _native.dtype_code(slots.dtype)


def validation_enabled() -> bool:
    """Device-side validation reads (slot bounds, FP8 scale checks) are on unless
    ``MUSA_AITER_SKIP_VALIDATION=1`` (alias ``MUSA_AITER_SKIP_SLOT_VALIDATION``) is set;
    with them off no host sync happens and the kernels skip out-of-range slots."""
    off = {"1", "true", "TRUE", "yes", "YES"}
    return os.environ.get("MUSA_AITER_SKIP_VALIDATION", "0") not in off and \
        os.environ.get("MUSA_AITER_SKIP_SLOT_VALIDATION", "0") not in off


def slot_max(slots: torch.Tensor) -> int:
    """Largest slot value (-1 when all are negative).  One D2H read on CUDA."""
    if slots.numel() == 0:
        return -1
    if slots.device.type != "cuda":
        return int(slots.to(torch.int64).max().item())
    ks, code = kernel_slots(slots)
    out = torch.empty(1, dtype=torch.int64, device=slots.device)
    _native.check(
        _native.load().mak_slot_max(_native.ptr(ks), code, ks.numel(), _native.ptr(out), _native.stream_ptr(slots.device)),
        "slot validation",
    )
    return int(out.item())


def check_slots_in_bounds(slots: torch.Tensor, nb: int, bs: int, name: str) -> None:
    """musa_aiter/ops/kv_transfer.py:3020-3028: raise before touching any data.

    On CUDA this is one reduction kernel plus an 8-byte read-back (the reference
    does two ``.item()`` syncs); ``MUSA_AITER_SKIP_VALIDATION=1`` skips it,
    in which case out-of-range slots are skipped by the kernels instead.
    """
    if slots.device.type == "cuda" and not validation_enabled():
        return
    max_slot = slot_max(slots)
    if max_slot >= nb * bs:
        raise ValueError(f"{name}: slot index {max_slot} out of bounds for caches (max {nb * bs - 1})")


def paged_desc(k: torch.Tensor, v: torch.Tensor | None, *, layered: bool) -> _native.PagedDesc:
    """Descriptor of a [L][NB][NH][HD][BS] (layered) or [NB][NH][HD][BS] cache pair."""
    if layered:
        nl, nb, nh, hd, bs = map(int, k.shape)
        sl, sb, sh, sd, so = k.stride()
    else:
        nl = 1
        nb, nh, hd, bs = map(int, k.shape)
        sb, sh, sd, so = k.stride()
        sl = 0
    assert so == 1 or bs == 1
    return _native.PagedDesc(
        k.data_ptr(),
        v.data_ptr() if v is not None else 0,
        nl,
        nb,
        nh,
        hd,
        bs,
        sl,
        sb,
        sh,
        sd,
        _native.dtype_code(k.dtype),
        0,
    )


def linear_desc(k: torch.Tensor, v: torch.Tensor | None, *, layered: bool) -> _native.LinearDesc:
    """Descriptor of [L][T][NH][HD] (layered) or [T][NH][HD] buffers (head_dim stride 1)."""
    if layered:
        nl, t, nh, hd = map(int, k.shape)
        sl, st, sh, sd = k.stride()
    else:
        t, nh, hd = map(int, k.shape)
        st, sh, sd = k.stride()
        sl = 0
    assert sd == 1 or hd == 1
    return _native.LinearDesc(
        k.data_ptr(), v.data_ptr() if v is not None else 0, t, sl, st, sh, _native.dtype_code(k.dtype), 0
    )


def unit_inner(t: torch.Tensor) -> bool:
    return t.dim() == 0 or t.stride(-1) == 1 or t.shape[-1] == 1


def same_geometry(a: torch.Tensor, b: torch.Tensor) -> bool:
    return a.shape == b.shape and a.stride() == b.stride() and a.dtype == b.dtype
