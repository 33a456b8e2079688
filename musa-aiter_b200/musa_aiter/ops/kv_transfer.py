"""KV-cache paged <-> linear movement and FP8 cache store/load on B200.

Public functions keep the names, signatures, return values and validation
messages of the reference module (musa_aiter/ops/kv_transfer.py); each one
validates, then runs one hand-written sm_100a kernel family through the C ABI
of ``libmak_kvcache.so``:

- tile caches ``[.., NB, NH, HD, BS]`` (block_size innermost) -> the tile engine
  (``mak_kv_paged_to_linear`` / ``mak_kv_linear_to_paged`` / FP8 variants);
- MLA flat caches ``[.., NB, BS, W]`` -> the row engine (``mak_rows_*``).

Every layer of a multi-layer call moves in one launch, on the caller's current
CUDA stream.  Scatters resolve duplicate slots on the device so the last token
wins, as in the reference's sequential loop.
"""

from __future__ import annotations

import ctypes
from typing import Literal

import torch

from .. import _build, _native
from ..dispatch import emit_native
from ._common import (
    check_slots_in_bounds,
    ensure_slotmapping_vector,
    kernel_slots,
    linear_desc,
    paged_desc,
    require_cuda,
    same_geometry,
    unit_inner,
)

__all__ = [
    "build_native_kv_transfer",
    "build_native_fp8_kv_cache",
    "is_native_kv_transfer_available",
    "is_native_fp8_kv_cache_available",
    "is_native_fp8_kv_vectorized_available",
    "native_kv_transfer_abi_version",
    "native_fp8_kv_cache_abi_version",
    "kv_paged_to_linear",
    "kv_linear_to_paged",
    "kv_paged_to_linear_multi_layer",
    "kv_linear_to_paged_multi_layer",
    "kv_paged_to_merged_linear",
    "kv_merged_linear_to_paged",
    "kv_paged_to_merged_linear_multi_layer",
    "kv_merged_linear_to_paged_multi_layer",
    "kv_linear_to_paged_fp8",
    "kv_paged_fp8_to_linear",
    "kv_linear_to_paged_fp8_multi_layer",
    "kv_paged_fp8_to_linear_multi_layer",
    "kv_paged_fp8_to_merged_linear",
    "kv_merged_linear_to_paged_fp8",
    "kv_paged_fp8_to_merged_linear_multi_layer",
    "kv_merged_linear_to_paged_fp8_multi_layer",
    "kv_paged_to_mla_linear",
    "kv_mla_linear_to_paged",
    "kv_paged_to_mla_linear_multi_layer",
    "kv_mla_linear_to_paged_multi_layer",
]


# ---------------------------------------------------------------------------
# build / probe API (musa_aiter/ops/kv_transfer.py:52-198)
# ---------------------------------------------------------------------------


def build_native_kv_transfer():
    """Compile the sm_100a kernel library (no GPU needed); returns a BuildResult."""
    return _build.build()


def build_native_fp8_kv_cache():
    """FP8 kernels live in the same library as every other kvcache kernel."""
    return _build.build()


def native_kv_transfer_abi_version() -> int | None:
    try:
        return int(_native.load().mak_abi_version())
    except Exception:
        return None


def native_fp8_kv_cache_abi_version() -> int | None:
    return native_kv_transfer_abi_version()


def is_native_kv_transfer_available() -> bool:
    return _native.is_available()


def is_native_fp8_kv_cache_available(fp8_format: str = "e4m3") -> bool:
    _normalize_fp8_format(fp8_format)
    return _native.is_available()


def is_native_fp8_kv_vectorized_available() -> bool:
    """The tile kernel always uses 16-byte vectors where the layout allows it."""
    return _native.is_available()


# ---------------------------------------------------------------------------
# shape validation (musa_aiter/ops/kv_transfer.py:2987-3044)
# ---------------------------------------------------------------------------


def _validate_paged_shapes(key_cache: torch.Tensor, value_cache: torch.Tensor, *, name: str) -> tuple[int, int, int, int]:
    if key_cache.dim() != 4 or value_cache.dim() != 4:
        raise ValueError(f"{name}: caches must be 4-D [blocks, kv_heads, head_dim, block_size]")
    if key_cache.shape != value_cache.shape:
        raise ValueError(f"{name}: key_cache and value_cache shapes must match")
    nb, nh, hd, bs = map(int, key_cache.shape)
    if nb <= 0 or nh <= 0 or hd <= 0 or bs <= 0:
        raise ValueError(f"{name}: all cache extents must be positive")
    return nb, nh, hd, bs


def _validate_stacked_paged_shapes(key_cache: torch.Tensor, value_cache: torch.Tensor, *, name: str):
    if key_cache.dim() != 5 or value_cache.dim() != 5:
        raise ValueError(f"{name}: caches must be 5-D [layers, blocks, kv_heads, head_dim, block_size]")
    if key_cache.shape != value_cache.shape:
        raise ValueError(f"{name}: key_cache and value_cache shapes must match")
    nl, nb, nh, hd, bs = map(int, key_cache.shape)
    if nl <= 0 or nb <= 0 or nh <= 0 or hd <= 0 or bs <= 0:
        raise ValueError(f"{name}: all cache extents must be positive")
    return nl, nb, nh, hd, bs


# ---------------------------------------------------------------------------
# tile engine calls
# ---------------------------------------------------------------------------


def _as_unit_inner(t: torch.Tensor) -> tuple[torch.Tensor, bool]:
    if unit_inner(t):
        return t, False
    return t.contiguous(), True


def _tile_gather(kc, vc, slots, ok, ov, *, layered: bool, fill_zero: bool, op: str,
                 fp8: tuple | None = None) -> None:
    """cache (k, v) -> linear (ok, ov); ``fp8`` = (k_scale, v_scale, mode, fmt_code) for FP8 caches."""
    lib = _native.load()
    dev = kc.device
    ks, code = kernel_slots(slots)
    kc, _ = _as_unit_inner(kc)
    vc, _ = _as_unit_inner(vc)
    ok_w, ok_tmp = _as_unit_inner(ok)
    ov_w, ov_tmp = _as_unit_inner(ov)
    stream = _native.stream_ptr(dev)
    if same_geometry(kc, vc) and same_geometry(ok_w, ov_w):
        groups = [(kc, vc, ok_w, ov_w, 0)]
    else:
        groups = [(kc, None, ok_w, None, 0), (vc, None, ov_w, None, 1)]
    for c0, c1, l0, l1, which in groups:
        pd = paged_desc(c0, c1, layered=layered)
        ld = linear_desc(l0, l1, layered=layered)
        if fp8 is None:
            rc = lib.mak_kv_paged_to_linear(ctypes.byref(pd), ctypes.byref(ld), _native.ptr(ks), code, int(fill_zero), stream)
        else:
            k_s, v_s, mode, fmt = fp8
            s0 = k_s if which == 0 else v_s
            s1 = v_s if c1 is not None else None
            rc = lib.mak_kv_paged_fp8_to_linear(
                ctypes.byref(pd), ctypes.byref(ld), _native.ptr(ks), code, _native.ptr(s0), _native.ptr(s1), mode, fmt, stream
            )
        _native.check(rc, op)
    if ok_tmp:
        ok.copy_(ok_w)
    if ov_tmp:
        ov.copy_(ov_w)


def _tile_scatter(kl, vl, kc, vc, slots, *, layered: bool, op: str, fp8: tuple | None = None) -> None:
    """linear (kl, vl) -> cache (kc, vc), last writer wins."""
    lib = _native.load()
    dev = kc.device
    ks, code = kernel_slots(slots)
    kl, _ = _as_unit_inner(kl)
    vl, _ = _as_unit_inner(vl)
    kc_w, kc_tmp = _as_unit_inner(kc)
    vc_w, vc_tmp = _as_unit_inner(vc)
    stream = _native.stream_ptr(dev)
    ws, nbytes = _native.workspace(ks.numel(), dev)
    if same_geometry(kc_w, vc_w) and same_geometry(kl, vl):
        groups = [(kl, vl, kc_w, vc_w, 0)]
    else:
        groups = [(kl, None, kc_w, None, 0), (vl, None, vc_w, None, 1)]
    for l0, l1, c0, c1, which in groups:
        pd = paged_desc(c0, c1, layered=layered)
        ld = linear_desc(l0, l1, layered=layered)
        if fp8 is None:
            rc = lib.mak_kv_linear_to_paged(
                ctypes.byref(ld), ctypes.byref(pd), _native.ptr(ks), code, _native.ptr(ws), nbytes, stream
            )
        else:
            k_s, v_s, mode, fmt = fp8
            s0 = k_s if which == 0 else v_s
            s1 = v_s if c1 is not None else None
            rc = lib.mak_kv_linear_to_paged_fp8(
                ctypes.byref(ld), ctypes.byref(pd), _native.ptr(ks), code, _native.ptr(s0), _native.ptr(s1), mode, fmt,
                _native.ptr(ws), nbytes, stream,
            )
        _native.check(rc, op)
    if kc_tmp:
        kc.copy_(kc_w)
    if vc_tmp:
        vc.copy_(vc_w)


# ---------------------------------------------------------------------------
# paged <-> linear (musa_aiter/ops/kv_transfer.py:3115-3457)
# ---------------------------------------------------------------------------


def _check_out(out_: torch.Tensor, shape: tuple, ref: torch.Tensor, name: str, what: str = "out buffer") -> None:
    if tuple(out_.shape) != tuple(shape):
        raise ValueError(f"{name}: {what} shape mismatch {tuple(out_.shape)}")
    if out_.dtype != ref.dtype:
        raise ValueError(f"{name}: {what} dtype mismatch")
    if out_.device != ref.device:
        raise ValueError(f"{name}: {what} device mismatch")


def kv_paged_to_linear(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    *,
    fill_skipped: Literal["zeros", "preserve"] = "zeros",
    out_k: torch.Tensor | None = None,
    out_v: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gather paged KV ``[NB, NH, HD, BS]`` at ``slot_mapping`` into ``[T, NH, HD]`` rows.

    ``fill_skipped="zeros"`` zeroes rows whose slot is negative; ``"preserve"``
    leaves them as they are in ``out_k``/``out_v`` (which it then requires).
    Reference: musa_aiter/ops/kv_transfer.py:3115-3206.
    """
    name = "kv_paged_to_linear"
    nb, nh, hd, bs = _validate_paged_shapes(key_cache, value_cache, name=name)
    tcount = slot_mapping.numel()
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if key_cache.device != value_cache.device or slots.device != key_cache.device:
        raise ValueError("kv_paged_to_linear: all tensors must be on the same device")
    check_slots_in_bounds(slots, nb, bs, name)
    if fill_skipped not in ("zeros", "preserve"):
        raise ValueError(f"{name}: fill_skipped must be 'zeros' or 'preserve'")
    for o in (out_k, out_v):
        if o is not None:
            _check_out(o, (tcount, nh, hd), key_cache, name)
    if fill_skipped == "preserve" and (out_k is None or out_v is None):
        raise ValueError(f"{name}: fill_skipped=preserve requires out_k/out_v buffers")
    require_cuda(name, key_cache, value_cache, slots, out_k, out_v)
    ok = out_k if out_k is not None else torch.empty((tcount, nh, hd), dtype=key_cache.dtype, device=key_cache.device)
    ov = out_v if out_v is not None else torch.empty((tcount, nh, hd), dtype=value_cache.dtype, device=key_cache.device)
    if tcount:
        _tile_gather(key_cache, value_cache, slots, ok, ov, layered=False, fill_zero=fill_skipped == "zeros", op=name)
    emit_native(name, key_cache, "sm100a tile gather")
    return ok, ov


def kv_paged_to_linear_multi_layer(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    *,
    fill_skipped: Literal["zeros", "preserve"] = "zeros",
    out_k: torch.Tensor | None = None,
    out_v: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gather ``[L, NB, NH, HD, BS]`` caches into ``[L, T, NH, HD]`` for all layers in one launch.

    Reference: musa_aiter/ops/kv_transfer.py:3209-3309.  When ``out_k``/``out_v``
    are given they are filled and returned (the reference returns a stacked copy
    with the same values).
    """
    name = "kv_paged_to_linear_multi_layer"
    nl, nb, nh, hd, bs = _validate_stacked_paged_shapes(key_cache, value_cache, name=name)
    tcount = slot_mapping.numel()
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if value_cache.device != key_cache.device or slots.device != key_cache.device:
        raise ValueError(f"{name}: all tensors must be on the same device")
    check_slots_in_bounds(slots, nb, bs, name)
    if out_k is not None and tuple(out_k.shape) != (nl, tcount, nh, hd):
        raise ValueError(f"{name}: out_k must be [num_layers, T, kv_heads, head_dim], got {tuple(out_k.shape)}")
    if out_v is not None and tuple(out_v.shape) != (nl, tcount, nh, hd):
        raise ValueError(f"{name}: out_v must be [num_layers, T, kv_heads, head_dim], got {tuple(out_v.shape)}")
    if fill_skipped == "preserve" and (out_k is None or out_v is None):
        raise ValueError(f"{name}: fill_skipped=preserve requires out_k and out_v")
    for o in (out_k, out_v):
        if o is not None:
            _check_out(o, (nl, tcount, nh, hd), key_cache, name)
    require_cuda(name, key_cache, value_cache, slots, out_k, out_v)
    ok = out_k if out_k is not None else torch.empty((nl, tcount, nh, hd), dtype=key_cache.dtype, device=key_cache.device)
    ov = out_v if out_v is not None else torch.empty((nl, tcount, nh, hd), dtype=value_cache.dtype, device=key_cache.device)
    if tcount:
        _tile_gather(key_cache, value_cache, slots, ok, ov, layered=True, fill_zero=fill_skipped == "zeros", op=name)
    emit_native(name, key_cache, "sm100a tile gather (all layers, one launch)")
    return ok, ov


def kv_linear_to_paged(
    key_linear: torch.Tensor,
    value_linear: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> None:
    """Scatter ``[T, NH, HD]`` rows into ``[NB, NH, HD, BS]`` caches in place.

    Negative slots are skipped; duplicate slots keep the last token's row.
    Reference: musa_aiter/ops/kv_transfer.py:3312-3379.
    """
    name = "kv_linear_to_paged"
    if key_linear.shape != value_linear.shape or key_linear.dim() != 3:
        raise ValueError("kv_linear_to_paged: key_linear/value_linear must be 3-D and match shapes")
    tcount = key_linear.shape[0]
    nb, nh, hd, bs = _validate_paged_shapes(key_cache, value_cache, name=name)
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if key_linear.shape[1:] != (nh, hd):
        raise ValueError(
            "kv_linear_to_paged: last dims must match caches [num_kv_heads, head_dim] "
            f"got tail {tuple(key_linear.shape[1:])} vs {(nh, hd)}",
        )
    dev = key_cache.device
    if any(x.device != dev for x in (key_linear, value_linear, key_cache, value_cache, slots)):
        raise ValueError("kv_linear_to_paged: all tensors must be on same device")
    check_slots_in_bounds(slots, nb, bs, name)
    if key_linear.dtype != key_cache.dtype or value_linear.dtype != value_cache.dtype:
        raise ValueError(f"{name}: linear and cache dtypes must match")
    require_cuda(name, key_linear, value_linear, key_cache, value_cache, slots)
    if tcount:
        _tile_scatter(key_linear, value_linear, key_cache, value_cache, slots, layered=False, op=name)
    emit_native(name, key_linear, "sm100a tile scatter")


def kv_linear_to_paged_multi_layer(
    key_linear: torch.Tensor,
    value_linear: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> None:
    """Scatter ``[L, T, NH, HD]`` into stacked caches (one launch). Reference: kv_transfer.py:3382-3457."""
    name = "kv_linear_to_paged_multi_layer"
    if key_linear.shape != value_linear.shape or key_linear.dim() != 4:
        raise ValueError(
            "kv_linear_to_paged_multi_layer: key_linear/value_linear must be 4-D "
            "[num_layers, num_tokens, num_kv_heads, head_dim] and match",
        )
    nl, tcount, nh_lin, hd_lin = map(int, key_linear.shape)
    nb, nh, hd, bs = _validate_stacked_paged_shapes(key_cache, value_cache, name=name)[1:]
    if nh_lin != nh or hd_lin != hd:
        raise ValueError(
            "kv_linear_to_paged_multi_layer: linear tail dims must match caches "
            f"got {(nh_lin, hd_lin)} vs cache {(nh, hd)}",
        )
    if key_cache.shape[0] != nl:
        raise ValueError(
            "kv_linear_to_paged_multi_layer: layer count mismatch " f"linear L={nl} vs cache L={key_cache.shape[0]}",
        )
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    dev = key_cache.device
    if any(x.device != dev for x in (key_linear, value_linear, key_cache, value_cache, slots)):
        raise ValueError("kv_linear_to_paged_multi_layer: all tensors must be on same device")
    check_slots_in_bounds(slots, nb, bs, name)
    if key_linear.dtype != key_cache.dtype or value_linear.dtype != value_cache.dtype:
        raise ValueError(f"{name}: linear and cache dtypes must match")
    require_cuda(name, key_linear, value_linear, key_cache, value_cache, slots)
    if tcount:
        _tile_scatter(key_linear, value_linear, key_cache, value_cache, slots, layered=True, op=name)
    emit_native(name, key_linear, "sm100a tile scatter (all layers, one launch)")


# ---------------------------------------------------------------------------
# merged [.., T, 2, NH, HD] layouts (musa_aiter/ops/kv_transfer.py:3556-3766)
# ---------------------------------------------------------------------------


def kv_paged_to_merged_linear(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    *,
    fill_skipped: Literal["zeros", "preserve"] = "zeros",
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Gather separate K/V caches into merged ``[T, 2, NH, HD]`` (reference kv_transfer.py:3556-3618)."""
    name = "kv_paged_to_merged_linear"
    nb, nh, hd, bs = _validate_paged_shapes(key_cache, value_cache, name=name)
    tcount = slot_mapping.numel()
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if value_cache.device != key_cache.device or slots.device != key_cache.device:
        raise ValueError(f"{name}: all tensors must be on the same device")
    if out is not None:
        if tuple(out.shape) != (tcount, 2, nh, hd):
            raise ValueError(f"{name}: out must be [T, 2, kv_heads, head_dim]")
        if out.device != key_cache.device or out.dtype != key_cache.dtype:
            raise ValueError(f"{name}: out dtype/device must match caches")
    if fill_skipped == "preserve" and out is None:
        raise ValueError(f"{name}: fill_skipped=preserve requires out")
    check_slots_in_bounds(slots, nb, bs, name)
    require_cuda(name, key_cache, value_cache, slots, out)
    res = out if out is not None else torch.empty((tcount, 2, nh, hd), dtype=key_cache.dtype, device=key_cache.device)
    if tcount:
        _tile_gather(key_cache, value_cache, slots, res[:, 0], res[:, 1], layered=False, fill_zero=fill_skipped == "zeros", op=name)
    emit_native(name, key_cache, "sm100a tile gather (merged strides)")
    return res


def kv_merged_linear_to_paged(
    merged_linear: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> None:
    """Scatter merged ``[T, 2, NH, HD]`` into separate caches (reference kv_transfer.py:3621-3654)."""
    name = "kv_merged_linear_to_paged"
    if merged_linear.dim() != 4 or merged_linear.shape[1] != 2:
        raise ValueError(f"{name}: merged_linear must be [T, 2, kv_heads, head_dim]")
    tcount = int(merged_linear.shape[0])
    nb, nh, hd, bs = _validate_paged_shapes(key_cache, value_cache, name=name)
    if tuple(merged_linear.shape[2:]) != (nh, hd):
        raise ValueError(f"{name}: merged tail dims must match caches")
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if any(x.device != key_cache.device for x in (merged_linear, key_cache, value_cache, slots)):
        raise ValueError(f"{name}: all tensors must be on same device")
    check_slots_in_bounds(slots, nb, bs, name)
    require_cuda(name, merged_linear, key_cache, value_cache, slots)
    if tcount:
        _tile_scatter(merged_linear[:, 0], merged_linear[:, 1], key_cache, value_cache, slots, layered=False, op=name)
    emit_native(name, merged_linear, "sm100a tile scatter (merged strides)")


def kv_paged_to_merged_linear_multi_layer(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    *,
    fill_skipped: Literal["zeros", "preserve"] = "zeros",
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Stacked caches -> merged ``[L, T, 2, NH, HD]`` (reference kv_transfer.py:3657-3724)."""
    name = "kv_paged_to_merged_linear_multi_layer"
    nl, nb, nh, hd, bs = _validate_stacked_paged_shapes(key_cache, value_cache, name=name)
    tcount = slot_mapping.numel()
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if value_cache.device != key_cache.device or slots.device != key_cache.device:
        raise ValueError(f"{name}: all tensors must be on the same device")
    if out is not None:
        if tuple(out.shape) != (nl, tcount, 2, nh, hd):
            raise ValueError(f"{name}: out must be [L, T, 2, kv_heads, head_dim]")
        if out.device != key_cache.device or out.dtype != key_cache.dtype:
            raise ValueError(f"{name}: out dtype/device must match caches")
    if fill_skipped == "preserve" and out is None:
        raise ValueError(f"{name}: fill_skipped=preserve requires out")
    check_slots_in_bounds(slots, nb, bs, name)
    require_cuda(name, key_cache, value_cache, slots, out)
    res = out if out is not None else torch.empty((nl, tcount, 2, nh, hd), dtype=key_cache.dtype, device=key_cache.device)
    if tcount:
        _tile_gather(key_cache, value_cache, slots, res[:, :, 0], res[:, :, 1], layered=True, fill_zero=fill_skipped == "zeros", op=name)
    emit_native(name, key_cache, "sm100a tile gather (merged strides, all layers)")
    return res


def kv_merged_linear_to_paged_multi_layer(
    merged_linear: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> None:
    """Merged ``[L, T, 2, NH, HD]`` -> stacked caches (reference kv_transfer.py:3727-3766)."""
    name = "kv_merged_linear_to_paged_multi_layer"
    if merged_linear.dim() != 5 or merged_linear.shape[2] != 2:
        raise ValueError(f"{name}: merged_linear must be [L, T, 2, kv_heads, head_dim]")
    nl, tcount, _, nh_lin, hd_lin = map(int, merged_linear.shape)
    nb, nh, hd, bs = _validate_stacked_paged_shapes(key_cache, value_cache, name=name)[1:]
    if nh_lin != nh or hd_lin != hd or key_cache.shape[0] != nl:
        raise ValueError(f"{name}: merged dims must match caches")
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if any(x.device != key_cache.device for x in (merged_linear, key_cache, value_cache, slots)):
        raise ValueError(f"{name}: all tensors must be on same device")
    check_slots_in_bounds(slots, nb, bs, name)
    require_cuda(name, merged_linear, key_cache, value_cache, slots)
    if tcount:
        _tile_scatter(merged_linear[:, :, 0], merged_linear[:, :, 1], key_cache, value_cache, slots, layered=True, op=name)
    emit_native(name, merged_linear, "sm100a tile scatter (merged strides, all layers)")


# ---------------------------------------------------------------------------
# FP8 caches (musa_aiter/ops/kv_transfer.py:2094-2398, 3460-3553)
# ---------------------------------------------------------------------------


def _normalize_fp8_format(fp8_format: str) -> str:
    normalized = fp8_format.lower().replace("-", "_")
    if normalized in ("fp8", "fp8_e4m3", "fp8_e4m3fn", "e4m3", "e4m3fn"):
        return "e4m3"
    if normalized in ("fp8_e5m2", "e5m2"):
        return "e5m2"
    raise ValueError(f"unsupported FP8 KV cache format: {fp8_format}")


_FMT_CODE = {"e4m3": _native.MAK_FP8_E4M3, "e5m2": _native.MAK_FP8_E5M2}


def _validate_fp8_cache_tensor(tensor: torch.Tensor, *, name: str) -> None:
    if tensor.dtype is torch.uint8:
        return
    if str(tensor.dtype) in ("torch.float8_e4m3fn", "torch.float8_e5m2"):
        return
    raise ValueError(f"{name}: FP8 cache storage must be torch.uint8 or a supported torch.float8 dtype")


def _ensure_fp8_scale(scale, *, device: torch.device, name: str, num_heads: int, num_layers: int | None = None) -> torch.Tensor:
    """musa_aiter/ops/kv_transfer.py:2110-2121: positive finite scalar, [NH] or [L, NH]."""
    scale_tensor = torch.as_tensor(scale, dtype=torch.float32, device=device)
    if not bool(torch.isfinite(scale_tensor).all()) or float(scale_tensor.min().item()) <= 0.0:
        raise ValueError(f"{name}: FP8 scale must be positive and finite")
    if scale_tensor.numel() == 1:
        return scale_tensor.reshape(())
    if scale_tensor.dim() == 1 and int(scale_tensor.shape[0]) == num_heads:
        return scale_tensor.reshape(num_heads)
    if num_layers is not None and scale_tensor.dim() == 2 and tuple(scale_tensor.shape) == (num_layers, num_heads):
        return scale_tensor.reshape(num_layers, num_heads)
    expected = "scalar or [kv_heads]" if num_layers is None else "scalar, [kv_heads], or [layers, kv_heads]"
    raise ValueError(f"{name}: FP8 scale must be {expected}")


def _scale_args(k_scale: torch.Tensor, v_scale: torch.Tensor, nl: int, nh: int):
    """Bring both scales to one kernel scale mode (per-layer-head when they differ)."""
    modes = {0: _native.MAK_SCALE_SCALAR, 1: _native.MAK_SCALE_PER_HEAD, 2: _native.MAK_SCALE_PER_LAYER_HEAD}
    if k_scale.dim() == v_scale.dim():
        mode = modes[k_scale.dim()]
        return k_scale.contiguous(), v_scale.contiguous(), mode
    full = lambda s: s.reshape(-1, nh if s.dim() else 1).expand(nl, nh).contiguous() if s.dim() < 2 else s.contiguous()  # noqa: E731
    return full(k_scale), full(v_scale), _native.MAK_SCALE_PER_LAYER_HEAD


def _u8_view(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype is torch.uint8 else t.view(torch.uint8)


def kv_linear_to_paged_fp8(
    key_linear: torch.Tensor,
    value_linear: torch.Tensor,
    key_cache_fp8: torch.Tensor,
    value_cache_fp8: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_scale: torch.Tensor | float,
    v_scale: torch.Tensor | float,
    *,
    fp8_format: Literal["e4m3", "e5m2"] = "e4m3",
) -> None:
    """Quantize ``[T, NH, HD]`` rows to FP8 bytes and scatter them into ``[NB, NH, HD, BS]`` caches.

    byte = encode(x / scale) with the reference encoder (kv_transfer.py:2161-2183);
    scale scalar or ``[NH]``.  Reference: kv_transfer.py:2203-2247.
    """
    name = "kv_linear_to_paged_fp8"
    fmt = _normalize_fp8_format(fp8_format)
    _validate_fp8_cache_tensor(key_cache_fp8, name=f"{name} key_cache_fp8")
    _validate_fp8_cache_tensor(value_cache_fp8, name=f"{name} value_cache_fp8")
    nb, nh, hd, bs = _validate_paged_shapes(key_cache_fp8, value_cache_fp8, name=name)
    if key_linear.shape != value_linear.shape or key_linear.dim() != 3:
        raise ValueError(f"{name}: key_linear and value_linear must be [tokens, kv_heads, head_dim]")
    tcount = int(key_linear.shape[0])
    if tuple(key_linear.shape[1:]) != (nh, hd):
        raise ValueError(f"{name}: linear shape does not match FP8 cache shape")
    if key_linear.device != value_linear.device or key_cache_fp8.device != key_linear.device or value_cache_fp8.device != key_linear.device:
        raise ValueError(f"{name}: all tensors must be on the same device")
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if slots.device != key_linear.device:
        raise ValueError(f"{name}: slot_mapping must be on the same device")
    check_slots_in_bounds(slots, nb, bs, name)
    ks = _ensure_fp8_scale(k_scale, device=key_linear.device, name="k_scale", num_heads=nh)
    vs = _ensure_fp8_scale(v_scale, device=value_linear.device, name="v_scale", num_heads=nh)
    if key_linear.dtype not in (torch.float16, torch.bfloat16, torch.float32) or value_linear.dtype != key_linear.dtype:
        raise ValueError(f"{name}: linear dtype must be float16, bfloat16 or float32")
    require_cuda(name, key_linear, value_linear, key_cache_fp8, value_cache_fp8, slots)
    ksa, vsa, mode = _scale_args(ks, vs, 1, nh)
    if tcount:
        _tile_scatter(key_linear, value_linear, _u8_view(key_cache_fp8), _u8_view(value_cache_fp8), slots,
                      layered=False, op=name, fp8=(ksa, vsa, mode, _FMT_CODE[fmt]))
    emit_native(name, key_linear, f"sm100a fused FP8 {fmt} quantize scatter")


def kv_paged_fp8_to_linear(
    key_cache_fp8: torch.Tensor,
    value_cache_fp8: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_scale: torch.Tensor | float,
    v_scale: torch.Tensor | float,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
    fp8_format: Literal["e4m3", "e5m2"] = "e4m3",
    out_k: torch.Tensor | None = None,
    out_v: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gather FP8 bytes and dequantize to ``out_dtype`` (zeros for skipped slots).

    value = (decode(byte) * scale) rounded to ``out_dtype`` (kv_transfer.py:2186-2200).
    Reference: kv_transfer.py:2250-2301.
    """
    name = "kv_paged_fp8_to_linear"
    fmt = _normalize_fp8_format(fp8_format)
    _validate_fp8_cache_tensor(key_cache_fp8, name=f"{name} key_cache_fp8")
    _validate_fp8_cache_tensor(value_cache_fp8, name=f"{name} value_cache_fp8")
    nb, nh, hd, bs = _validate_paged_shapes(key_cache_fp8, value_cache_fp8, name=name)
    tcount = int(slot_mapping.numel())
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if slots.device != key_cache_fp8.device:
        raise ValueError(f"{name}: slot_mapping must be on the same device")
    check_slots_in_bounds(slots, nb, bs, name)
    ks = _ensure_fp8_scale(k_scale, device=key_cache_fp8.device, name="k_scale", num_heads=nh)
    vs = _ensure_fp8_scale(v_scale, device=value_cache_fp8.device, name="v_scale", num_heads=nh)
    if out_dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError(f"{name}: out_dtype must be float16, bfloat16 or float32")
    for o in (out_k, out_v):
        if o is not None:
            if tuple(o.shape) != (tcount, nh, hd):
                raise ValueError(f"{name}: output shape mismatch")
            if o.dtype is not out_dtype:
                raise ValueError(f"{name}: output dtype mismatch")
    require_cuda(name, key_cache_fp8, value_cache_fp8, slots, out_k, out_v)
    dev = key_cache_fp8.device
    ok = out_k if out_k is not None else torch.empty((tcount, nh, hd), dtype=out_dtype, device=dev)
    ov = out_v if out_v is not None else torch.empty((tcount, nh, hd), dtype=out_dtype, device=dev)
    ksa, vsa, mode = _scale_args(ks, vs, 1, nh)
    if tcount:
        _tile_gather(_u8_view(key_cache_fp8), _u8_view(value_cache_fp8), slots, ok, ov, layered=False, fill_zero=True,
                     op=name, fp8=(ksa, vsa, mode, _FMT_CODE[fmt]))
    emit_native(name, key_cache_fp8, f"sm100a fused FP8 {fmt} gather dequantize")
    return ok, ov


def kv_linear_to_paged_fp8_multi_layer(
    key_linear: torch.Tensor,
    value_linear: torch.Tensor,
    key_cache_fp8: torch.Tensor,
    value_cache_fp8: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_scale: torch.Tensor | float,
    v_scale: torch.Tensor | float,
    *,
    fp8_format: Literal["e4m3", "e5m2"] = "e4m3",
) -> None:
    """``[L, T, NH, HD]`` -> FP8 ``[L, NB, NH, HD, BS]``; scale scalar, ``[NH]`` or ``[L, NH]``.

    Reference: kv_transfer.py:2304-2347.
    """
    name = "kv_linear_to_paged_fp8_multi_layer"
    fmt = _normalize_fp8_format(fp8_format)
    _validate_fp8_cache_tensor(key_cache_fp8, name=f"{name} key_cache_fp8")
    _validate_fp8_cache_tensor(value_cache_fp8, name=f"{name} value_cache_fp8")
    nl, nb, nh, hd, bs = _validate_stacked_paged_shapes(key_cache_fp8, value_cache_fp8, name=name)
    if key_linear.shape != value_linear.shape or key_linear.dim() != 4:
        raise ValueError(f"{name}: key_linear and value_linear must be [layers, tokens, kv_heads, head_dim]")
    if key_linear.shape[0] != nl or tuple(key_linear.shape[2:]) != (nh, hd):
        raise ValueError(f"{name}: linear shape does not match FP8 cache shape")
    if key_linear.device != value_linear.device or key_cache_fp8.device != key_linear.device or value_cache_fp8.device != key_linear.device:
        raise ValueError(f"{name}: all tensors must be on the same device")
    tcount = int(key_linear.shape[1])
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if slots.device != key_linear.device:
        raise ValueError(f"{name}: slot_mapping must be on the same device")
    check_slots_in_bounds(slots, nb, bs, name)
    ks = _ensure_fp8_scale(k_scale, device=key_linear.device, name="k_scale", num_heads=nh, num_layers=nl)
    vs = _ensure_fp8_scale(v_scale, device=value_linear.device, name="v_scale", num_heads=nh, num_layers=nl)
    if key_linear.dtype not in (torch.float16, torch.bfloat16, torch.float32) or value_linear.dtype != key_linear.dtype:
        raise ValueError(f"{name}: linear dtype must be float16, bfloat16 or float32")
    require_cuda(name, key_linear, value_linear, key_cache_fp8, value_cache_fp8, slots)
    ksa, vsa, mode = _scale_args(ks, vs, nl, nh)
    if tcount:
        _tile_scatter(key_linear, value_linear, _u8_view(key_cache_fp8), _u8_view(value_cache_fp8), slots,
                      layered=True, op=name, fp8=(ksa, vsa, mode, _FMT_CODE[fmt]))
    emit_native(name, key_linear, f"sm100a fused FP8 {fmt} quantize scatter (all layers)")


def kv_paged_fp8_to_linear_multi_layer(
    key_cache_fp8: torch.Tensor,
    value_cache_fp8: torch.Tensor,
    slot_mapping: torch.Tensor,
    k_scale: torch.Tensor | float,
    v_scale: torch.Tensor | float,
    *,
    out_dtype: torch.dtype = torch.bfloat16,
    fp8_format: Literal["e4m3", "e5m2"] = "e4m3",
    out_k: torch.Tensor | None = None,
    out_v: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """FP8 ``[L, NB, NH, HD, BS]`` -> ``[L, T, NH, HD]`` dequantized. Reference: kv_transfer.py:2350-2398."""
    name = "kv_paged_fp8_to_linear_multi_layer"
    fmt = _normalize_fp8_format(fp8_format)
    _validate_fp8_cache_tensor(key_cache_fp8, name=f"{name} key_cache_fp8")
    _validate_fp8_cache_tensor(value_cache_fp8, name=f"{name} value_cache_fp8")
    nl, nb, nh, hd, bs = _validate_stacked_paged_shapes(key_cache_fp8, value_cache_fp8, name=name)
    tcount = int(slot_mapping.numel())
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if slots.device != key_cache_fp8.device:
        raise ValueError(f"{name}: slot_mapping must be on the same device")
    check_slots_in_bounds(slots, nb, bs, name)
    ks = _ensure_fp8_scale(k_scale, device=key_cache_fp8.device, name="k_scale", num_heads=nh, num_layers=nl)
    vs = _ensure_fp8_scale(v_scale, device=value_cache_fp8.device, name="v_scale", num_heads=nh, num_layers=nl)
    if out_dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError(f"{name}: out_dtype must be float16, bfloat16 or float32")
    for o in (out_k, out_v):
        if o is not None:
            if tuple(o.shape) != (nl, tcount, nh, hd):
                raise ValueError(f"{name}: output shape mismatch")
            if o.dtype is not out_dtype:
                raise ValueError(f"{name}: output dtype mismatch")
    require_cuda(name, key_cache_fp8, value_cache_fp8, slots, out_k, out_v)
    dev = key_cache_fp8.device
    ok = out_k if out_k is not None else torch.empty((nl, tcount, nh, hd), dtype=out_dtype, device=dev)
    ov = out_v if out_v is not None else torch.empty((nl, tcount, nh, hd), dtype=out_dtype, device=dev)
    ksa, vsa, mode = _scale_args(ks, vs, nl, nh)
    if tcount:
        _tile_gather(_u8_view(key_cache_fp8), _u8_view(value_cache_fp8), slots, ok, ov, layered=True, fill_zero=True,
                     op=name, fp8=(ksa, vsa, mode, _FMT_CODE[fmt]))
    emit_native(name, key_cache_fp8, f"sm100a fused FP8 {fmt} gather dequantize (all layers)")
    return ok, ov


def kv_paged_fp8_to_merged_linear(
    key_cache_fp8, value_cache_fp8, slot_mapping, k_scale, v_scale, *, out_dtype=torch.bfloat16, fp8_format="e4m3", out=None
) -> torch.Tensor:
    """FP8 caches -> merged ``[T, 2, NH, HD]`` (reference kv_transfer.py:3460-3486)."""
    name = "kv_paged_fp8_to_merged_linear"
    _, nh, hd, _ = _validate_paged_shapes(key_cache_fp8, value_cache_fp8, name=name)
    tcount = int(slot_mapping.numel())
    if out is not None:
        if tuple(out.shape) != (tcount, 2, nh, hd):
            raise ValueError(f"{name}: out must be [T, 2, kv_heads, head_dim]")
        if out.device != key_cache_fp8.device or out.dtype is not out_dtype:
            raise ValueError(f"{name}: out dtype/device mismatch")
    res = out if out is not None else torch.empty((tcount, 2, nh, hd), dtype=out_dtype, device=key_cache_fp8.device)
    kv_paged_fp8_to_linear(key_cache_fp8, value_cache_fp8, slot_mapping, k_scale, v_scale, out_dtype=out_dtype,
                           fp8_format=fp8_format, out_k=res[:, 0], out_v=res[:, 1])
    return res


def kv_merged_linear_to_paged_fp8(
    merged_linear, key_cache_fp8, value_cache_fp8, slot_mapping, k_scale, v_scale, *, fp8_format="e4m3"
) -> None:
    """Merged ``[T, 2, NH, HD]`` -> FP8 caches (reference kv_transfer.py:3489-3505)."""
    if merged_linear.dim() != 4 or merged_linear.shape[1] != 2:
        raise ValueError("kv_merged_linear_to_paged_fp8: merged_linear must be [T, 2, kv_heads, head_dim]")
    kv_linear_to_paged_fp8(merged_linear[:, 0], merged_linear[:, 1], key_cache_fp8, value_cache_fp8, slot_mapping,
                           k_scale, v_scale, fp8_format=fp8_format)


def kv_paged_fp8_to_merged_linear_multi_layer(
    key_cache_fp8, value_cache_fp8, slot_mapping, k_scale, v_scale, *, out_dtype=torch.bfloat16, fp8_format="e4m3", out=None
) -> torch.Tensor:
    """FP8 stacked caches -> merged ``[L, T, 2, NH, HD]`` (reference kv_transfer.py:3508-3534)."""
    name = "kv_paged_fp8_to_merged_linear_multi_layer"
    nl, _, nh, hd, _ = _validate_stacked_paged_shapes(key_cache_fp8, value_cache_fp8, name=name)
    tcount = int(slot_mapping.numel())
    if out is not None:
        if tuple(out.shape) != (nl, tcount, 2, nh, hd):
            raise ValueError(f"{name}: out must be [L, T, 2, kv_heads, head_dim]")
        if out.device != key_cache_fp8.device or out.dtype is not out_dtype:
            raise ValueError(f"{name}: out dtype/device mismatch")
    res = out if out is not None else torch.empty((nl, tcount, 2, nh, hd), dtype=out_dtype, device=key_cache_fp8.device)
    kv_paged_fp8_to_linear_multi_layer(key_cache_fp8, value_cache_fp8, slot_mapping, k_scale, v_scale, out_dtype=out_dtype,
                                       fp8_format=fp8_format, out_k=res[:, :, 0], out_v=res[:, :, 1])
    return res


def kv_merged_linear_to_paged_fp8_multi_layer(
    merged_linear, key_cache_fp8, value_cache_fp8, slot_mapping, k_scale, v_scale, *, fp8_format="e4m3"
) -> None:
    """Merged ``[L, T, 2, NH, HD]`` -> FP8 stacked caches (reference kv_transfer.py:3537-3553)."""
    if merged_linear.dim() != 5 or merged_linear.shape[2] != 2:
        raise ValueError("kv_merged_linear_to_paged_fp8_multi_layer: merged_linear must be [L, T, 2, kv_heads, head_dim]")
    kv_linear_to_paged_fp8_multi_layer(merged_linear[:, :, 0], merged_linear[:, :, 1], key_cache_fp8, value_cache_fp8,
                                       slot_mapping, k_scale, v_scale, fp8_format=fp8_format)


# ---------------------------------------------------------------------------
# MLA flat caches [.., NB, BS, W] (musa_aiter/ops/kv_transfer.py:3769-4118)
# ---------------------------------------------------------------------------


def _rows_side_paged(cache: torch.Tensor, layered: bool):
    """Row-side descriptor of [L, NB, BS, W] (layered) or [NB, BS, W] with unit inner stride."""
    e = cache.element_size()
    if layered:
        nl = cache.shape[0]
        ptrs = [cache.data_ptr() + i * cache.stride(0) * e for i in range(nl)]
        nb, bs = cache.shape[1], cache.shape[2]
        sb, st = cache.stride(1), cache.stride(2)
    else:
        ptrs = [cache.data_ptr()]
        nb, bs = cache.shape[0], cache.shape[1]
        sb, st = cache.stride(0), cache.stride(1)
    return _native.rows_desc(ptrs, int(bs), int(sb * e), int(st * e), int(nb * bs))


def _rows_side_linear(buf: torch.Tensor, layered: bool):
    """Row-side descriptor of [L, T, W] (layered) or [T, W]."""
    e = buf.element_size()
    if layered:
        ptrs = [buf.data_ptr() + i * buf.stride(0) * e for i in range(buf.shape[0])]
        t, st = buf.shape[1], buf.stride(1)
    else:
        ptrs = [buf.data_ptr()]
        t, st = buf.shape[0], buf.stride(0)
    return _native.rows_desc(ptrs, 1, int(st * e), 0, int(t))


def _mla_gather(cache: torch.Tensor, slots: torch.Tensor, out: torch.Tensor, *, layered: bool, op: str) -> None:
    lib = _native.load()
    cache, _ = _as_unit_inner(cache)
    work, tmp = _as_unit_inner(out)
    ks, code = kernel_slots(slots)
    pd, pa = _rows_side_paged(cache, layered)
    ld, la = _rows_side_linear(work, layered)
    rb = cache.shape[-1] * cache.element_size()
    rc = lib.mak_rows_gather(ctypes.byref(pd), ctypes.byref(ld), None, rb, _native.ptr(ks), code, ks.numel(), 1,
                             _native.stream_ptr(cache.device))
    _native.check(rc, op)
    if tmp:
        out.copy_(work)


def _mla_scatter(lin: torch.Tensor, cache: torch.Tensor, slots: torch.Tensor, *, layered: bool, op: str, ws=None) -> None:
    lib = _native.load()
    lin, _ = _as_unit_inner(lin)
    work, tmp = _as_unit_inner(cache)
    ks, code = kernel_slots(slots)
    pd, pa = _rows_side_paged(work, layered)
    ld, la = _rows_side_linear(lin, layered)
    rb = cache.shape[-1] * cache.element_size()
    if ws is None:
        ws = _native.workspace(ks.numel(), cache.device)
    buf, nbytes = ws
    rc = lib.mak_rows_scatter(ctypes.byref(ld), ctypes.byref(pd), None, rb, _native.ptr(ks), code, ks.numel(), 0,
                              _native.ptr(buf), nbytes, _native.stream_ptr(cache.device))
    _native.check(rc, op)
    if tmp:
        cache.copy_(work)


def _validate_flat_paged_shapes(first_cache, second_cache, *, name: str) -> tuple[int, int, int, int]:
    if first_cache.dim() != 3 or second_cache.dim() != 3:
        raise ValueError(f"{name}: caches must be 3-D [blocks, block_size, hidden_dim]")
    if first_cache.shape[:2] != second_cache.shape[:2]:
        raise ValueError(f"{name}: caches must share [blocks, block_size]")
    nb, bs, first_dim = map(int, first_cache.shape)
    second_dim = int(second_cache.shape[2])
    if nb <= 0 or bs <= 0 or first_dim <= 0 or second_dim <= 0:
        raise ValueError(f"{name}: all cache extents must be positive")
    return nb, bs, first_dim, second_dim


def _validate_stacked_mla_shapes(kv_cache, k_pe_cache, *, name: str):
    if kv_cache.dim() != 4 or k_pe_cache.dim() != 4:
        raise ValueError(f"{name}: caches must be [layers, blocks, block_size, hidden_dim]")
    if tuple(kv_cache.shape[:3]) != tuple(k_pe_cache.shape[:3]):
        raise ValueError(f"{name}: caches must share [layers, blocks, block_size]")
    nl, nb, bs, kv_dim = map(int, kv_cache.shape)
    pe_dim = int(k_pe_cache.shape[3])
    if nl <= 0 or nb <= 0 or bs <= 0 or kv_dim <= 0 or pe_dim <= 0:
        raise ValueError(f"{name}: all cache extents must be positive")
    return nl, nb, bs, kv_dim, pe_dim


def kv_paged_to_mla_linear(
    kv_cache: torch.Tensor,
    k_pe_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    *,
    out_kv: torch.Tensor | None = None,
    out_k_pe: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """MLA flat caches ``[NB, BS, kv_dim]`` + ``[NB, BS, pe_dim]`` -> ``[T, kv_dim]`` + ``[T, pe_dim]``.

    Reference: kv_transfer.py:3841-3903 (negative slots give zero rows).
    """
    name = "kv_paged_to_mla_linear"
    nb, bs, kv_dim, pe_dim = _validate_flat_paged_shapes(kv_cache, k_pe_cache, name=name)
    tcount = slot_mapping.numel()
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if k_pe_cache.device != kv_cache.device or slots.device != kv_cache.device:
        raise ValueError(f"{name}: all tensors must be on the same device")
    check_slots_in_bounds(slots, nb, bs, name)
    if out_kv is not None and tuple(out_kv.shape) != (tcount, kv_dim):
        raise ValueError(f"{name}: first_out shape mismatch {tuple(out_kv.shape)}")
    if out_k_pe is not None and tuple(out_k_pe.shape) != (tcount, pe_dim):
        raise ValueError(f"{name}: second_out shape mismatch {tuple(out_k_pe.shape)}")
    require_cuda(name, kv_cache, k_pe_cache, slots, out_kv, out_k_pe)
    okv = out_kv if out_kv is not None else torch.empty((tcount, kv_dim), dtype=kv_cache.dtype, device=kv_cache.device)
    ope = out_k_pe if out_k_pe is not None else torch.empty((tcount, pe_dim), dtype=k_pe_cache.dtype, device=kv_cache.device)
    if okv.dtype != kv_cache.dtype or ope.dtype != k_pe_cache.dtype:
        raise ValueError(f"{name}: output dtypes must match caches")
    if tcount:
        _mla_gather(kv_cache, slots, okv, layered=False, op=name)
        _mla_gather(k_pe_cache, slots, ope, layered=False, op=name)
    emit_native(name, kv_cache, "sm100a row gather (MLA flat)")
    return okv, ope


def kv_mla_linear_to_paged(
    kv_linear: torch.Tensor,
    k_pe_linear: torch.Tensor,
    kv_cache: torch.Tensor,
    k_pe_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> None:
    """``[T, kv_dim]`` + ``[T, pe_dim]`` -> MLA flat caches (last writer wins). Reference: kv_transfer.py:3906-3962."""
    name = "kv_mla_linear_to_paged"
    if kv_linear.dim() != 2 or k_pe_linear.dim() != 2:
        raise ValueError(f"{name}: linear buffers must be [T, hidden_dim]")
    if kv_linear.shape[0] != k_pe_linear.shape[0]:
        raise ValueError(f"{name}: linear buffers must share token count")
    tcount = int(kv_linear.shape[0])
    nb, bs, kv_dim, pe_dim = _validate_flat_paged_shapes(kv_cache, k_pe_cache, name=name)
    if tuple(kv_linear.shape[1:]) != (kv_dim,) or tuple(k_pe_linear.shape[1:]) != (pe_dim,):
        raise ValueError(f"{name}: linear hidden dims must match caches")
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if any(x.device != kv_cache.device for x in (kv_linear, k_pe_linear, kv_cache, k_pe_cache, slots)):
        raise ValueError(f"{name}: all tensors must be on same device")
    check_slots_in_bounds(slots, nb, bs, name)
    if kv_linear.dtype != kv_cache.dtype or k_pe_linear.dtype != k_pe_cache.dtype:
        raise ValueError(f"{name}: dtypes must match caches")
    require_cuda(name, kv_linear, k_pe_linear, kv_cache, k_pe_cache, slots)
    if tcount:
        ws = _native.workspace(tcount, kv_cache.device)
        _mla_scatter(kv_linear, kv_cache, slots, layered=False, op=name, ws=ws)
        _mla_scatter(k_pe_linear, k_pe_cache, slots, layered=False, op=name, ws=ws)
    emit_native(name, kv_linear, "sm100a row scatter (MLA flat)")


def kv_paged_to_mla_linear_multi_layer(
    kv_cache: torch.Tensor,
    k_pe_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Stacked ``[L, NB, BS, W]`` MLA caches -> ``[L, T, W]`` (reference kv_transfer.py:3982-4050)."""
    name = "kv_paged_to_mla_linear_multi_layer"
    nl, nb, bs, kv_dim, pe_dim = _validate_stacked_mla_shapes(kv_cache, k_pe_cache, name=name)
    if k_pe_cache.dtype != kv_cache.dtype or k_pe_cache.device != kv_cache.device:
        raise ValueError(f"{name}: caches must share dtype and device")
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=int(slot_mapping.numel()), name=name)
    if slots.device != kv_cache.device:
        raise ValueError(f"{name}: slot_mapping must share device")
    check_slots_in_bounds(slots, nb, bs, name)
    require_cuda(name, kv_cache, k_pe_cache, slots)
    t = slots.numel()
    okv = torch.empty((nl, t, kv_dim), dtype=kv_cache.dtype, device=kv_cache.device)
    ope = torch.empty((nl, t, pe_dim), dtype=k_pe_cache.dtype, device=kv_cache.device)
    if t:
        _mla_gather(kv_cache, slots, okv, layered=True, op=name)
        _mla_gather(k_pe_cache, slots, ope, layered=True, op=name)
    emit_native(name, kv_cache, "sm100a row gather (MLA flat, all layers)")
    return okv, ope


def kv_mla_linear_to_paged_multi_layer(
    kv_linear: torch.Tensor,
    k_pe_linear: torch.Tensor,
    kv_cache: torch.Tensor,
    k_pe_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> bool:
    """``[L, T, W]`` -> stacked MLA caches (reference kv_transfer.py:4053-4118)."""
    name = "kv_mla_linear_to_paged_multi_layer"
    nl, nb, bs, kv_dim, pe_dim = _validate_stacked_mla_shapes(kv_cache, k_pe_cache, name=name)
    if kv_linear.dim() != 3 or k_pe_linear.dim() != 3:
        raise ValueError(f"{name}: linear buffers must be [layers, tokens, hidden]")
    if kv_linear.shape[0] != nl or k_pe_linear.shape[0] != nl:
        raise ValueError(f"{name}: layer counts must match caches")
    if kv_linear.shape[1] != k_pe_linear.shape[1]:
        raise ValueError(f"{name}: token counts must match")
    if tuple(kv_linear.shape[2:]) != (kv_dim,) or tuple(k_pe_linear.shape[2:]) != (pe_dim,):
        raise ValueError(f"{name}: hidden dims must match caches")
    if kv_linear.dtype != kv_cache.dtype or k_pe_linear.dtype != k_pe_cache.dtype:
        raise ValueError(f"{name}: dtypes must match caches")
    if any(t.device != kv_cache.device for t in (kv_linear, k_pe_linear, kv_cache, k_pe_cache, slot_mapping)):
        raise ValueError(f"{name}: all tensors must share device")
    tcount = int(kv_linear.shape[1])
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    check_slots_in_bounds(slots, nb, bs, name)
    require_cuda(name, kv_linear, k_pe_linear, kv_cache, k_pe_cache, slots)
    if tcount:
        ws = _native.workspace(tcount, kv_cache.device)
        _mla_scatter(kv_linear, kv_cache, slots, layered=True, op=name, ws=ws)
        _mla_scatter(k_pe_linear, k_pe_cache, slots, layered=True, op=name, ws=ws)
    emit_native(name, kv_linear, "sm100a row scatter (MLA flat, all layers)")
    return True
