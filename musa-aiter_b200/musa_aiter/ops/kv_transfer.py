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
import math
import struct
import threading
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
    validation_enabled,
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
    "mla_fp8_row_bytes",
    "kv_mla_linear_to_paged_fp8_rows",
    "kv_paged_fp8_rows_to_mla_linear",
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
        smap, sents, sepoch = _native.seg_map(dev, stream, ks.numel())
        if fp8 is None:
            rc = lib.mak_kv_paged_to_linear_mapped(ctypes.byref(pd), ctypes.byref(ld), _native.ptr(ks), code,
                                                   int(fill_zero), smap, sents, sepoch, stream)
        else:
            k_s, v_s, mode, fmt = fp8
            s0 = k_s if which == 0 else v_s
            s1 = v_s if c1 is not None else None
            rc = lib.mak_kv_paged_fp8_to_linear_mapped(
                ctypes.byref(pd), ctypes.byref(ld), _native.ptr(ks), code, _native.ptr(s0), _native.ptr(s1), mode, fmt,
                smap, sents, sepoch, stream,
            )
        _native.check(rc, op)
    if ok_tmp:
        ok.copy_(ok_w)
    if ov_tmp:
        ov.copy_(ov_w)


def _tile_scatter(kl, vl, kc, vc, slots, *, layered: bool, op: str, fp8: tuple | None = None) -> None:
    """linear (kl, vl) -> cache (kc, vc), last writer wins: through this stream's owner table
    (``mak_kv_linear_to_paged[_fp8]_owned``), or a workspace from torch's caching allocator where
    owner tables do not apply (stream capture, very large caches)."""
    lib = _native.load()
    dev = kc.device
    ks, code = kernel_slots(slots)
    kl, _ = _as_unit_inner(kl)
    vl, _ = _as_unit_inner(vl)
    kc_w, kc_tmp = _as_unit_inner(kc)
    vc_w, vc_tmp = _as_unit_inner(vc)
    stream = _native.stream_ptr(dev)
    ws = None
    if same_geometry(kc_w, vc_w) and same_geometry(kl, vl):
        groups = [(kl, vl, kc_w, vc_w, 0)]
    else:
        groups = [(kl, None, kc_w, None, 0), (vl, None, vc_w, None, 1)]
    for l0, l1, c0, c1, which in groups:
        pd = paged_desc(c0, c1, layered=layered)
        ld = linear_desc(l0, l1, layered=layered)
        n_slots = int(pd.num_blocks) * int(pd.block_size)
        smap, sents, sepoch = _native.seg_map(dev, stream, ks.numel())
        if fp8 is None:
            owned = lambda own, orows, epoch: lib.mak_kv_linear_to_paged_owned(  # noqa: E731
                ctypes.byref(ld), ctypes.byref(pd), _native.ptr(ks), code, own, orows, epoch, smap, sents, sepoch, stream)
        else:
            k_s, v_s, mode, fmt = fp8
            s0 = k_s if which == 0 else v_s
            s1 = v_s if c1 is not None else None
            owned = lambda own, orows, epoch: lib.mak_kv_linear_to_paged_fp8_owned(  # noqa: E731
                ctypes.byref(ld), ctypes.byref(pd), _native.ptr(ks), code, _native.ptr(s0), _native.ptr(s1), mode, fmt,
                own, orows, epoch, smap, sents, sepoch, stream)
        rc = _native.owned_scatter(dev, stream, n_slots, ks.numel(), owned)
        if rc is None:
            if ws is None:
                ws, nbytes = _native.workspace(ks.numel(), dev)
            if fp8 is None:
                rc = lib.mak_kv_linear_to_paged_mapped(
                    ctypes.byref(ld), ctypes.byref(pd), _native.ptr(ks), code, _native.ptr(ws), nbytes, smap, sents,
                    sepoch, stream,
                )
            else:
                rc = lib.mak_kv_linear_to_paged_fp8_mapped(
                    ctypes.byref(ld), ctypes.byref(pd), _native.ptr(ks), code, _native.ptr(s0), _native.ptr(s1), mode,
                    fmt, _native.ptr(ws), nbytes, smap, sents, sepoch, stream,
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


# Python-number FP8 scales placed on a device once: (device index, float32 bits) -> 0-d tensor that
# is never written again, so every stream may read it.
_SCALAR_SCALES: dict[tuple[int, int], torch.Tensor] = {}
_SCALAR_SCALES_LOCK = threading.Lock()
_SCALAR_SCALES_MAX = 1024


def _device_scalar_scale(value: float, device: torch.device) -> torch.Tensor:
    """A float32 0-d device tensor holding ``value``.  The first use of a value on a device fills it
    and waits for the fill, then the tensor is reused; under stream capture the fill is captured
    with the call instead (no wait is allowed there)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    key = (index, struct.unpack("<I", struct.pack("<f", value))[0])
    cached = _SCALAR_SCALES.get(key)
    if cached is not None:
        return cached
    dev = torch.device("cuda", index)
    if torch.cuda.is_current_stream_capturing():
        return torch.full((), value, dtype=torch.float32, device=dev)
    tensor = torch.full((), value, dtype=torch.float32, device=dev)
    torch.cuda.current_stream(dev).synchronize()
    with _SCALAR_SCALES_LOCK:
        if len(_SCALAR_SCALES) >= _SCALAR_SCALES_MAX:
            _SCALAR_SCALES.clear()
        _SCALAR_SCALES[key] = tensor
    return tensor


def _ensure_fp8_scale(scale, *, device: torch.device, name: str, num_heads: int, num_layers: int | None = None) -> torch.Tensor:
    """musa_aiter/ops/kv_transfer.py:2110-2121: positive finite scalar, [NH] or [L, NH].

    A Python number is checked on the host and placed on the device once per value (copying it from
    host memory on every call would synchronise the stream each time, a fill launch per call costs
    a launch).
    """
    if isinstance(scale, (int, float)) and not isinstance(scale, bool):
        value = float(scale)
        if not math.isfinite(value) or value <= 0.0:
            raise ValueError(f"{name}: FP8 scale must be positive and finite")
        if device.type != "cuda":
            return torch.full((), value, dtype=torch.float32, device=device)
        return _device_scalar_scale(value, device)
    scale_tensor = torch.as_tensor(scale, dtype=torch.float32, device=device)
    if scale_tensor.device.type != "cuda" or validation_enabled():
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


def _rows_side_paged(cache: torch.Tensor, layered: bool) -> tuple:
    """Row geometry ``(ptrs, rows_per_block, block_stride, row_stride, num_rows)`` of
    [L, NB, BS, W] (layered: one plane per layer) or [NB, BS, W], unit inner stride."""
    e = cache.element_size()
    base = cache.data_ptr()
    if layered:
        s0, sb, st = cache.stride()[:3]
        ptrs = [base + i * s0 * e for i in range(cache.shape[0])]
        nb, bs = cache.shape[1], cache.shape[2]
    else:
        sb, st = cache.stride()[:2]
        ptrs = [base]
        nb, bs = cache.shape[0], cache.shape[1]
    return ptrs, int(bs), int(sb * e), int(st * e), int(nb * bs)


def _rows_side_linear(buf: torch.Tensor, layered: bool) -> tuple:
    """Row geometry of [L, T, W] (layered) or [T, W]."""
    e = buf.element_size()
    base = buf.data_ptr()
    if layered:
        s0, st = buf.stride()[:2]
        ptrs = [base + i * s0 * e for i in range(buf.shape[0])]
        t = buf.shape[1]
    else:
        ptrs = [base]
        t, st = buf.shape[0], buf.stride(0)
    return ptrs, 1, int(st * e), 0, int(t)


def _mla_cache_side(c1: torch.Tensor, c2: torch.Tensor, layered: bool):
    """(packed paged descriptors of the latent and rope caches, row widths), memoised per cache pair."""
    key = ("mla", layered, c1.data_ptr(), c1.shape, c1.stride(), c1.dtype, c2.data_ptr(), c2.shape, c2.stride(), c2.dtype)

    def build():
        buf = _native.rows_pack(_rows_side_paged(c1, layered), _rows_side_paged(c2, layered))
        rb = (ctypes.c_int64 * 2)(c1.shape[-1] * c1.element_size(), c2.shape[-1] * c2.element_size())
        return buf, ctypes.addressof(buf), rb

    return _native.cached(key, build)


def _mla_pair_gather(kv_cache: torch.Tensor, pe_cache: torch.Tensor, slots: torch.Tensor, okv: torch.Tensor,
                     ope: torch.Tensor, *, layered: bool, op: str) -> None:
    """Latent and rope caches -> linear rows in ONE launch (two plane geometries, one slot vector)."""
    lib = _native.load()
    c1 = kv_cache if kv_cache.stride(-1) == 1 else kv_cache.contiguous()
    c2 = pe_cache if pe_cache.stride(-1) == 1 else pe_cache.contiguous()
    w1, t1 = _as_unit_inner(okv)
    w2, t2 = _as_unit_inner(ope)
    ks, code = kernel_slots(slots)
    _, paged, rb = _mla_cache_side(c1, c2, layered)
    lin = _native.rows_pack(_rows_side_linear(w1, layered), _rows_side_linear(w2, layered))
    rc = lib.mak_rows_gatherv(paged, ctypes.addressof(lin), 2, rb, 0, ks.data_ptr(), code, ks.numel(), 1,
                              _native.stream_ptr(c1.device))
    _native.check(rc, op)
    if t1:
        okv.copy_(w1)
    if t2:
        ope.copy_(w2)


def _mla_pair_scatter(kv_linear: torch.Tensor, pe_linear: torch.Tensor, kv_cache: torch.Tensor, pe_cache: torch.Tensor,
                      slots: torch.Tensor, *, layered: bool, op: str) -> None:
    """Linear rows -> latent and rope caches in ONE launch with one last-writer resolution."""
    lib = _native.load()
    l1, _ = _as_unit_inner(kv_linear)
    l2, _ = _as_unit_inner(pe_linear)
    w1, t1 = _as_unit_inner(kv_cache)
    w2, t2 = _as_unit_inner(pe_cache)
    ks, code = kernel_slots(slots)
    _, paged, rb = _mla_cache_side(w1, w2, layered)
    lin = _native.rows_pack(_rows_side_linear(l1, layered), _rows_side_linear(l2, layered))
    n = ks.numel()
    dev = w1.device
    sp = _native.stream_ptr(dev)
    rows = w1.shape[-3] * w1.shape[-2]
    rc = _native.owned_scatter(dev, sp, rows, n, lambda own, orows, epoch: lib.mak_rows_scatterv_owned(
        ctypes.addressof(lin), paged, 2, rb, 0, ks.data_ptr(), code, n, 0, own, orows, epoch, sp))
    if rc is None:
        ws, nbytes = _native.workspace(n, dev)
        rc = lib.mak_rows_scatterv(ctypes.addressof(lin), paged, 2, rb, 0, ks.data_ptr(), code, n, 0, ws.data_ptr(),
                                   nbytes, sp)
    _native.check(rc, op)
    if t1:
        kv_cache.copy_(w1)
    if t2:
        pe_cache.copy_(w2)


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
        _mla_pair_gather(kv_cache, k_pe_cache, slots, okv, ope, layered=False, op=name)
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
        _mla_pair_scatter(kv_linear, k_pe_linear, kv_cache, k_pe_cache, slots, layered=False, op=name)
    emit_native(name, kv_linear, "sm100a row scatter (MLA flat)")


def kv_paged_to_mla_linear_multi_layer(
    kv_cache: torch.Tensor,
    k_pe_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Stacked ``[L, NB, BS, W]`` MLA caches -> ``[L, T, W]`` (reference kv_transfer.py:3982-4050)."""
    name = "kv_paged_to_mla_linear_multi_layer"
    nl, nb, bs, kv_dim, pe_dim = _validate_stacked_mla_shapes(kv_cache, k_pe_cache, name=name)
    dev_id = kv_cache.get_device()
    if k_pe_cache.dtype != kv_cache.dtype or k_pe_cache.get_device() != dev_id:
        raise ValueError(f"{name}: caches must share dtype and device")
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=int(slot_mapping.numel()), name=name)
    if slots.get_device() != dev_id:
        raise ValueError(f"{name}: slot_mapping must share device")
    check_slots_in_bounds(slots, nb, bs, name)
    require_cuda(name, kv_cache, k_pe_cache, slots)
    t = slots.numel()
    okv = torch.empty((nl, t, kv_dim), dtype=kv_cache.dtype, device=kv_cache.device)
    ope = torch.empty((nl, t, pe_dim), dtype=k_pe_cache.dtype, device=kv_cache.device)
    if t:
        _mla_pair_gather(kv_cache, k_pe_cache, slots, okv, ope, layered=True, op=name)
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
    dev_id = kv_cache.get_device()
    if any(t.get_device() != dev_id for t in (kv_linear, k_pe_linear, k_pe_cache, slot_mapping)):
        raise ValueError(f"{name}: all tensors must share device")
    tcount = int(kv_linear.shape[1])
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    check_slots_in_bounds(slots, nb, bs, name)
    require_cuda(name, kv_linear, k_pe_linear, kv_cache, k_pe_cache, slots)
    if tcount:
        _mla_pair_scatter(kv_linear, k_pe_linear, kv_cache, k_pe_cache, slots, layered=True, op=name)
    emit_native(name, kv_linear, "sm100a row scatter (MLA flat, all layers)")
    return True


# ---------------------------------------------------------------------------
# MLA FP8 rows with per-group scales (no reference API: the reference moves
# such rows only as opaque bytes, kv_transfer.py:4411-4452, 4588-4616)
# ---------------------------------------------------------------------------

MLA_FP8_GROUP = 128


def mla_fp8_row_bytes(kv_dim: int = 512, pe_dim: int = 64) -> int:
    """Bytes of one FP8 MLA row: ``kv_dim`` codes, ``kv_dim/128`` fp32 scales, ``pe_dim`` 16-bit rope values
    (512 + 16 + 128 = 656 for DeepSeek MLA)."""
    return int(kv_dim) + (int(kv_dim) // MLA_FP8_GROUP) * 4 + int(pe_dim) * 2


def _mla_fp8_args(kv, pe, cache_rows, name):
    """Normalise to layered views: kv [L,T,kvd], pe [L,T,ped], cache [L,NB,BS,row]."""
    if kv.dim() not in (2, 3) or pe.dim() != kv.dim():
        raise ValueError(f"{name}: latent and rope buffers must both be [T, dim] or [layers, T, dim]")
    if cache_rows.dim() != kv.dim() + 1:
        raise ValueError(f"{name}: cache must be [blocks, block_size, row_bytes] or [layers, blocks, block_size, row_bytes]")
    if kv.dim() == 2:
        kv, pe, cache_rows = kv.unsqueeze(0), pe.unsqueeze(0), cache_rows.unsqueeze(0)
    if kv.shape[:2] != pe.shape[:2] or kv.shape[0] != cache_rows.shape[0]:
        raise ValueError(f"{name}: layer and token counts of latent, rope and cache must agree")
    if kv.dtype not in (torch.float16, torch.bfloat16) or pe.dtype != kv.dtype:
        raise ValueError(f"{name}: latent and rope must share float16 or bfloat16")
    if cache_rows.dtype is not torch.uint8:
        raise ValueError(f"{name}: FP8 row cache storage must be torch.uint8")
    kvd, ped = int(kv.shape[2]), int(pe.shape[2])
    if kvd not in (256, 512, 1024):
        raise ValueError(f"{name}: kv_dim must be 256, 512 or 1024 (groups of 128), got {kvd}")
    if ped % 8 or ped > 256:
        raise ValueError(f"{name}: pe_dim must be a multiple of 8 up to 256, got {ped}")
    if int(cache_rows.shape[3]) != mla_fp8_row_bytes(kvd, ped):
        raise ValueError(f"{name}: cache row is {int(cache_rows.shape[3])} bytes, expected {mla_fp8_row_bytes(kvd, ped)}")
    return kv, pe, cache_rows


def _mla_fp8_descs(kv, pe, cache_rows):
    lin = _native.MlaLinearDesc(kv.data_ptr(), pe.data_ptr(), int(kv.shape[0]), int(kv.shape[1]), int(kv.shape[2]),
                                int(pe.shape[2]), kv.stride(0), kv.stride(1), pe.stride(0), pe.stride(1),
                                _native.dtype_code(kv.dtype), 0)
    key = ("mlafp8", cache_rows.data_ptr(), cache_rows.shape, cache_rows.stride())

    def build():
        base = cache_rows.data_ptr()
        s0, sb, st, _ = cache_rows.stride()
        nb, bs = int(cache_rows.shape[1]), int(cache_rows.shape[2])
        return _native.rows_pack(([base + i * s0 for i in range(cache_rows.shape[0])], bs, sb, st, nb * bs))

    return lin, _native.cached(key, build)


def _rows_ok(t: torch.Tensor, align: int) -> bool:
    e = t.element_size()
    return t.stride(-1) == 1 and (t.data_ptr() | (t.stride(0) * e) | (t.stride(1) * e)) % align == 0


def kv_mla_linear_to_paged_fp8_rows(
    kv_linear: torch.Tensor,
    k_pe_linear: torch.Tensor,
    cache_rows: torch.Tensor,
    slot_mapping: torch.Tensor,
    *,
    fp8_format: Literal["e4m3", "e5m2"] = "e4m3",
) -> bool:
    """Quantise MLA latent rows in groups of 128 and scatter them, with their scales and the rope part,
    into FP8 row caches ``[NB, BS, row]`` / ``[L, NB, BS, row]`` (uint8, ``row = mla_fp8_row_bytes``).

    Group scale = amax of the group's finite |x| / fp8_max (448 E4M3, 57344 E5M2); each value is encoded with the reference
    FP8 rule as ``x / scale`` (kv_transfer.py:2161-2183).  Last writer wins for duplicate slots,
    negative slots are skipped.  One fused launch (plus the duplicate-slot resolution) for all layers.
    """
    name = "kv_mla_linear_to_paged_fp8_rows"
    fmt = _normalize_fp8_format(fp8_format)
    kv, pe, cache = _mla_fp8_args(kv_linear, k_pe_linear, cache_rows, name)
    tcount = int(kv.shape[1])
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    if cache.stride(-1) != 1:
        raise ValueError(f"{name}: cache rows must be contiguous")
    require_cuda(name, kv, pe, cache, slots)
    check_slots_in_bounds(slots, int(cache.shape[1]), int(cache.shape[2]), name)
    if tcount and kv.shape[0]:
        if not _rows_ok(kv, 16):
            kv = kv.contiguous()
        if not _rows_ok(pe, 8):
            pe = pe.contiguous()
        lib = _native.load()
        ks, code = kernel_slots(slots)
        lin, buf = _mla_fp8_descs(kv, pe, cache)
        dev = kv.device
        sp = _native.stream_ptr(dev)
        rows = int(cache.shape[1]) * int(cache.shape[2])
        rc = _native.owned_scatter(dev, sp, rows, tcount, lambda own, orows, epoch: lib.mak_mla_fp8_rows_store_owned(
            ctypes.byref(lin), ctypes.addressof(buf), ks.data_ptr(), code, _FMT_CODE[fmt], own, orows, epoch, sp))
        if rc is None:
            ws, nbytes = _native.workspace(tcount, dev)
            rc = lib.mak_mla_fp8_rows_store(ctypes.byref(lin), ctypes.addressof(buf), ks.data_ptr(), code,
                                            _FMT_CODE[fmt], ws.data_ptr(), nbytes, sp)
        _native.check(rc, name)
    emit_native(name, kv_linear, "sm100a fused group-quantise + row scatter (MLA FP8 rows)")
    return True


def kv_paged_fp8_rows_to_mla_linear(
    cache_rows: torch.Tensor,
    slot_mapping: torch.Tensor,
    *,
    kv_dim: int = 512,
    pe_dim: int = 64,
    out_dtype: torch.dtype = torch.bfloat16,
    fp8_format: Literal["e4m3", "e5m2"] = "e4m3",
    out_kv: torch.Tensor | None = None,
    out_k_pe: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Gather FP8 MLA rows and dequantise them (``code * scale`` in fp32, RNE to ``out_dtype``):
    ``[NB, BS, row]`` -> ``[T, kv_dim]`` + ``[T, pe_dim]``, or ``[L, NB, BS, row]`` -> ``[L, T, ...]``.
    Rows of negative slots are zero.  The rope part is returned bit-exact (stored in ``out_dtype``)."""
    name = "kv_paged_fp8_rows_to_mla_linear"
    fmt = _normalize_fp8_format(fp8_format)
    layered = cache_rows.dim() == 4
    tcount = int(slot_mapping.numel())
    slots = ensure_slotmapping_vector(slot_mapping, expected_len=tcount, name=name)
    lead = (int(cache_rows.shape[0]),) if layered else ()
    okv = out_kv if out_kv is not None else torch.empty(lead + (tcount, kv_dim), dtype=out_dtype, device=cache_rows.device)
    ope = out_k_pe if out_k_pe is not None else torch.empty(lead + (tcount, pe_dim), dtype=out_dtype, device=cache_rows.device)
    if tuple(okv.shape) != lead + (tcount, kv_dim) or tuple(ope.shape) != lead + (tcount, pe_dim):
        raise ValueError(f"{name}: output shapes must be {lead + (tcount, kv_dim)} and {lead + (tcount, pe_dim)}")
    kv, pe, cache = _mla_fp8_args(okv, ope, cache_rows, name)
    if cache.stride(-1) != 1:
        raise ValueError(f"{name}: cache rows must be contiguous")
    require_cuda(name, kv, pe, cache, slots)
    check_slots_in_bounds(slots, int(cache.shape[1]), int(cache.shape[2]), name)
    if tcount and kv.shape[0]:
        work_kv = kv if _rows_ok(kv, 16) else torch.empty(kv.shape, dtype=kv.dtype, device=kv.device)
        work_pe = pe if _rows_ok(pe, 8) else torch.empty(pe.shape, dtype=pe.dtype, device=pe.device)
        lib = _native.load()
        ks, code = kernel_slots(slots)
        lin, buf = _mla_fp8_descs(work_kv, work_pe, cache)
        _native.check(lib.mak_mla_fp8_rows_load(ctypes.addressof(buf), ctypes.byref(lin), ks.data_ptr(), code,
                                                _FMT_CODE[fmt], _native.stream_ptr(kv.device)), name)
        if work_kv is not kv:
            kv.copy_(work_kv)
        if work_pe is not pe:
            pe.copy_(work_pe)
    emit_native(name, cache_rows, "sm100a fused row gather + group dequantise (MLA FP8 rows)")
    return okv, ope


# ---------------------------------------------------------------------------
# Flash-style dense [B, S, NH, HD] layouts (musa_aiter/ops/kv_transfer.py:1527-1795)
# ---------------------------------------------------------------------------


def _index_tensor_ok(t: torch.Tensor) -> bool:
    return t.dtype in (torch.int16, torch.int32, torch.int64)


def _flash_block_check(bt_cpu: torch.Tensor, lens_cpu: torch.Tensor, nb: int, bs: int, name: str) -> None:
    """First invalid block id among the blocks each sequence needs, in sequence-major order."""
    if bt_cpu.numel() == 0 or lens_cpu.numel() == 0:
        return
    needed = (lens_cpu.clamp(min=0) + bs - 1) // bs
    cols = torch.arange(bt_cpu.shape[1]).unsqueeze(0)
    used = cols < needed.unsqueeze(1)
    bad = used & ((bt_cpu < 0) | (bt_cpu >= nb))
    if bool(bad.any()):
        idx = int(torch.nonzero(bad.flatten())[0])
        raise ValueError(f"{name}: invalid block id {int(bt_cpu.flatten()[idx])}")


def _flash_cache_back_check(seq_lens: torch.Tensor, block_tables: torch.Tensor, nb: int, bs: int, dense_len: int,
                            name: str) -> None:
    """kv_transfer.py:1625-1726 checks, sequence by sequence in batch order: the first sequence with a
    length outside [0, dense_len], too few block-table columns, or an invalid block id among the blocks
    it needs raises that error (the checks vectorised over the batch, one host copy of each table)."""
    lens_cpu = seq_lens.to(device="cpu", dtype=torch.long)
    bt_cpu = block_tables.to(device="cpu", dtype=torch.long)
    need = (lens_cpu.clamp(min=0) + bs - 1) // bs
    e_len = (lens_cpu < 0) | (lens_cpu > dense_len)
    e_cols = need > int(bt_cpu.shape[1])
    used = torch.arange(bt_cpu.shape[1]).unsqueeze(0) < need.unsqueeze(1)
    bad = used & ((bt_cpu < 0) | (bt_cpu >= nb))
    err = e_len | e_cols | bad.any(dim=1)
    if not bool(err.any()):
        return
    b = int(torch.nonzero(err)[0])
    if bool(e_len[b]):
        raise ValueError(f"{name}: seq_lens exceeds dense sequence length")
    if bool(e_cols[b]):
        raise ValueError(f"{name}: block_tables does not contain enough columns")
    j = int(torch.nonzero(bad[b])[0])
    raise ValueError(f"{name}: invalid block id {int(bt_cpu[b, j])}")


def _dense_slots(block_tables: torch.Tensor, seq_lens: torch.Tensor, bs: int, dense_len: int) -> torch.Tensor:
    from .kv_transfer_plan import build_slot_mapping

    return build_slot_mapping(block_tables, seq_lens, bs, max_seq_len=dense_len)


def kv_load_and_reshape_flash(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    *,
    max_seq_len: int | None = None,
    out_k: torch.Tensor | None = None,
    out_v: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Paged ``[NB, NH, HD, BS]`` caches -> dense ``[B, S, NH, HD]`` (zero padding).

    Slots come from the block tables on the device (``mak_build_slot_mapping``)
    and one tile-gather launch moves every sequence.  Reference: kv_transfer.py:1527-1622.
    """
    name = "kv_load_and_reshape_flash"
    nb, nh, hd, bs = _validate_paged_shapes(key_cache, value_cache, name=name)
    if block_tables.dim() != 2:
        raise ValueError(f"{name}: block_tables must be [batch, max_blocks]")
    if seq_lens.dim() != 1 or seq_lens.shape[0] != block_tables.shape[0]:
        raise ValueError(f"{name}: seq_lens must be [batch]")
    if key_cache.device != value_cache.device or block_tables.device != key_cache.device or seq_lens.device != key_cache.device:
        raise ValueError(f"{name}: all tensors must be on the same device")
    if not _index_tensor_ok(block_tables):
        raise ValueError(f"{name}: block_tables must use an integer dtype")
    if not _index_tensor_ok(seq_lens):
        raise ValueError(f"{name}: seq_lens must use an integer dtype")
    batch = int(block_tables.shape[0])
    # the host copy of seq_lens serves the length checks and, without max_seq_len, the dense length;
    # with max_seq_len given and validation off it is skipped (the device slot builder clamps)
    check = seq_lens.device.type != "cuda" or validation_enabled()
    lens_cpu = seq_lens.to(device="cpu", dtype=torch.long) if (check or max_seq_len is None) else None
    if lens_cpu is not None and lens_cpu.numel() > 0 and int(lens_cpu.min()) < 0:
        raise ValueError(f"{name}: seq_lens must be non-negative")
    inferred = int(lens_cpu.max()) if lens_cpu is not None and lens_cpu.numel() > 0 else 0
    dense_len = inferred if max_seq_len is None else int(max_seq_len)
    if dense_len < inferred:
        raise ValueError(f"{name}: max_seq_len is smaller than seq_lens max")
    if (dense_len + bs - 1) // bs > int(block_tables.shape[1]):
        raise ValueError(f"{name}: block_tables does not contain enough columns")
    shape = (batch, dense_len, nh, hd)
    for o, c, w in ((out_k, key_cache, "out_k"), (out_v, value_cache, "out_v")):
        if o is not None and (tuple(o.shape) != shape or o.dtype != c.dtype or o.device != c.device):
            raise ValueError(f"{name}: {w} must match [B, S, kv_heads, head_dim] dtype/device")
    if check:
        _flash_block_check(block_tables.to(device="cpu", dtype=torch.long), lens_cpu, nb, bs, name)
    require_cuda(name, key_cache, value_cache, block_tables, seq_lens, out_k, out_v)
    ok = out_k if out_k is not None else torch.empty(shape, dtype=key_cache.dtype, device=key_cache.device)
    ov = out_v if out_v is not None else torch.empty(shape, dtype=value_cache.dtype, device=value_cache.device)
    if batch * dense_len:
        slots = _dense_slots(block_tables, seq_lens, bs, dense_len)
        _tile_gather(key_cache, value_cache, slots, ok.view(batch * dense_len, nh, hd) if ok.is_contiguous() else ok.reshape(-1, nh, hd),
                     ov.view(batch * dense_len, nh, hd) if ov.is_contiguous() else ov.reshape(-1, nh, hd),
                     layered=False, fill_zero=True, op=name)
    emit_native(name, key_cache, "sm100a device slot builder + tile gather (zero padding)")
    return ok, ov


def kv_reshape_and_cache_back_flash(
    dense_k: torch.Tensor,
    dense_v: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
) -> bool:
    """Dense ``[B, S, NH, HD]`` -> paged caches at the block-table slots. Reference: kv_transfer.py:1625-1726."""
    name = "kv_reshape_and_cache_back_flash"
    if dense_k.dim() != 4 or dense_v.dim() != 4:
        raise ValueError("dense Flash KV tensors must be [batch, seq, heads, head_dim]")
    if dense_k.shape != dense_v.shape or dense_k.dtype != dense_v.dtype:
        raise ValueError("dense K and V tensors must have matching shape and dtype")
    if dense_k.device != dense_v.device:
        raise ValueError("dense K and V tensors must be on the same device")
    nb, nh, hd, bs = _validate_paged_shapes(key_cache, value_cache, name=name)
    if key_cache.dtype != dense_k.dtype or value_cache.dtype != dense_v.dtype:
        raise ValueError("dense and paged KV tensors must have matching dtypes")
    if key_cache.device != dense_k.device or value_cache.device != dense_k.device:
        raise ValueError("dense and paged KV tensors must be on the same device")
    if tuple(dense_k.shape[2:]) != (nh, hd):
        raise ValueError("dense KV head shape does not match paged cache")
    if block_tables.dim() != 2:
        raise ValueError(f"{name}: block_tables must be [batch, max_blocks]")
    if seq_lens.dim() != 1 or seq_lens.shape[0] != block_tables.shape[0]:
        raise ValueError(f"{name}: seq_lens must be [batch]")
    if dense_k.shape[0] != block_tables.shape[0]:
        raise ValueError(f"{name}: dense batch does not match block_tables")
    if block_tables.device != dense_k.device or seq_lens.device != dense_k.device:
        raise ValueError(f"{name}: all tensors must be on the same device")
    if not _index_tensor_ok(block_tables):
        raise ValueError(f"{name}: block_tables must use an integer dtype")
    if not _index_tensor_ok(seq_lens):
        raise ValueError(f"{name}: seq_lens must use an integer dtype")
    batch, dense_len = int(dense_k.shape[0]), int(dense_k.shape[1])
    if batch and (seq_lens.device.type != "cuda" or validation_enabled()):
        _flash_cache_back_check(seq_lens, block_tables, nb, bs, dense_len, name)
    require_cuda(name, dense_k, dense_v, key_cache, value_cache, block_tables, seq_lens)
    if batch * dense_len:
        slots = _dense_slots(block_tables, seq_lens, bs, dense_len)
        _tile_scatter(dense_k.reshape(-1, nh, hd), dense_v.reshape(-1, nh, hd), key_cache, value_cache, slots,
                      layered=False, op=name)
    emit_native(name, dense_k, "sm100a device slot builder + tile scatter")
    return True


def kv_load_and_dequantize_fp8_flash(
    key_cache_fp8: torch.Tensor,
    value_cache_fp8: torch.Tensor,
    block_tables: torch.Tensor,
    seq_lens: torch.Tensor,
    k_scale: torch.Tensor | float,
    v_scale: torch.Tensor | float,
    *,
    max_seq_len: int | None = None,
    out_dtype: torch.dtype = torch.bfloat16,
    fp8_format: Literal["e4m3", "e5m2"] = "e4m3",
    out_k: torch.Tensor | None = None,
    out_v: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """FP8 paged caches -> dense dequantized ``[B, S, NH, HD]`` in one fused launch. Reference: kv_transfer.py:1729-1795."""
    name = "kv_load_and_dequantize_fp8_flash"
    fmt = _normalize_fp8_format(fp8_format)
    nb, nh, hd, bs = _validate_paged_shapes(key_cache_fp8, value_cache_fp8, name=name)
    if block_tables.dim() != 2:
        raise ValueError(f"{name}: block_tables must be [batch, max_blocks]")
    if seq_lens.dim() != 1 or seq_lens.shape[0] != block_tables.shape[0]:
        raise ValueError(f"{name}: seq_lens must be [batch]")
    if key_cache_fp8.device != value_cache_fp8.device or block_tables.device != key_cache_fp8.device or seq_lens.device != key_cache_fp8.device:
        raise ValueError(f"{name}: all tensors must be on the same device")
    if not _index_tensor_ok(block_tables) or not _index_tensor_ok(seq_lens):
        raise ValueError(f"{name}: block_tables and seq_lens must be integer tensors")
    batch = int(block_tables.shape[0])
    # the host copy of seq_lens serves the length checks and, without max_seq_len, the dense length;
    # with max_seq_len given and validation off it is skipped (the device slot builder clamps)
    check = seq_lens.device.type != "cuda" or validation_enabled()
    lens_cpu = seq_lens.to(device="cpu", dtype=torch.long) if (check or max_seq_len is None) else None
    if lens_cpu is not None and lens_cpu.numel() > 0 and int(lens_cpu.min()) < 0:
        raise ValueError(f"{name}: seq_lens must be non-negative")
    inferred = int(lens_cpu.max()) if lens_cpu is not None and lens_cpu.numel() > 0 else 0
    dense_len = inferred if max_seq_len is None else int(max_seq_len)
    if dense_len < inferred:
        raise ValueError(f"{name}: max_seq_len is smaller than seq_lens max")
    if (dense_len + bs - 1) // bs > int(block_tables.shape[1]):
        raise ValueError(f"{name}: block_tables does not contain enough columns")
    shape = (batch, dense_len, nh, hd)
    for o, w in ((out_k, "out_k"), (out_v, "out_v")):
        if o is not None and (tuple(o.shape) != shape or o.dtype is not out_dtype or o.device != key_cache_fp8.device):
            raise ValueError(f"{name}: {w} must match [B, S, kv_heads, head_dim] dtype/device")
    if check:
        _flash_block_check(block_tables.to(device="cpu", dtype=torch.long), lens_cpu, nb, bs, name)
    _validate_fp8_cache_tensor(key_cache_fp8, name=f"{name} key_cache_fp8")
    _validate_fp8_cache_tensor(value_cache_fp8, name=f"{name} value_cache_fp8")
    require_cuda(name, key_cache_fp8, value_cache_fp8, block_tables, seq_lens, out_k, out_v)
    ok = out_k if out_k is not None else torch.empty(shape, dtype=out_dtype, device=key_cache_fp8.device)
    ov = out_v if out_v is not None else torch.empty(shape, dtype=out_dtype, device=key_cache_fp8.device)
    if batch * dense_len:
        ks = _ensure_fp8_scale(k_scale, device=key_cache_fp8.device, name="k_scale", num_heads=nh)
        vs = _ensure_fp8_scale(v_scale, device=key_cache_fp8.device, name="v_scale", num_heads=nh)
        ksa, vsa, mode = _scale_args(ks, vs, 1, nh)
        slots = _dense_slots(block_tables, seq_lens, bs, dense_len)
        _tile_gather(_u8_view(key_cache_fp8), _u8_view(value_cache_fp8), slots, ok.reshape(-1, nh, hd), ov.reshape(-1, nh, hd),
                     layered=False, fill_zero=True, op=name, fp8=(ksa, vsa, mode, _FMT_CODE[fmt]))
    emit_native(name, key_cache_fp8, f"sm100a fused FP8 {fmt} dense dequantize gather")
    return ok, ov


def kv_triton_indexed_to_dense(
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    kv_indptr: torch.Tensor,
    kv_indices: torch.Tensor,
    *,
    max_seq_len: int,
    out_k: torch.Tensor | None = None,
    out_v: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """SGLang token pool ``[Ntok, NH, HD]`` + CSR indices -> dense ``[B, S, NH, HD]`` (zero padding).

    No host sync: the dense slot vector is built on the device
    (``mak_build_indexed_slots``) and one row-gather launch moves K and V.
    Reference: kv_transfer.py:1291-1366.
    """
    name = "kv_triton_indexed_to_dense"
    if key_cache.dim() != 3 or value_cache.dim() != 3:
        raise ValueError(f"{name}: key/value cache must be [tokens, kv_heads, head_dim]")
    if key_cache.shape != value_cache.shape or key_cache.dtype != value_cache.dtype or key_cache.device != value_cache.device:
        raise ValueError(f"{name}: key/value cache shape, dtype, and device must match")
    if kv_indptr.dim() != 1 or kv_indptr.numel() < 2:
        raise ValueError(f"{name}: kv_indptr must be [batch + 1]")
    if kv_indices.dim() != 1:
        raise ValueError(f"{name}: kv_indices must be 1-D")
    if kv_indptr.device != key_cache.device or kv_indices.device != key_cache.device:
        raise ValueError(f"{name}: all tensors must be on the same device")
    if not _index_tensor_ok(kv_indptr) or not _index_tensor_ok(kv_indices):
        raise ValueError(f"{name}: indices must use integer dtype")
    batch = int(kv_indptr.shape[0] - 1)
    dense_len = int(max_seq_len)
    if dense_len < 0:
        raise ValueError(f"{name}: max_seq_len must be non-negative")
    ntok, nh, hd = map(int, key_cache.shape)
    shape = (batch, dense_len, nh, hd)
    for o, c, w in ((out_k, key_cache, "out_k"), (out_v, value_cache, "out_v")):
        if o is not None and (tuple(o.shape) != shape or o.dtype != c.dtype or o.device != c.device or not o.is_contiguous()):
            raise ValueError(f"{name}: {w} must match [B, S, kv_heads, head_dim] dtype/device and be contiguous")
    require_cuda(name, key_cache, value_cache, kv_indptr, kv_indices, out_k, out_v)
    ok = out_k if out_k is not None else torch.empty(shape, dtype=key_cache.dtype, device=key_cache.device)
    ov = out_v if out_v is not None else torch.empty(shape, dtype=value_cache.dtype, device=key_cache.device)
    total = batch * dense_len
    if total:
        lib = _native.load()
        ip, ip_code = kernel_slots(kv_indptr)
        ix, ix_code = kernel_slots(kv_indices)
        slots = torch.empty(total, dtype=torch.int64, device=key_cache.device)
        stream = _native.stream_ptr(key_cache.device)
        _native.check(lib.mak_build_indexed_slots(_native.ptr(ip), ip_code, _native.ptr(ix), ix_code, ix.numel(), batch,
                                                  dense_len, _native.ptr(slots), stream), name)
        kc, _ = _as_unit_inner(key_cache)
        vc, _ = _as_unit_inner(value_cache)
        if kc.stride(1) != hd or vc.stride(1) != hd:
            kc, vc = kc.contiguous(), vc.contiguous()
        e = kc.element_size()
        pd, pa = _native.rows_desc([kc.data_ptr(), vc.data_ptr()], 1, kc.stride(0) * e, 0, ntok)
        ld, la = _native.rows_desc([ok.data_ptr(), ov.data_ptr()], 1, nh * hd * e, 0, total)
        _native.check(lib.mak_rows_gather(ctypes.byref(pd), ctypes.byref(ld), None, nh * hd * e, _native.ptr(slots),
                                          _native.MAK_DT_I64, total, 1, stream), name)
    emit_native(name, key_cache, "sm100a device CSR slot builder + row gather")
    return ok, ov


# ---------------------------------------------------------------------------
# whole-block copies (musa_aiter/ops/kv_transfer.py:1871-2091)
# ---------------------------------------------------------------------------


def _validate_block_copy_shapes(src_k, src_v, dst_k, dst_v, *, name: str) -> tuple[int, int, bool]:
    if src_k.shape != src_v.shape:
        raise ValueError(f"{name}: source key/value cache shapes must match")
    if dst_k.shape != dst_v.shape:
        raise ValueError(f"{name}: destination key/value cache shapes must match")
    if src_k.dim() not in (4, 5) or dst_k.dim() != src_k.dim():
        raise ValueError(f"{name}: caches must be 4-D single-layer or 5-D multi-layer paged tensors")
    if src_k.dtype != src_v.dtype or dst_k.dtype != dst_v.dtype:
        raise ValueError(f"{name}: key/value dtype pairs must match")
    if src_k.dtype != dst_k.dtype:
        raise ValueError(f"{name}: source and destination dtypes must match")
    if src_k.dim() == 4:
        if src_k.shape[1:] != dst_k.shape[1:]:
            raise ValueError(f"{name}: single-layer cache tails must match")
        return int(src_k.shape[0]), int(dst_k.shape[0]), False
    if src_k.shape[0] != dst_k.shape[0] or src_k.shape[2:] != dst_k.shape[2:]:
        raise ValueError(f"{name}: multi-layer cache layer count and tails must match")
    return int(src_k.shape[1]), int(dst_k.shape[1]), True


def _ensure_block_mapping_pairs(block_mapping: torch.Tensor, *, src_blocks: int, dst_blocks: int, name: str) -> torch.Tensor:
    if block_mapping.dim() != 2 or block_mapping.shape[1] != 2:
        raise ValueError(f"{name}: block_mapping must be [num_pairs, 2] with source and destination block ids")
    if not _index_tensor_ok(block_mapping):
        raise ValueError(f"{name}: block_mapping must use an integer dtype")
    pairs = block_mapping.to(device="cpu", dtype=torch.long)
    if pairs.numel() == 0:
        return pairs
    valid = (pairs[:, 0] >= 0) & (pairs[:, 1] >= 0)
    if not bool(valid.any()):
        return pairs
    src_max = int(pairs[valid, 0].max())
    dst_max = int(pairs[valid, 1].max())
    if src_max >= src_blocks:
        raise ValueError(f"{name}: source block index {src_max} out of bounds for {src_blocks} blocks")
    if dst_max >= dst_blocks:
        raise ValueError(f"{name}: destination block index {dst_max} out of bounds for {dst_blocks} blocks")
    return pairs


def _count_and_copy_blocks(block_mapping: torch.Tensor, dst: torch.Tensor, *, src_blocks: int, dst_blocks: int,
                           name: str, launch) -> int:
    """Valid-pair count of ``block_mapping`` and ``launch(device int64 pairs)`` for the copy.

    With validation off and the mapping already on the caches' device, the host neither copies
    the mapping back for bounds checks (the row kernel skips out-of-range blocks) nor waits for
    the stream before launching: the count goes to pinned memory behind an event, the copy is
    queued, and the host waits for the count only, so the next call's host work overlaps this
    copy.  Otherwise the reference's host checks run first (ValueError on out-of-range blocks).
    """
    if block_mapping.device == dst.device and not validation_enabled():
        if block_mapping.dim() != 2 or block_mapping.shape[1] != 2:
            raise ValueError(f"{name}: block_mapping must be [num_pairs, 2] with source and destination block ids")
        if not _index_tensor_ok(block_mapping):
            raise ValueError(f"{name}: block_mapping must use an integer dtype")
        if block_mapping.numel() == 0:
            return 0
        pairs = block_mapping.to(dtype=torch.int64)
        host = torch.empty((), dtype=torch.int64, pin_memory=True)
        host.copy_(((pairs[:, 0] >= 0) & (pairs[:, 1] >= 0)).sum(), non_blocking=True)
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream(dst.device))
        launch(pairs)
        ready.synchronize()
        return int(host)
    pairs = _ensure_block_mapping_pairs(block_mapping, src_blocks=src_blocks, dst_blocks=dst_blocks, name=name)
    count = int(((pairs[:, 0] >= 0) & (pairs[:, 1] >= 0)).sum()) if pairs.numel() else 0
    if count:
        launch(block_mapping.to(device=dst.device, dtype=torch.int64))
    return count


def _block_planes(k: torch.Tensor, v: torch.Tensor, multi_layer: bool):
    """One plane per (kv, layer); a row is one whole block (its [NH, HD, BS] tail must be contiguous)."""
    e = k.element_size()
    planes = []
    for t in (k, v):
        if multi_layer:
            planes += [t.data_ptr() + l * t.stride(0) * e for l in range(t.shape[0])]
        else:
            planes.append(t.data_ptr())
    bdim = 1 if multi_layer else 0
    return planes, k.stride(bdim) * e, int(k.shape[bdim])


def _block_tail_contiguous(t: torch.Tensor, multi_layer: bool) -> bool:
    tail = t[0, 0] if multi_layer else t[0]
    return tail.is_contiguous()


def _copy_blocks(src_k, src_v, dst_k, dst_v, pairs_dev: torch.Tensor, multi_layer: bool, name: str) -> None:
    for t in (src_k, src_v, dst_k, dst_v):
        if not _block_tail_contiguous(t, multi_layer) or (multi_layer and t.stride(0) % 1):
            raise ValueError(f"{name}: each cache block must be contiguous")
    if src_k.stride() != src_v.stride() or dst_k.stride() != dst_v.stride():
        raise ValueError(f"{name}: key and value caches must share strides")
    sp, s_bstride, s_nb = _block_planes(src_k, src_v, multi_layer)
    dp, d_bstride, d_nb = _block_planes(dst_k, dst_v, multi_layer)
    tail = src_k[0, 0] if multi_layer else src_k[0]
    row = tail.numel() * src_k.element_size()
    src_idx = pairs_dev[:, 0].contiguous()
    dst_idx = torch.where(src_idx >= 0, pairs_dev[:, 1], torch.full_like(src_idx, -1)).contiguous()
    n = int(src_idx.numel())
    sd, sa = _native.rows_desc(sp, 1, s_bstride, 0, s_nb)
    dd, da = _native.rows_desc(dp, 1, d_bstride, 0, d_nb)
    rc = _native.rows_copy(ctypes.byref(sd), ctypes.byref(dd), row, _native.ptr(src_idx), _native.MAK_DT_I64,
                           _native.ptr(dst_idx), _native.MAK_DT_I64, n, d_nb, dst_k.device,
                           _native.stream_ptr(dst_k.device))
    _native.check(rc, name)


def kv_copy_paged_blocks(
    src_key_cache: torch.Tensor,
    src_value_cache: torch.Tensor,
    dst_key_cache: torch.Tensor,
    dst_value_cache: torch.Tensor,
    block_mapping: torch.Tensor,
) -> int:
    """Copy whole blocks by ``[P, 2]`` (src, dst) pairs for 1 or L layers; returns the valid-pair count.

    Every (kv, layer) plane goes in one row-engine launch (a block is one row).
    Reference: kv_transfer.py:2035-2091.
    """
    name = "kv_copy_paged_blocks"
    src_blocks, dst_blocks, multi = _validate_block_copy_shapes(src_key_cache, src_value_cache, dst_key_cache,
                                                                dst_value_cache, name=name)
    require_cuda(name, src_key_cache, src_value_cache, dst_key_cache, dst_value_cache)
    count = _count_and_copy_blocks(
        block_mapping, dst_key_cache, src_blocks=src_blocks, dst_blocks=dst_blocks, name=name,
        launch=lambda dp: _copy_blocks(src_key_cache, src_value_cache, dst_key_cache, dst_value_cache, dp, multi, name))
    emit_native(name, dst_key_cache, "sm100a row engine, one block per row")
    return count


def kv_copy_paged_blocks_fp8(
    src_key_cache_fp8: torch.Tensor,
    src_value_cache_fp8: torch.Tensor,
    dst_key_cache_fp8: torch.Tensor,
    dst_value_cache_fp8: torch.Tensor,
    block_mapping: torch.Tensor,
) -> int:
    """Raw FP8 (uint8 / float8) block copy. Reference: kv_transfer.py:1871-1906."""
    name = "kv_copy_paged_blocks_fp8"
    src_blocks, dst_blocks, multi = _validate_block_copy_shapes(src_key_cache_fp8, src_value_cache_fp8, dst_key_cache_fp8,
                                                                dst_value_cache_fp8, name=name)
    for t in (src_key_cache_fp8, src_value_cache_fp8, dst_key_cache_fp8, dst_value_cache_fp8):
        _validate_fp8_cache_tensor(t, name=name)
    require_cuda(name, src_key_cache_fp8, src_value_cache_fp8, dst_key_cache_fp8, dst_value_cache_fp8)
    count = _count_and_copy_blocks(
        block_mapping, dst_key_cache_fp8, src_blocks=src_blocks, dst_blocks=dst_blocks, name=name,
        launch=lambda dp: _copy_blocks(_u8_view(src_key_cache_fp8), _u8_view(src_value_cache_fp8),
                                       _u8_view(dst_key_cache_fp8), _u8_view(dst_value_cache_fp8), dp, multi, name))
    emit_native(name, dst_key_cache_fp8, "sm100a row engine, one FP8 block per row")
    return count


# ---------------------------------------------------------------------------
# DSV4 opaque byte rows (musa_aiter/ops/kv_transfer.py:4411-4736)
# ---------------------------------------------------------------------------

import threading as _threading  # noqa: E402
import time as _time  # noqa: E402
from dataclasses import dataclass as _dataclass  # noqa: E402

from .kv_layout import KVLayoutSpec, KVScaleKind  # noqa: E402


@_dataclass(frozen=True)
class InterleavedFp8Layout:
    """DSV4 interleaved FP8 block-scale page row: ``[value region][scale region]``.

    Same fields and checks as the reference descriptor (kv_transfer.py:4411-4452).
    """

    value_bytes: int
    scale_bytes: int
    scale_granularity: int

    def __post_init__(self) -> None:
        if self.value_bytes <= 0 or self.scale_bytes <= 0:
            raise ValueError("InterleavedFp8Layout: value_bytes and scale_bytes must be positive")
        if self.scale_granularity <= 0:
            raise ValueError("InterleavedFp8Layout: scale_granularity must be positive")

    @property
    def item_bytes(self) -> int:
        return self.value_bytes + self.scale_bytes

    def as_kv_layout_spec(self, *, num_layers: int, num_blocks: int, block_size: int, dtype_name: str = "uint8") -> KVLayoutSpec:
        return KVLayoutSpec.dsv4(num_layers=num_layers, num_blocks=num_blocks, block_size=block_size,
                                 row_bytes=self.item_bytes, block_stride_bytes=self.item_bytes * block_size,
                                 dtype_name=dtype_name, scale_kind=KVScaleKind.BLOCKED, value_bytes=self.value_bytes,
                                 scale_bytes=self.scale_bytes)


@_dataclass
class PoolSpec:
    """One pool of a DSV4 multi-pool copy: per-layer uint8 ``[pages, item_bytes]`` tensors."""

    src_ptrs: list
    dst_ptrs: list
    item_bytes: int


_stats_lock = _threading.Lock()
_stats = {"pinned_calls": 0, "unpinned_calls": 0, "pinned_bytes": 0, "unpinned_bytes": 0,
          "pinned_ns_total": 0, "unpinned_ns_total": 0}


def kv_transfer_stats() -> dict:
    """Pinned vs unpinned call counts, bytes and host-side ns of the byte-row copies."""
    with _stats_lock:
        return dict(_stats)


def reset_kv_transfer_stats() -> None:
    with _stats_lock:
        for k in _stats:
            _stats[k] = 0


def _record_stats(src: torch.Tensor, dst: torch.Tensor, rows: int, item_bytes: int, ns: int) -> None:
    host = src if src.device.type == "cpu" else (dst if dst.device.type == "cpu" else None)
    pinned = host is None or bool(host.is_pinned())
    key = "pinned" if pinned else "unpinned"
    with _stats_lock:
        _stats[f"{key}_calls"] += 1
        _stats[f"{key}_bytes"] += rows * item_bytes
        _stats[f"{key}_ns_total"] += ns


def _check_row_indices(indices: torch.Tensor, num_rows: int, name: str) -> None:
    """Host indices are range-checked eagerly (IndexError); device indices are guarded in the kernel."""
    if indices.numel() == 0 or indices.device.type != "cpu":
        return
    idx = indices.to(torch.long)
    lo, hi = int(idx.min()), int(idx.max())
    if lo < 0:
        raise IndexError(f"{name} row index {lo} is negative")
    if hi >= num_rows:
        raise IndexError(f"{name} row index {hi} out of bounds for {num_rows} rows")


def _validate_rows_args(src, dst, src_indices, dst_indices, *, name: str) -> int:
    if not isinstance(src, torch.Tensor) or not isinstance(dst, torch.Tensor):
        raise TypeError(f"{name}: src and dst must be torch.Tensor")
    if src.dtype is not torch.uint8 or dst.dtype is not torch.uint8:
        raise ValueError(f"{name}: src and dst must be uint8 byte rows, got src={src.dtype}, dst={dst.dtype}")
    if src.dim() != 2 or dst.dim() != 2:
        raise ValueError(f"{name}: src and dst must be [rows, item_bytes]")
    item = int(src.shape[1])
    if int(dst.shape[1]) != item:
        raise ValueError(f"{name}: src and dst item_bytes must match, got src={item}, dst={int(dst.shape[1])}")
    if item <= 0:
        raise ValueError(f"{name}: item_bytes must be positive")
    for ix in (src_indices, dst_indices):
        if not (isinstance(ix, torch.Tensor) and ix.dim() == 1 and _index_tensor_ok(ix)):
            raise ValueError(f"{name}: indices must use an integer dtype")
    if src_indices.numel() != dst_indices.numel():
        raise ValueError(f"{name}: src_indices and dst_indices must have the same length")
    _check_row_indices(src_indices, int(src.shape[0]), f"{name}: src")
    _check_row_indices(dst_indices, int(dst.shape[0]), f"{name}: dst")
    return item


def _addressable(t: torch.Tensor) -> bool:
    """The GPU can address CUDA tensors and pinned host tensors (unified addressing)."""
    return t.device.type == "cuda" or (t.device.type == "cpu" and bool(t.is_pinned()))


def _rows_copy_planes(srcs: list[torch.Tensor], dsts: list[torch.Tensor], src_indices, dst_indices, name: str) -> None:
    """dst[l][dst_idx[i]] = src[l][src_idx[i]] for every plane pair, one launch."""
    _native.load()
    s0, d0 = srcs[0], dsts[0]
    dev = s0.device if s0.device.type == "cuda" else d0.device
    if dev.type != "cuda":
        raise RuntimeError(f"{name}: at least one side must be a CUDA tensor")
    for side, first in ((srcs, s0), (dsts, d0)):
        for t in side:
            if not _addressable(t):
                raise RuntimeError(f"{name}: host tensors must be pinned for the GPU to address them")
            if t.stride(1) != 1 or t.stride() != first.stride() or t.shape[0] != first.shape[0]:
                raise ValueError(f"{name}: byte rows must be contiguous and share one geometry per side")
    si, sc = kernel_slots(src_indices.to(dev))
    di, dc = kernel_slots(dst_indices.to(dev))
    n = int(si.numel())
    if n == 0:
        return
    sd, sa = _native.rows_desc([t.data_ptr() for t in srcs], 1, s0.stride(0), 0, int(s0.shape[0]))
    dd, da = _native.rows_desc([t.data_ptr() for t in dsts], 1, d0.stride(0), 0, int(d0.shape[0]))
    rc = _native.rows_copy(ctypes.byref(sd), ctypes.byref(dd), int(s0.shape[1]), _native.ptr(si), sc, _native.ptr(di), dc,
                           n, int(d0.shape[0]), dev, _native.stream_ptr(dev))
    _native.check(rc, name)


def kv_copy_paged_rows(
    src: torch.Tensor,
    dst: torch.Tensor,
    src_indices: torch.Tensor,
    dst_indices: torch.Tensor,
    *,
    layout: InterleavedFp8Layout | None = None,
) -> None:
    """``dst[dst_indices[i]] = src[src_indices[i]]`` for uint8 byte rows (DSV4 pages).

    Host index tensors are range-checked (IndexError); device indices are guarded
    in the kernel and out-of-range rows are skipped, as in the reference
    (kv_transfer.py:4518-4557).  Source or destination may be pinned host memory.
    """
    name = "kv_copy_paged_rows"
    item = _validate_rows_args(src, dst, src_indices, dst_indices, name=name)
    if layout is not None and layout.item_bytes != item:
        raise ValueError(f"{name}: layout.item_bytes={layout.item_bytes} != tensor row width {item}")
    t0 = _time.perf_counter_ns()
    _rows_copy_planes([src], [dst], src_indices, dst_indices, name)
    _record_stats(src, dst, int(src_indices.numel()), item, _time.perf_counter_ns() - t0)
    emit_native(name, src, "sm100a row engine (DSV4 byte rows)")


def _validate_layer_table(src_ptrs, dst_ptrs, src_indices, dst_indices, *, name: str) -> int:
    if not isinstance(src_ptrs, (list, tuple)) or not isinstance(dst_ptrs, (list, tuple)):
        raise TypeError(f"{name}: src_ptrs and dst_ptrs must be lists of tensors")
    if len(src_ptrs) == 0 or len(dst_ptrs) == 0:
        raise ValueError(f"{name}: ptr-tables must be non-empty")
    if len(src_ptrs) != len(dst_ptrs):
        raise ValueError(f"{name}: src/dst layer counts must match, got {len(src_ptrs)} vs {len(dst_ptrs)}")
    item = int(src_ptrs[0].shape[1])
    for layer, (s, d) in enumerate(zip(src_ptrs, dst_ptrs)):
        _validate_rows_args(s, d, src_indices, dst_indices, name=f"{name}[layer{layer}]")
        if int(d.shape[1]) != item:
            raise ValueError(f"{name}: layer {layer} item_bytes mismatch, expected {item}, got {int(d.shape[1])}")
    return item


def kv_copy_paged_rows_layer_table(src_ptrs, dst_ptrs, src_indices: torch.Tensor, dst_indices: torch.Tensor) -> None:
    """All layers' byte-row copies in one launch (plane pointers in the kernel parameters).

    Reference: kv_transfer.py:4588-4616.
    """
    name = "kv_copy_paged_rows_layer_table"
    item = _validate_layer_table(src_ptrs, dst_ptrs, src_indices, dst_indices, name=name)
    t0 = _time.perf_counter_ns()
    _rows_copy_planes(list(src_ptrs), list(dst_ptrs), src_indices, dst_indices, name)
    _record_stats(src_ptrs[0], dst_ptrs[0], int(src_indices.numel()) * len(src_ptrs), item, _time.perf_counter_ns() - t0)
    emit_native(name, src_ptrs[0], f"sm100a row engine ({len(src_ptrs)} layers, item_bytes={item}, one launch)")


def kv_copy_paged_rows_multi_pool(pools: list[PoolSpec], indices: torch.Tensor, *, direction: Literal["H2D", "D2H"]) -> None:
    """Pools sharing one page-index vector (DSV4 KV/SWA/C4/C128/indexer/state), H2D or D2H.

    Pinned host pools are addressed by the kernel directly; a pageable host
    pool cannot be addressed by the GPU, so its rows are staged through a
    pinned bounce buffer (the host-side index copy runs on the CPU there).
    Reference: kv_transfer.py:4619-4660.
    """
    name = "kv_copy_paged_rows_multi_pool"
    if direction not in ("H2D", "D2H"):
        raise ValueError(f"{name}: direction must be 'H2D' or 'D2H', got {direction!r}")
    if not isinstance(pools, (list, tuple)) or len(pools) == 0:
        raise ValueError(f"{name}: pools must be a non-empty list of PoolSpec")
    for i, pool in enumerate(pools):
        if not isinstance(pool, PoolSpec):
            raise TypeError(f"{name}: pools[{i}] must be PoolSpec")
        item = _validate_layer_table(pool.src_ptrs, pool.dst_ptrs, indices, indices, name=f"{name}[pool{i}]")
        if pool.item_bytes != item:
            raise ValueError(f"{name}: pools[{i}].item_bytes={pool.item_bytes} != tensor row width {item}")
    for pool in pools:
        t0 = _time.perf_counter_ns()
        srcs, dsts = list(pool.src_ptrs), list(pool.dst_ptrs)
        if all(_addressable(t) for t in srcs + dsts):
            _rows_copy_planes(srcs, dsts, indices, indices, name)
        else:
            for s, d in zip(srcs, dsts):
                _staged_rows_copy(s, d, indices, name)
        _record_stats(srcs[0], dsts[0], int(indices.numel()) * len(srcs), pool.item_bytes, _time.perf_counter_ns() - t0)
    emit_native(name, pools[0].dst_ptrs[0] if direction == "H2D" else pools[0].src_ptrs[0],
                f"sm100a row engine ({len(pools)} pools, direction={direction})")


_bounce_lock = _threading.Lock()
_bounce_in_flight: list = []  # (event, pinned bounce buffer) pairs still read by a queued kernel


def _hold_bounce(bounce: torch.Tensor, dev: torch.device) -> None:
    """Keep a pinned bounce buffer alive until the kernel queued on the current stream that
    reads it has run: torch's pinned-memory cache would otherwise hand the block to the next
    ``pin_memory`` allocation as soon as the tensor is released, while the copy is still queued."""
    ev = torch.cuda.Event()
    ev.record(torch.cuda.current_stream(dev))
    with _bounce_lock:
        _bounce_in_flight[:] = [(e, b) for e, b in _bounce_in_flight if not e.query()]
        _bounce_in_flight.append((ev, bounce))


def _staged_rows_copy(src: torch.Tensor, dst: torch.Tensor, indices: torch.Tensor, name: str) -> None:
    """Copy rows where one side is pageable host memory, through a pinned bounce buffer."""
    rows = indices.to(torch.long)
    n = int(rows.numel())
    if n == 0:
        return
    if src.device.type == "cpu" and not src.is_pinned():
        bounce = torch.empty((n, src.shape[1]), dtype=torch.uint8, pin_memory=True)
        torch.index_select(src, 0, rows.cpu(), out=bounce)
        ident = torch.arange(n, device=dst.device if dst.device.type == "cuda" else "cpu")
        _rows_copy_planes([bounce], [dst], ident, rows.to(ident.device), name)
        if dst.device.type == "cuda":
            _hold_bounce(bounce, dst.device)
    else:
        bounce = torch.empty((n, dst.shape[1]), dtype=torch.uint8, pin_memory=True)
        dev = src.device
        ident = torch.arange(n, device=dev)
        _rows_copy_planes([src], [bounce], rows.to(dev), ident, name)
        torch.cuda.current_stream(dev).synchronize()
        dst.index_copy_(0, rows.cpu(), bounce)


# ---------------------------------------------------------------------------
# CacheGen-style codec (musa_aiter/ops/kv_transfer.py:1111-1217)
# ---------------------------------------------------------------------------


def kv_cachegen_encode(tensor: torch.Tensor, *, num_bins: int = 256) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Uniform-bin uint8 encode with codebook and empirical CDF, all computed on the device with
    no read-back (the reference reads min/max back for ``torch.linspace``; the device codebook is
    bit-identical to it).  Reference: kv_transfer.py:1111-1172."""
    name = "kv_cachegen_encode"
    if num_bins < 2 or num_bins > 256:
        raise ValueError(f"{name}: num_bins must be in [2, 256]")
    if not tensor.is_floating_point():
        raise ValueError(f"{name}: tensor must use a floating dtype")
    require_cuda(name, tensor)
    dev = tensor.device
    if tensor.numel() == 0:
        return (torch.empty_like(tensor, dtype=torch.uint8), torch.zeros(num_bins, dtype=torch.float32, device=dev),
                torch.zeros(num_bins + 1, dtype=torch.float32, device=dev))
    if tensor.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        tensor = tensor.float()
    x = tensor.contiguous()
    lib = _native.load()
    stream = _native.stream_ptr(dev)
    code = _native.dtype_code(x.dtype)
    mm = torch.empty(2, dtype=torch.float32, device=dev)
    _native.check(lib.mak_minmax(_native.ptr(x), code, x.numel(), _native.ptr(mm), stream), name)
    # Everything stays on the device: min/max, the codes with their histogram and CDF, and the
    # codebook (torch.linspace's float32 arithmetic, or min in every bin when max == min), so the
    # call queues its launches and returns without waiting for the stream.  A slab with
    # max == min takes the same launches: every code is 0 (the NaN of 0 * inf is clamped to 0),
    # so counts = [n, 0, ...] and the CDF is [0, 1, ..., 1].
    codes = torch.empty(x.shape, dtype=torch.uint8, device=dev)
    counts = torch.empty(num_bins, dtype=torch.int64, device=dev)
    cdf = torch.empty(num_bins + 1, dtype=torch.float32, device=dev)
    codebook = torch.empty(num_bins, dtype=torch.float32, device=dev)
    _native.check(lib.mak_cachegen_encode(_native.ptr(x), code, x.numel(), _native.ptr(mm), num_bins, _native.ptr(codes),
                                          _native.ptr(counts), _native.ptr(cdf), stream), name)
    _native.check(lib.mak_cachegen_codebook(_native.ptr(mm), num_bins, _native.ptr(codebook), stream), name)
    emit_native(name, tensor, "sm100a min/max + encode/histogram + CDF kernels")
    return codes, codebook, cdf


def kv_cachegen_decode(encoded: torch.Tensor, codebook: torch.Tensor, *, dtype: torch.dtype | None = None) -> torch.Tensor:
    """``codebook[encoded]`` (optionally cast to ``dtype``). Reference: kv_transfer.py:1175-1217."""
    name = "kv_cachegen_decode"
    if encoded.dtype != torch.uint8:
        raise ValueError(f"{name}: encoded must be uint8")
    if codebook.dim() != 1 or codebook.numel() < 2 or codebook.numel() > 256:
        raise ValueError(f"{name}: codebook must be 1-D with 2..256 bins")
    if codebook.device != encoded.device:
        raise ValueError(f"{name}: encoded and codebook must be on same device")
    if not codebook.is_floating_point():
        raise ValueError(f"{name}: codebook must use a floating dtype")
    if encoded.numel() > 0 and (encoded.device.type != "cuda" or validation_enabled()) and \
            int(encoded.max().item()) >= int(codebook.numel()):
        raise ValueError(f"{name}: encoded bin exceeds codebook size")
    require_cuda(name, encoded, codebook)
    out_dtype = codebook.dtype if dtype is None else dtype
    cb = codebook if codebook.dtype in (torch.float16, torch.bfloat16, torch.float32) else codebook.float()
    cb = cb.contiguous()
    enc = encoded.contiguous()
    work_dtype = out_dtype if out_dtype in (torch.float16, torch.bfloat16, torch.float32) else torch.float32
    out = torch.empty(enc.shape, dtype=work_dtype, device=enc.device)
    if enc.numel():
        rc = _native.load().mak_cachegen_decode(_native.ptr(enc), enc.numel(), _native.ptr(cb), _native.dtype_code(cb.dtype),
                                                cb.numel(), _native.ptr(out), _native.dtype_code(work_dtype),
                                                _native.stream_ptr(enc.device))
        _native.check(rc, name)
    emit_native(name, encoded, "sm100a codebook decode")
    return out if work_dtype == out_dtype else out.to(out_dtype)
