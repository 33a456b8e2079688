"""LMCache / SGLang-MP KV buffer pack and unpack on B200.

Same public ABI as the reference facade (musa_aiter/ops/lmcache_kv_transfer.py):
the legacy 6-D cache ``[NL, 2, NB, BS, NH, HS]``, LMCache layer lists of
``[2, NB, BS, NH, HS]``, SGLang MP ``2 x NL x [NB, BS, NH, HS]`` split caches,
and the MLA ``[NL, NB, BS, HS]`` / list forms, against contiguous (or strided)
LMCache buffers ``[2, NL, T, NH*HS]`` / ``[NL, T, HS]`` / ``[1, NL, T, HS]``.

Every form maps onto the row engine of ``libmak_kvcache.so``: each (kv, layer)
cache tensor is one plane, a token row (NH*HS elements) is the unit, and ALL
planes move in one launch whatever their count (the reference launches once
per (kv, layer) or caps the pointer table at 64-128 layers,
csrc/kvcache/lmcache_kv_transfer_ext.cpp:200, kv_transfer_float.mu:2032-2086).
Strided buffers are addressed in place through per-plane pointers, so
non-contiguous memory tensors need no staging copy.
"""

from __future__ import annotations

import ctypes
from typing import Any

import torch

from .. import _native
from ..dispatch import emit_native
from ._common import kernel_slots, require_cuda

_LMCACHE_KV_TRANSFER_ABI_VERSION = 1

__all__ = [
    "clear_native_lmcache_kv_transfer_cache",
    "is_native_lmcache_kv_transfer_available",
    "is_native_lmcache_two_x_nl_kv_transfer_available",
    "native_lmcache_kv_transfer_abi_version",
    "lmcache_kv_buffer_to_paged",
    "lmcache_paged_to_kv_buffer",
    "lmcache_kv_buffer_to_paged_mla",
    "lmcache_paged_to_kv_buffer_mla",
    "lmcache_kv_paged_to_buffer",
    "lmcache_kv_buffer_to_paged_two_x_nl",
    "lmcache_kv_paged_to_buffer_two_x_nl",
    "lmcache_mla_buffer_to_paged",
    "lmcache_mla_paged_to_buffer",
]


def native_lmcache_kv_transfer_abi_version() -> int:
    return _LMCACHE_KV_TRANSFER_ABI_VERSION


def clear_native_lmcache_kv_transfer_cache() -> None:
    """Nothing is cached per symbol here (prototypes are bound once at load)."""


def is_native_lmcache_kv_transfer_available() -> bool:
    return _native.is_available()


def is_native_lmcache_two_x_nl_kv_transfer_available() -> bool:
    return _native.is_available()


# ---------------------------------------------------------------------------
# row-plane descriptors
# ---------------------------------------------------------------------------


def _row_elems(t: torch.Tensor, lead: int) -> int:
    n = 1
    for s in t.shape[lead:]:
        n *= int(s)
    return n


def _rows_contiguous(t: torch.Tensor, lead: int) -> bool:
    """True when the dims after the first ``lead`` ones form one contiguous row."""
    expected = 1
    for size, stride in zip(reversed(t.shape[lead:]), reversed(t.stride()[lead:])):
        if size != 1 and stride != expected:
            return False
        expected *= size
    return True


class _Planes:
    """A list of same-geometry plane views turned into a ``mak_rows_desc``."""

    def __init__(self, planes: list[torch.Tensor], *, paged: bool):
        self.planes = planes
        self.paged = paged
        first = planes[0]
        e = first.element_size()
        if paged:  # [NB, BS, row...]
            self.rows_per_block = int(first.shape[1])
            self.block_stride = int(first.stride(0)) * e
            self.row_stride = int(first.stride(1)) * e
            self.num_rows = int(first.shape[0]) * int(first.shape[1])
            lead = 2
        else:  # [T, row...]
            self.rows_per_block = 1
            self.block_stride = int(first.stride(0)) * e
            self.row_stride = 0
            self.num_rows = int(first.shape[0])
            lead = 1
        self.row_bytes = _row_elems(first, lead) * e
        self.uniform = all(
            p.shape == first.shape and p.stride() == first.stride() and p.dtype == first.dtype and _rows_contiguous(p, lead)
            for p in planes
        )

    def desc(self):
        return _native.rows_desc([p.data_ptr() for p in self.planes], self.rows_per_block, self.block_stride,
                                 self.row_stride, self.num_rows)


def _check_uniform(op: str, *sides: _Planes) -> None:
    for s in sides:
        if not s.uniform:
            raise ValueError(f"{op}: every cache/buffer plane must share one strided layout with contiguous token rows")


def _gather(op: str, paged: list[torch.Tensor], linear: list[torch.Tensor], slots: torch.Tensor) -> None:
    """paged planes [NB, BS, row] -> linear planes [T_mem, row]; zero rows for skipped / tail tokens."""
    if not paged:
        return
    lib = _native.load()
    p = _Planes(paged, paged=True)
    q = _Planes(linear, paged=False)
    _check_uniform(op, p, q)
    if p.row_bytes != q.row_bytes:
        raise ValueError(f"{op}: cache row and buffer row sizes differ ({p.row_bytes} vs {q.row_bytes} bytes)")
    ks, code = kernel_slots(slots)
    pd, pa = p.desc()
    ld, la = q.desc()
    rc = lib.mak_rows_gather(ctypes.byref(pd), ctypes.byref(ld), None, p.row_bytes, _native.ptr(ks), code, ks.numel(), 1,
                             _native.stream_ptr(paged[0].device))
    _native.check(rc, op)


def _scatter(op: str, linear: list[torch.Tensor], paged: list[torch.Tensor], slots: torch.Tensor, skip_prefix: int) -> None:
    """linear planes row (skip_prefix + t) -> paged planes row slots[t] (last writer wins)."""
    if not paged or slots.numel() == 0:
        return
    lib = _native.load()
    p = _Planes(paged, paged=True)
    q = _Planes(linear, paged=False)
    _check_uniform(op, p, q)
    if p.row_bytes != q.row_bytes:
        raise ValueError(f"{op}: cache row and buffer row sizes differ ({p.row_bytes} vs {q.row_bytes} bytes)")
    ks, code = kernel_slots(slots)
    n = ks.numel()
    dev = paged[0].device
    sp = _native.stream_ptr(dev)
    pd, pa = p.desc()
    ld, la = q.desc()
    skip = int(skip_prefix)
    rc = _native.owned_scatter(dev, sp, int(p.num_rows), n, lambda own, rows, epoch: lib.mak_rows_scatterv_owned(
        ctypes.byref(ld), ctypes.byref(pd), 1, None, p.row_bytes, ks.data_ptr(), code, n, skip, own, rows, epoch, sp))
    if rc is None:
        ws, nbytes = _native.workspace(n, dev)
        rc = lib.mak_rows_scatter(ctypes.byref(ld), ctypes.byref(pd), None, p.row_bytes, ks.data_ptr(), code, n, skip,
                                  ws.data_ptr(), nbytes, sp)
    _native.check(rc, op)


# Fast descriptors: plane pointers computed from a base pointer and strides (or
# read straight off a list of uniform tensors) with no per-plane tensor views.
# Each returns None when the layout needs the general path above.


def _stacked_buffer_side(buf: torch.Tensor, n0: int, n1: int) -> tuple | None:
    """``[n0, n1, T, row]`` buffer -> planes (i0, i1) in i0-major order, token rows of ``row`` elements."""
    if not _rows_contiguous(buf, 3):
        return None
    e = buf.element_size()
    s0, s1, st = buf.stride()[:3]
    base = buf.data_ptr()
    ptrs = [base + (i0 * s0 + i1 * s1) * e for i0 in range(n0) for i1 in range(n1)]
    return ptrs, 1, st * e, 0, int(buf.shape[2])


def _layer_buffer_side(buf: torch.Tensor) -> tuple | None:
    """``[NL, T, row]`` buffer -> one plane per layer."""
    if not _rows_contiguous(buf, 2):
        return None
    e = buf.element_size()
    s0, st = buf.stride()[:2]
    base = buf.data_ptr()
    return [base + i * s0 * e for i in range(buf.shape[0])], 1, st * e, 0, int(buf.shape[1])


def _stacked_cache_side(cache: torch.Tensor, plane_offsets: list[int], nb_dim: int, dtype: torch.dtype) -> tuple | None:
    """Planes at element offsets ``plane_offsets`` of ``cache``; blocks and slots on dims ``nb_dim``, ``nb_dim+1``."""
    if cache.dtype != dtype or not _rows_contiguous(cache, nb_dim + 2):
        return None
    e = cache.element_size()
    base = cache.data_ptr()
    st = cache.stride()
    nb, bs = int(cache.shape[nb_dim]), int(cache.shape[nb_dim + 1])
    return [base + o * e for o in plane_offsets], bs, st[nb_dim] * e, st[nb_dim + 1] * e, nb * bs


def _list_cache_side(caches: list[torch.Tensor], plane_offsets: list[int], nb_dim: int, dtype: torch.dtype) -> tuple | None:
    """Uniform list of caches (same shape, strides and ``dtype``), each giving the planes at ``plane_offsets``."""
    first = caches[0]
    shape, stride = first.shape, first.stride()
    if first.dtype != dtype or not _rows_contiguous(first, nb_dim + 2):
        return None
    e = first.element_size()
    ptrs = []
    for o in plane_offsets:
        for c in caches:
            if c.stride() != stride or c.shape != shape or c.dtype != dtype:
                return None
            ptrs.append(c.data_ptr() + o * e)
    nb, bs = int(shape[nb_dim]), int(shape[nb_dim + 1])
    return ptrs, bs, stride[nb_dim] * e, stride[nb_dim + 1] * e, nb * bs


def _fast_gather(op: str, paged: tuple, linear: tuple, row_bytes: int, slots: torch.Tensor, device) -> None:
    lib = _native.load()
    ks, code = kernel_slots(slots)
    buf = _native.rows_pack(paged, linear)
    base = ctypes.addressof(buf)
    rc = lib.mak_rows_gather(base, base + 48, None, row_bytes, ks.data_ptr(), code, ks.numel(), 1,
                             _native.stream_ptr(device))
    _native.check(rc, op)


def _fast_scatter(op: str, linear: tuple, paged: tuple, row_bytes: int, slots: torch.Tensor, skip_prefix: int,
                  device) -> None:
    if slots.numel() == 0:
        return
    lib = _native.load()
    ks, code = kernel_slots(slots)
    n = ks.numel()
    buf = _native.rows_pack(linear, paged)
    base = ctypes.addressof(buf)
    sp = _native.stream_ptr(device)
    skip = int(skip_prefix)
    rc = _native.owned_scatter(device, sp, paged[4], n, lambda own, rows, epoch: lib.mak_rows_scatterv_owned(
        base, base + 48, 1, None, row_bytes, ks.data_ptr(), code, n, skip, own, rows, epoch, sp))
    if rc is None:
        ws, nbytes = _native.workspace(n, device)
        rc = lib.mak_rows_scatter(base, base + 48, None, row_bytes, ks.data_ptr(), code, n, skip, ws.data_ptr(),
                                  nbytes, sp)
    _native.check(rc, op)


# ---------------------------------------------------------------------------
# contract validation (musa_aiter/ops/lmcache_kv_transfer.py:323-544)
# ---------------------------------------------------------------------------


def _slot_values(slot_mapping: torch.Tensor) -> list[int]:
    return [int(v) for v in slot_mapping.detach().cpu().reshape(-1).tolist()]


def _validate_slots(slot_mapping: torch.Tensor, *, num_tokens: int, num_blocks: int, block_size: int) -> None:
    """lmcache_kv_transfer.py:396-413: rank/length always, range only for host slot tensors."""
    if slot_mapping.dim() != 1:
        raise ValueError("LMCache slot_mapping rank must be 1")
    if int(slot_mapping.numel()) != num_tokens:
        raise ValueError("LMCache slot_mapping length must equal num_tokens")
    if slot_mapping.device.type != "cpu":
        return
    max_slot = num_blocks * block_size
    if slot_mapping.numel():
        top = int(slot_mapping.to(torch.int64).max().item())
        if top >= max_slot:
            raise ValueError(f"LMCache slot_mapping value out of range: slot={top} max={max_slot - 1}")


def _validate_non_mla_contract(kv_buffer: torch.Tensor, paged_kv_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    if kv_buffer.dim() != 4:
        raise ValueError("LMCache non-MLA kv_buffer rank must be 4: [2, NL, T, NH*HS]")
    if paged_kv_cache.dim() != 6:
        raise ValueError("LMCache non-MLA paged_kv_cache rank must be 6: [NL, 2, NB, BS, NH, HS]")
    if int(kv_buffer.shape[0]) != 2 or int(paged_kv_cache.shape[1]) != 2:
        raise ValueError("LMCache non-MLA layout requires K/V axis size 2")
    num_layers, num_tokens, hidden = int(kv_buffer.shape[1]), int(kv_buffer.shape[2]), int(kv_buffer.shape[3])
    cache_layers, _, num_blocks, block_size, num_heads, head_size = map(int, paged_kv_cache.shape)
    if num_layers != cache_layers:
        raise ValueError("LMCache non-MLA layer count mismatch")
    if hidden != num_heads * head_size:
        raise ValueError("LMCache non-MLA hidden size must equal num_heads * head_size")
    _validate_slots(slot_mapping, num_tokens=num_tokens, num_blocks=num_blocks, block_size=block_size)


def _validate_mla_contract(kv_buffer: torch.Tensor, paged_kv_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    if kv_buffer.dim() != 3:
        raise ValueError("LMCache MLA kv_buffer rank must be 3: [NL, T, HS]")
    if paged_kv_cache.dim() != 4:
        raise ValueError("LMCache MLA paged_kv_cache rank must be 4: [NL, NB, BS, HS]")
    num_layers, num_tokens, hidden = map(int, kv_buffer.shape)
    cache_layers, num_blocks, block_size, cache_hidden = map(int, paged_kv_cache.shape)
    if num_layers != cache_layers:
        raise ValueError("LMCache MLA layer count mismatch")
    if hidden != cache_hidden:
        raise ValueError("LMCache MLA hidden size mismatch")
    _validate_slots(slot_mapping, num_tokens=num_tokens, num_blocks=num_blocks, block_size=block_size)


def _contains_nested_cache_list(kvcaches: list[Any]) -> bool:
    return any(isinstance(axis_or_tensor, list) for axis_or_tensor in kvcaches)


def _validate_two_x_nl_contract(memory_tensor, kvcaches, slot_mapping, skip_prefix_n_tokens, block_size, num_heads,
                                head_size) -> tuple | None:
    """Reference checks (lmcache_kv_transfer.py:323-393); returns the caches' row-plane geometry when
    they share one strided layout with contiguous token rows, else None."""
    name = "LMCache TWO_X_NL_X_NB_BS_NH_HS"
    if memory_tensor.dim() != 4 or int(memory_tensor.shape[0]) != 2:
        raise ValueError(f"{name} memory_tensor must be [2, NL, T, NH*HS]")
    if len(kvcaches) != 2 or not all(isinstance(axis, list) for axis in kvcaches):
        raise ValueError(f"{name} cache must be [K_layers, V_layers]")
    if not kvcaches[0] or len(kvcaches[0]) != len(kvcaches[1]):
        raise ValueError(f"{name} K/V layer lists must be non-empty and have equal length")
    num_layers = len(kvcaches[0])
    if int(memory_tensor.shape[1]) != num_layers:
        raise ValueError(f"{name} layer count mismatch")
    if min(block_size, num_heads, head_size) <= 0:
        raise ValueError(f"{name} block_size, num_heads, and head_size must be positive")
    if int(memory_tensor.shape[3]) != num_heads * head_size:
        raise ValueError(f"{name} hidden size must equal num_heads * head_size")
    if memory_tensor.dtype not in (torch.float16, torch.bfloat16, torch.float32):
        raise ValueError(f"{name} supports float16, bfloat16, and float32")
    if slot_mapping.dtype not in (torch.int32, torch.int64):
        raise ValueError(f"{name} slot_mapping must be int32 or int64")
    if skip_prefix_n_tokens < 0:
        raise ValueError(f"{name} skip_prefix_n_tokens must be non-negative")
    if skip_prefix_n_tokens + int(slot_mapping.numel()) > int(memory_tensor.shape[2]):
        raise ValueError(f"{name} transfer range exceeds memory_tensor token extent")
    first = kvcaches[0][0]
    if not isinstance(first, torch.Tensor) or first.dim() != 4:
        raise ValueError(f"{name} each cache tensor must be [NB, BS, NH, HS]")
    num_blocks = int(first.shape[0])
    expected_shape = (num_blocks, block_size, num_heads, head_size)
    if num_blocks <= 0:
        raise ValueError(f"{name} num_blocks must be positive")
    # One pass over the 2*NL caches: the reference's checks in its order, and (as a by-product)
    # the plane pointers when every cache shares one strided layout with contiguous token rows.
    mdt, mdev = memory_tensor.dtype, memory_tensor.get_device()
    stride0 = first.stride()
    uniform = _rows_contiguous(first, 2)
    ptrs = []
    for kv_axis, layers in enumerate(kvcaches):
        for layer, cache in enumerate(layers):
            if not isinstance(cache, torch.Tensor) or cache.shape != expected_shape:
                raise ValueError(f"{name} cache[{kv_axis}][{layer}] must have shape {expected_shape}")
            if cache.dtype != mdt:
                raise ValueError(f"{name} cache dtype must match memory_tensor")
            if cache.get_device() != mdev:
                raise ValueError(f"{name} caches and memory_tensor must share a device")
            if uniform:
                if cache.stride() == stride0:
                    ptrs.append(cache.data_ptr())
                else:
                    uniform = False
    if slot_mapping.get_device() != mdev:
        raise ValueError(f"{name} slot_mapping and data tensors must share a device")
    _validate_slots(slot_mapping, num_tokens=int(slot_mapping.numel()), num_blocks=num_blocks, block_size=block_size)
    if not uniform:
        return None
    e = first.element_size()
    return ptrs, block_size, stride0[0] * e, stride0[1] * e, num_blocks * block_size


def _validate_non_mla_list_contract(memory_tensor, kvcaches, slot_mapping, block_size, num_heads, head_size) -> None:
    if memory_tensor.dim() != 4 or int(memory_tensor.shape[0]) != 2:
        raise ValueError("LMCache list non-MLA memory_tensor rank must be 4: [2, NL, T, NH*HS]")
    if len(kvcaches) != int(memory_tensor.shape[1]):
        raise ValueError("LMCache list non-MLA layer count mismatch")
    if int(memory_tensor.shape[3]) != num_heads * head_size:
        raise ValueError("LMCache list non-MLA hidden size must equal num_heads * head_size")
    if not kvcaches:
        raise ValueError("LMCache list non-MLA kvcaches must not be empty")
    num_blocks = int(kvcaches[0].shape[1])
    for kvcache in kvcaches:
        if (
            kvcache.dim() != 5
            or int(kvcache.shape[0]) != 2
            or int(kvcache.shape[2]) != block_size
            or int(kvcache.shape[3]) != num_heads
            or int(kvcache.shape[4]) != head_size
        ):
            raise ValueError("LMCache list non-MLA kvcache rank must be 5: [2, NB, BS, NH, HS]")
        if int(kvcache.shape[1]) != num_blocks:
            raise ValueError("LMCache list non-MLA num_blocks mismatch")
    _validate_slots(slot_mapping, num_tokens=int(slot_mapping.numel()), num_blocks=num_blocks, block_size=block_size)


def _validate_mla_list_contract(memory_tensor, kvcaches, slot_mapping, block_size, head_size) -> None:
    if memory_tensor.dim() != 4 or int(memory_tensor.shape[0]) != 1:
        raise ValueError("LMCache list MLA memory_tensor rank must be 4: [1, NL, T, HS]")
    if len(kvcaches) != int(memory_tensor.shape[1]):
        raise ValueError("LMCache list MLA layer count mismatch")
    if not kvcaches:
        raise ValueError("LMCache list MLA kvcaches must not be empty")
    num_blocks = int(kvcaches[0].shape[0])
    for kvcache in kvcaches:
        if kvcache.dim() != 3 or int(kvcache.shape[1]) != block_size or int(kvcache.shape[2]) != head_size:
            raise ValueError("LMCache list MLA kvcache rank must be 3: [NB, BS, HS]")
        if int(kvcache.shape[0]) != num_blocks:
            raise ValueError("LMCache list MLA num_blocks mismatch")
    _validate_slots(slot_mapping, num_tokens=int(slot_mapping.numel()), num_blocks=num_blocks, block_size=block_size)


def _check_slot_dtype(slot_mapping: torch.Tensor, what: str) -> None:
    if slot_mapping.dtype not in (torch.int16, torch.int32, torch.int64):
        raise ValueError(f"{what} slot_mapping must be an integer tensor (int16/int32/int64)")


def _check_token_range(memory_tensor: torch.Tensor, slot_mapping: torch.Tensor, skip: int, what: str) -> None:
    if skip < 0:
        raise ValueError(f"{what} skip_prefix_n_tokens must be non-negative")
    if skip + int(slot_mapping.numel()) > int(memory_tensor.shape[-2]):
        raise ValueError(f"{what} transfer range exceeds memory_tensor token extent")


# ---------------------------------------------------------------------------
# public API (musa_aiter/ops/lmcache_kv_transfer.py:51-294)
# ---------------------------------------------------------------------------


def lmcache_kv_buffer_to_paged(
    kv_buffer: torch.Tensor,
    paged_kv_cache: torch.Tensor | list[torch.Tensor] | list[list[torch.Tensor]],
    slot_mapping: torch.Tensor,
    *args: Any,
) -> bool:
    """Scatter an LMCache non-MLA chunk into a paged KV cache.

    Layouts (reference lmcache_kv_transfer.py:51-98): the 6-D tensor
    ``[NL, 2, NB, BS, NH, HS]``; a layer list of ``[2, NB, BS, NH, HS]``; or the
    SGLang MP ``[K_layers, V_layers]`` nested list.  List forms take
    ``skip_prefix_n_tokens, block_size, num_heads, head_size`` positionally.
    """
    if isinstance(paged_kv_cache, list):
        if len(args) != 4:
            raise TypeError("LMCache list-cache buffer_to_paged expects skip_prefix_n_tokens, block_size, num_heads, head_size")
        skip_prefix_n_tokens, block_size, num_heads, head_size = map(int, args)
        if _contains_nested_cache_list(paged_kv_cache):
            return lmcache_kv_buffer_to_paged_two_x_nl(
                kv_buffer, paged_kv_cache, slot_mapping, skip_prefix_n_tokens, block_size, num_heads, head_size
            )
        return _list_buffer_to_paged(kv_buffer, paged_kv_cache, slot_mapping, skip_prefix_n_tokens, block_size, num_heads, head_size)

    _validate_non_mla_contract(kv_buffer, paged_kv_cache, slot_mapping)
    _check_slot_dtype(slot_mapping, "LMCache non-MLA")
    require_cuda("lmcache_kv_buffer_to_paged", kv_buffer, paged_kv_cache, slot_mapping)
    nl = int(kv_buffer.shape[1])
    hidden = int(kv_buffer.shape[3])
    nb, bs = int(paged_kv_cache.shape[2]), int(paged_kv_cache.shape[3])
    if not _rows_contiguous(paged_kv_cache, 4):
        raise ValueError("LMCache non-MLA paged_kv_cache token rows [NH, HS] must be contiguous")
    sl, skv = paged_kv_cache.stride()[:2]
    offsets = [kv * skv + layer * sl for kv in range(2) for layer in range(nl)]
    pside = _stacked_cache_side(paged_kv_cache, offsets, 2, kv_buffer.dtype)
    lside = _stacked_buffer_side(kv_buffer, 2, nl)
    if pside is not None and lside is not None:
        _fast_scatter("lmcache_kv_buffer_to_paged", lside, pside, hidden * kv_buffer.element_size(), slot_mapping, 0,
                      kv_buffer.device)
    else:
        paged = [paged_kv_cache[layer, kv].view(nb, bs, hidden) for kv in range(2) for layer in range(nl)]
        linear = [kv_buffer[kv, layer] for kv in range(2) for layer in range(nl)]
        _scatter("lmcache_kv_buffer_to_paged", linear, paged, slot_mapping, 0)
    emit_native("lmcache_kv_buffer_to_paged", kv_buffer, "sm100a row scatter (6-D cache, all layers)")
    return True


def lmcache_paged_to_kv_buffer(paged_kv_cache: torch.Tensor, kv_buffer: torch.Tensor, slot_mapping: torch.Tensor) -> bool:
    """Gather the 6-D paged cache into ``[2, NL, T, NH*HS]`` (reference lmcache_kv_transfer.py:101-115)."""
    _validate_non_mla_contract(kv_buffer, paged_kv_cache, slot_mapping)
    _check_slot_dtype(slot_mapping, "LMCache non-MLA")
    require_cuda("lmcache_paged_to_kv_buffer", kv_buffer, paged_kv_cache, slot_mapping)
    nl = int(kv_buffer.shape[1])
    hidden = int(kv_buffer.shape[3])
    nb, bs = int(paged_kv_cache.shape[2]), int(paged_kv_cache.shape[3])
    sl, skv = paged_kv_cache.stride()[:2]
    offsets = [kv * skv + layer * sl for kv in range(2) for layer in range(nl)]
    pside = _stacked_cache_side(paged_kv_cache, offsets, 2, kv_buffer.dtype)
    lside = _stacked_buffer_side(kv_buffer, 2, nl)
    if pside is not None and lside is not None:
        _fast_gather("lmcache_paged_to_kv_buffer", pside, lside, hidden * kv_buffer.element_size(), slot_mapping,
                     kv_buffer.device)
    else:
        paged = [paged_kv_cache[layer, kv].reshape(nb, bs, hidden) for kv in range(2) for layer in range(nl)]
        linear = [kv_buffer[kv, layer] for kv in range(2) for layer in range(nl)]
        _gather("lmcache_paged_to_kv_buffer", paged, linear, slot_mapping)
    emit_native("lmcache_paged_to_kv_buffer", kv_buffer, "sm100a row gather (6-D cache, all layers)")
    return True


def lmcache_kv_buffer_to_paged_mla(kv_buffer: torch.Tensor, paged_kv_cache: torch.Tensor, slot_mapping: torch.Tensor) -> bool:
    """``[NL, T, HS]`` -> ``[NL, NB, BS, HS]`` (reference lmcache_kv_transfer.py:118-132)."""
    _validate_mla_contract(kv_buffer, paged_kv_cache, slot_mapping)
    _check_slot_dtype(slot_mapping, "LMCache MLA")
    require_cuda("lmcache_kv_buffer_to_paged_mla", kv_buffer, paged_kv_cache, slot_mapping)
    nl = int(kv_buffer.shape[0])
    pside = _stacked_cache_side(paged_kv_cache, [i * paged_kv_cache.stride(0) for i in range(nl)], 1, kv_buffer.dtype)
    lside = _layer_buffer_side(kv_buffer)
    if pside is not None and lside is not None:
        _fast_scatter("lmcache_kv_buffer_to_paged_mla", lside, pside, int(kv_buffer.shape[2]) * kv_buffer.element_size(),
                      slot_mapping, 0, kv_buffer.device)
    else:
        _scatter("lmcache_kv_buffer_to_paged_mla", [kv_buffer[i] for i in range(nl)],
                 [paged_kv_cache[i] for i in range(nl)], slot_mapping, 0)
    emit_native("lmcache_kv_buffer_to_paged_mla", kv_buffer, "sm100a row scatter (MLA, all layers)")
    return True


def lmcache_paged_to_kv_buffer_mla(paged_kv_cache: torch.Tensor, kv_buffer: torch.Tensor, slot_mapping: torch.Tensor) -> bool:
    """``[NL, NB, BS, HS]`` -> ``[NL, T, HS]`` with zeros for skipped slots (reference :135-151)."""
    _validate_mla_contract(kv_buffer, paged_kv_cache, slot_mapping)
    _check_slot_dtype(slot_mapping, "LMCache MLA")
    require_cuda("lmcache_paged_to_kv_buffer_mla", kv_buffer, paged_kv_cache, slot_mapping)
    nl = int(kv_buffer.shape[0])
    pside = _stacked_cache_side(paged_kv_cache, [i * paged_kv_cache.stride(0) for i in range(nl)], 1, kv_buffer.dtype)
    lside = _layer_buffer_side(kv_buffer)
    if pside is not None and lside is not None:
        _fast_gather("lmcache_paged_to_kv_buffer_mla", pside, lside, int(kv_buffer.shape[2]) * kv_buffer.element_size(),
                     slot_mapping, kv_buffer.device)
    else:
        _gather("lmcache_paged_to_kv_buffer_mla", [paged_kv_cache[i] for i in range(nl)],
                [kv_buffer[i] for i in range(nl)], slot_mapping)
    emit_native("lmcache_paged_to_kv_buffer_mla", kv_buffer, "sm100a row gather (MLA, all layers)")
    return True


def lmcache_kv_paged_to_buffer(
    kvcaches: list[torch.Tensor] | list[list[torch.Tensor]],
    memory_tensor: torch.Tensor,
    slot_mapping: torch.Tensor,
    block_size: int,
    num_heads: int,
    head_size: int,
) -> bool:
    """Gather LMCache list caches (or SGLang MP nested lists) into ``[2, NL, T, NH*HS]``.

    The whole memory tensor is written: token rows past ``len(slot_mapping)``
    and rows of negative slots become zeros (reference lmcache_kv_transfer.py:154-173, 473-490).
    """
    if _contains_nested_cache_list(kvcaches):
        return lmcache_kv_paged_to_buffer_two_x_nl(kvcaches, memory_tensor, slot_mapping, block_size, num_heads, head_size)
    _validate_non_mla_list_contract(memory_tensor, kvcaches, slot_mapping, block_size, num_heads, head_size)
    _check_slot_dtype(slot_mapping, "LMCache list non-MLA")
    require_cuda("lmcache_kv_paged_to_buffer", memory_tensor, slot_mapping, *kvcaches)
    nl = len(kvcaches)
    hidden = num_heads * head_size
    skv = kvcaches[0].stride(0)
    pside = _list_cache_side(kvcaches, [0, skv], 1, memory_tensor.dtype)
    lside = _stacked_buffer_side(memory_tensor, 2, nl)
    if pside is not None and lside is not None:
        _fast_gather("lmcache_kv_paged_to_buffer", pside, lside, hidden * memory_tensor.element_size(), slot_mapping,
                     memory_tensor.device)
    else:
        paged = [kvcaches[layer][kv].view(kvcaches[layer].shape[1], block_size, hidden) if kvcaches[layer][kv].is_contiguous()
                 else kvcaches[layer][kv].reshape(kvcaches[layer].shape[1], block_size, hidden)
                 for kv in range(2) for layer in range(nl)]
        linear = [memory_tensor[kv, layer] for kv in range(2) for layer in range(nl)]
        _gather("lmcache_kv_paged_to_buffer", paged, linear, slot_mapping)
    emit_native("lmcache_kv_paged_to_buffer", memory_tensor, "sm100a row gather (layer list, all layers, one launch)")
    return True


def _list_buffer_to_paged(memory_tensor, kvcaches, slot_mapping, skip_prefix_n_tokens, block_size, num_heads, head_size) -> bool:
    """Layer-list scatter (reference lmcache_kv_transfer.py:451-470)."""
    _validate_non_mla_list_contract(memory_tensor, kvcaches, slot_mapping, block_size, num_heads, head_size)
    _check_slot_dtype(slot_mapping, "LMCache list non-MLA")
    _check_token_range(memory_tensor, slot_mapping, skip_prefix_n_tokens, "LMCache list non-MLA")
    require_cuda("lmcache_kv_buffer_to_paged", memory_tensor, slot_mapping, *kvcaches)
    nl = len(kvcaches)
    hidden = num_heads * head_size
    pside = _list_cache_side(kvcaches, [0, kvcaches[0].stride(0)], 1, memory_tensor.dtype)
    lside = _stacked_buffer_side(memory_tensor, 2, nl)
    if pside is not None and lside is not None:
        _fast_scatter("lmcache_kv_buffer_to_paged", lside, pside, hidden * memory_tensor.element_size(), slot_mapping,
                      skip_prefix_n_tokens, memory_tensor.device)
    else:
        paged = []
        for kv in range(2):
            for layer in range(nl):
                plane = kvcaches[layer][kv]
                if not _rows_contiguous(plane, 2):
                    raise ValueError("LMCache list non-MLA kvcache token rows must be contiguous")
                paged.append(plane.view(plane.shape[0], block_size, hidden))
        linear = [memory_tensor[kv, layer] for kv in range(2) for layer in range(nl)]
        _scatter("lmcache_kv_buffer_to_paged", linear, paged, slot_mapping, skip_prefix_n_tokens)
    emit_native("lmcache_kv_buffer_to_paged", memory_tensor, "sm100a row scatter (layer list, all layers, one launch)")
    return True


def lmcache_kv_buffer_to_paged_two_x_nl(
    memory_tensor: torch.Tensor,
    kvcaches: list[list[torch.Tensor]],
    slot_mapping: torch.Tensor,
    skip_prefix_n_tokens: int,
    block_size: int,
    num_heads: int,
    head_size: int,
) -> bool:
    """Scatter into SGLang MP ``2 x NL x [NB, BS, NH, HS]`` caches, all 2*NL tensors in one launch.

    Reference: lmcache_kv_transfer.py:176-226 (memory token ``skip + t`` goes to ``slot_mapping[t]``).
    """
    pside = _validate_two_x_nl_contract(memory_tensor, kvcaches, slot_mapping, skip_prefix_n_tokens, block_size, num_heads,
                                        head_size)
    require_cuda("lmcache_kv_buffer_to_paged_two_x_nl", memory_tensor, slot_mapping, kvcaches[0][0])
    nl = len(kvcaches[0])
    hidden = num_heads * head_size
    lside = _stacked_buffer_side(memory_tensor, 2, nl)
    if pside is not None and lside is not None:
        _fast_scatter("lmcache_kv_buffer_to_paged_two_x_nl", lside, pside, hidden * memory_tensor.element_size(),
                      slot_mapping, skip_prefix_n_tokens, memory_tensor.device)
    else:
        paged = []
        for kv in range(2):
            for cache in kvcaches[kv]:
                if not _rows_contiguous(cache, 2):
                    raise ValueError("LMCache TWO_X_NL_X_NB_BS_NH_HS cache token rows must be contiguous")
                paged.append(cache.view(cache.shape[0], block_size, hidden))
        linear = [memory_tensor[kv, layer] for kv in range(2) for layer in range(nl)]
        _scatter("lmcache_kv_buffer_to_paged_two_x_nl", linear, paged, slot_mapping, skip_prefix_n_tokens)
    emit_native("lmcache_kv_buffer_to_paged_two_x_nl", memory_tensor, "sm100a row scatter (2 x NL planes, one launch)")
    return True


def lmcache_kv_paged_to_buffer_two_x_nl(
    kvcaches: list[list[torch.Tensor]],
    memory_tensor: torch.Tensor,
    slot_mapping: torch.Tensor,
    block_size: int,
    num_heads: int,
    head_size: int,
) -> bool:
    """Gather SGLang MP caches into ``[2, NL, T, H]`` (whole buffer written; reference :229-269)."""
    pside = _validate_two_x_nl_contract(memory_tensor, kvcaches, slot_mapping, 0, block_size, num_heads, head_size)
    require_cuda("lmcache_kv_paged_to_buffer_two_x_nl", memory_tensor, slot_mapping, kvcaches[0][0])
    nl = len(kvcaches[0])
    hidden = num_heads * head_size
    lside = _stacked_buffer_side(memory_tensor, 2, nl)
    if pside is not None and lside is not None:
        _fast_gather("lmcache_kv_paged_to_buffer_two_x_nl", pside, lside, hidden * memory_tensor.element_size(),
                     slot_mapping, memory_tensor.device)
    else:
        paged = []
        for kv in range(2):
            for cache in kvcaches[kv]:
                paged.append(cache.view(cache.shape[0], block_size, hidden) if _rows_contiguous(cache, 2)
                             else cache.reshape(cache.shape[0], block_size, hidden))
        linear = [memory_tensor[kv, layer] for kv in range(2) for layer in range(nl)]
        _gather("lmcache_kv_paged_to_buffer_two_x_nl", paged, linear, slot_mapping)
    emit_native("lmcache_kv_paged_to_buffer_two_x_nl", memory_tensor, "sm100a row gather (2 x NL planes, one launch)")
    return True


def lmcache_mla_buffer_to_paged(
    memory_tensor: torch.Tensor,
    kvcaches: list[torch.Tensor],
    slot_mapping: torch.Tensor,
    skip_prefix_n_tokens: int,
    block_size: int,
    head_size: int,
) -> bool:
    """``[1, NL, T, HS]`` -> list of ``[NB, BS, HS]`` (reference lmcache_kv_transfer.py:272-282, 473-485)."""
    _validate_mla_list_contract(memory_tensor, kvcaches, slot_mapping, block_size, head_size)
    _check_slot_dtype(slot_mapping, "LMCache list MLA")
    _check_token_range(memory_tensor, slot_mapping, skip_prefix_n_tokens, "LMCache list MLA")
    require_cuda("lmcache_mla_buffer_to_paged", memory_tensor, slot_mapping, *kvcaches)
    for c in kvcaches:
        if not _rows_contiguous(c, 2):
            raise ValueError("LMCache list MLA kvcache token rows must be contiguous")
    pside = _list_cache_side(list(kvcaches), [0], 0, memory_tensor.dtype)
    lside = _stacked_buffer_side(memory_tensor, 1, len(kvcaches))
    if pside is not None and lside is not None:
        _fast_scatter("lmcache_mla_buffer_to_paged", lside, pside, int(memory_tensor.shape[3]) * memory_tensor.element_size(),
                      slot_mapping, skip_prefix_n_tokens, memory_tensor.device)
    else:
        _scatter("lmcache_mla_buffer_to_paged", [memory_tensor[0, i] for i in range(len(kvcaches))], list(kvcaches),
                 slot_mapping, skip_prefix_n_tokens)
    emit_native("lmcache_mla_buffer_to_paged", memory_tensor, "sm100a row scatter (MLA list, one launch)")
    return True


def lmcache_mla_paged_to_buffer(
    kvcaches: list[torch.Tensor],
    memory_tensor: torch.Tensor,
    slot_mapping: torch.Tensor,
    block_size: int,
    head_size: int,
) -> bool:
    """List of ``[NB, BS, HS]`` -> ``[1, NL, T, HS]`` (whole buffer written; reference :285-294, 488-502)."""
    _validate_mla_list_contract(memory_tensor, kvcaches, slot_mapping, block_size, head_size)
    _check_slot_dtype(slot_mapping, "LMCache list MLA")
    require_cuda("lmcache_mla_paged_to_buffer", memory_tensor, slot_mapping, *kvcaches)
    pside = _list_cache_side(list(kvcaches), [0], 0, memory_tensor.dtype)
    lside = _stacked_buffer_side(memory_tensor, 1, len(kvcaches))
    if pside is not None and lside is not None:
        _fast_gather("lmcache_mla_paged_to_buffer", pside, lside, int(memory_tensor.shape[3]) * memory_tensor.element_size(),
                     slot_mapping, memory_tensor.device)
    else:
        _gather("lmcache_mla_paged_to_buffer", list(kvcaches), [memory_tensor[0, i] for i in range(len(kvcaches))],
                slot_mapping)
    emit_native("lmcache_mla_paged_to_buffer", memory_tensor, "sm100a row gather (MLA list, one launch)")
    return True


def lmcache_kv_strided_block_transfer(
    staging: "torch.Tensor | int",
    paged_ptrs: list[int],
    block_ids: torch.Tensor,
    direction: int,
    num_layers: int,
    idx_start: int,
    n_valid: int,
    offset_in_object: int,
    staging_tokens: int,
    block_size: int,
    row_bytes: int,
    paged_block_stride: int,
    mode: int,
    value_bytes: int = 0,
    scale_bytes: int = 0,
) -> bool:
    """Staging ``[NL, staging_tokens, row_bytes]`` <-> padded paged pages, all layers in one launch.

    Reference contract (lmcache_kv_transfer.py:1294-1403): mode 0 plain rows,
    mode 1 per-block values-then-scales; direction 0 staging -> paged, 1 back.
    Invalid arguments return False (the caller picks another path) instead of
    raising; ``block_ids`` must be a contiguous CUDA int64 tensor and
    ``paged_ptrs`` a host list of per-layer page base addresses.  In mode 1
    ``value_bytes + scale_bytes`` must equal ``row_bytes``.
    """
    if num_layers <= 0 or n_valid <= 0 or block_size <= 0 or staging_tokens <= 0:
        return False
    if row_bytes <= 0 or row_bytes % 4 != 0 or mode not in (0, 1) or int(direction) not in (0, 1):
        return False
    if mode == 1 and (value_bytes <= 0 or scale_bytes <= 0 or value_bytes % 4 or scale_bytes % 4
                      or value_bytes + scale_bytes != row_bytes):
        return False
    if not isinstance(paged_ptrs, (list, tuple)) or len(paged_ptrs) != num_layers:
        return False
    if not isinstance(block_ids, torch.Tensor) or block_ids.dtype is not torch.int64 or block_ids.device.type != "cuda" \
            or not block_ids.is_contiguous():
        return False
    if idx_start < 0 or idx_start + n_valid > int(block_ids.numel()):
        return False
    staging_ptr = int(staging.data_ptr()) if isinstance(staging, torch.Tensor) else int(staging)
    if staging_ptr <= 0:
        return False
    lib = _native.load()
    arr = (ctypes.c_uint64 * num_layers)(*map(int, paged_ptrs))
    with torch.cuda.device(block_ids.device):
        rc = lib.mak_lmcache_strided_block_transfer(
            ctypes.c_void_p(staging_ptr), arr, _native.ptr(block_ids), int(direction), int(num_layers), int(idx_start),
            int(n_valid), int(offset_in_object), int(staging_tokens), int(block_size), int(row_bytes),
            int(paged_block_stride), int(mode), int(value_bytes), int(scale_bytes), _native.stream_ptr(block_ids.device),
        )
    if rc != 0:
        return False
    emit_native("lmcache_kv_strided_block_transfer", block_ids, f"sm100a strided block transfer mode={mode} dir={direction}")
    return True
