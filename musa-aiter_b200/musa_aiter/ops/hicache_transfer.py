"""SGLang HiCache layout transfers on B200.

Same public functions, two-index-table model and checks as the reference
(musa_aiter/ops/hicache_transfer.py): tensors are ``layer_first``
``[layers, pages, item]`` or ``page_first`` ``[pages, layers, item]``; page
index -1 skips an entry.  Every (kv, layer) plane of a call moves in one
row-engine launch (``mak_rows_copy``), with either side allowed to be pinned
host memory (the HiCache host pool), which the kernel addresses directly.
"""

from __future__ import annotations

import ctypes
from typing import Literal

import torch

from .. import _build, _native
from ..dispatch import emit_native
from ._common import kernel_slots, validation_enabled

LayoutName = Literal["layer_first", "page_first"]
_ABI_VERSION = 1


def build_native_hicache_transfer():
    return _build.build()


def native_hicache_transfer_abi_version() -> int | None:
    return _ABI_VERSION if _native.is_available() else None


def is_native_hicache_transfer_available() -> bool:
    return _native.is_available()


def _layout_geometry(tensor: torch.Tensor, layout: LayoutName) -> tuple[int, int, int, int, int]:
    """(layers, pages, item_elements, page_stride_bytes, layer_stride_bytes); reference :97-117."""
    if not isinstance(tensor, torch.Tensor) or tensor.dim() != 3:
        raise ValueError("HiCache tensors must be rank-3 [layers/pages/item] or [pages/layers/item]")
    if not tensor.is_contiguous():
        raise ValueError("HiCache tensors must be contiguous")
    e = tensor.element_size()
    if layout == "layer_first":
        layers, pages, item = map(int, tensor.shape)
        page_stride = item * e
        layer_stride = pages * page_stride
    elif layout == "page_first":
        pages, layers, item = map(int, tensor.shape)
        layer_stride = item * e
        page_stride = layers * layer_stride
    else:
        raise ValueError(f"unsupported HiCache layout={layout!r}")
    if layers <= 0 or pages <= 0 or item <= 0:
        raise ValueError("HiCache layer/page/item dimensions must be positive")
    return layers, pages, item, page_stride, layer_stride


def _validate_inputs(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, src_layout, dst_layout, start_layer,
                     num_layers, *, mla: bool):
    if not isinstance(src_indices, torch.Tensor) or not isinstance(dst_indices, torch.Tensor):
        raise TypeError("HiCache index tables must be torch.Tensor values")
    if src_indices.dim() != 1 or dst_indices.dim() != 1:
        raise ValueError("HiCache index tables must be 1-D")
    if src_indices.numel() != dst_indices.numel():
        raise ValueError("source and destination index tables must have the same length")
    if src_indices.dtype not in (torch.int32, torch.int64) or dst_indices.dtype not in (torch.int32, torch.int64):
        raise ValueError("HiCache index tables must use int32 or int64")
    if src_k.dtype != dst_k.dtype:
        raise ValueError("source and destination K tensors must have the same dtype")
    if src_v is not None or dst_v is not None:
        if mla:
            raise ValueError("MLA HiCache transfer does not accept a value plane")
        if src_v is None or dst_v is None:
            raise ValueError("source and destination value tensors must be provided together")
        if src_v.dtype != src_k.dtype or dst_v.dtype != dst_k.dtype:
            raise ValueError("K and V tensors must use the same dtype")
        if src_v.device != src_k.device or dst_v.device != dst_k.device:
            raise ValueError("K and V tensors must be on the same device")
    elif not mla:
        raise ValueError("non-MLA HiCache transfer requires K and V tensors")
    sg = _layout_geometry(src_k, src_layout)
    dg = _layout_geometry(dst_k, dst_layout)
    if sg[2] * src_k.element_size() != dg[2] * dst_k.element_size():
        raise ValueError("source and destination item byte sizes must match")
    if src_v is not None and _layout_geometry(src_v, src_layout) != sg:
        raise ValueError("source K and V layouts must match")
    if dst_v is not None and _layout_geometry(dst_v, dst_layout) != dg:
        raise ValueError("destination K and V layouts must match")
    if start_layer < 0 or num_layers <= 0:
        raise ValueError("start_layer and num_layers must be non-negative/positive")
    if start_layer + num_layers > min(sg[0], dg[0]):
        raise ValueError("requested layer range exceeds source or destination")
    item_bytes = sg[2] * src_k.element_size()
    if item_bytes % 8 != 0:
        raise ValueError("HiCache item byte size must be divisible by 8")
    return sg, dg, item_bytes


def _validate_page_indices(src_indices, dst_indices, src_pages: int, dst_pages: int) -> None:
    """Reference :171-184: entries must be -1 or in range (read back to the host).

    With device index tables and ``MUSA_AITER_SKIP_VALIDATION=1`` the read-back, which waits for
    the stream on every call, is skipped: the row kernel skips rows whose page index is negative
    or out of range on either side."""
    if src_indices.device.type == "cuda" and dst_indices.device.type == "cuda" and not validation_enabled():
        return
    s = src_indices.to(device="cpu", dtype=torch.long)
    d = dst_indices.to(device="cpu", dtype=torch.long)
    if s.numel() == 0:
        return
    if bool((s < -1).any()) or bool((d < -1).any()):
        raise ValueError("HiCache page indices must be -1 or non-negative")
    if bool((s >= src_pages).any()) or bool((d >= dst_pages).any()):
        raise ValueError("HiCache page index is out of range")


def _device_of(*tensors: torch.Tensor) -> torch.device:
    for t in tensors:
        if t is not None and t.device.type == "cuda":
            return t.device
    raise RuntimeError("HiCache transfer: the B200 backend needs a CUDA tensor on one side (no CPU fallback)")


def _check_addressable(*tensors) -> None:
    for t in tensors:
        if t is None:
            continue
        if t.device.type == "cpu" and not t.is_pinned():
            raise RuntimeError("HiCache transfer: host tensors must be pinned so the GPU can address them")


def _transfer(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, *, src_layout: LayoutName, dst_layout: LayoutName,
              start_layer: int, num_layers: int, mla: bool) -> bool:
    sg, dg, item_bytes = _validate_inputs(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, src_layout, dst_layout,
                                          start_layer, num_layers, mla=mla)
    _validate_page_indices(src_indices, dst_indices, sg[1], dg[1])
    dev = _device_of(src_k, dst_k)
    _check_addressable(src_k, dst_k, src_v, dst_v)
    n = int(src_indices.numel())
    if n == 0:
        return True
    layers = range(start_layer, start_layer + num_layers)
    src_planes = [src_k.data_ptr() + l * sg[4] for l in layers]
    dst_planes = [dst_k.data_ptr() + l * dg[4] for l in layers]
    if src_v is not None:
        src_planes += [src_v.data_ptr() + l * sg[4] for l in layers]
        dst_planes += [dst_v.data_ptr() + l * dg[4] for l in layers]
    si, sc = kernel_slots(src_indices.to(dev))
    di, dc = kernel_slots(dst_indices.to(dev))
    sd, sa = _native.rows_desc(src_planes, 1, sg[3], 0, sg[1])
    dd, da = _native.rows_desc(dst_planes, 1, dg[3], 0, dg[1])
    rc = _native.rows_copy(ctypes.byref(sd), ctypes.byref(dd), item_bytes, _native.ptr(si), sc, _native.ptr(di), dc, n,
                           int(dg[1]), dev, _native.stream_ptr(dev))
    _native.check(rc, "hicache_transfer")
    emit_native("hicache_transfer", src_k, f"sm100a row engine {src_layout}->{dst_layout}, {len(src_planes)} planes, one launch")
    return True


def hicache_transfer_kv_per_layer(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, *, layer_id: int = 0) -> bool:
    return _transfer(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, src_layout="layer_first",
                     dst_layout="layer_first", start_layer=layer_id, num_layers=1, mla=False)


def hicache_transfer_kv_per_layer_pf_lf(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, *, layer_id: int = 0) -> bool:
    return _transfer(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, src_layout="page_first",
                     dst_layout="layer_first", start_layer=layer_id, num_layers=1, mla=False)


def hicache_transfer_kv_all_layer(src_k, dst_k, src_v, dst_v, src_indices, dst_indices) -> bool:
    return _transfer(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, src_layout="layer_first",
                     dst_layout="layer_first", start_layer=0, num_layers=int(src_k.shape[0]), mla=False)


def hicache_transfer_kv_all_layer_lf_pf(src_k, dst_k, src_v, dst_v, src_indices, dst_indices) -> bool:
    return _transfer(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, src_layout="layer_first",
                     dst_layout="page_first", start_layer=0, num_layers=int(src_k.shape[0]), mla=False)


def hicache_transfer_kv_per_layer_mla(src, dst, src_indices, dst_indices, *, layer_id: int = 0, value=None) -> bool:
    if value is not None:
        raise ValueError("MLA HiCache transfer does not accept a value plane")
    return _transfer(src, dst, None, None, src_indices, dst_indices, src_layout="layer_first", dst_layout="layer_first",
                     start_layer=layer_id, num_layers=1, mla=True)


def hicache_transfer_kv_per_layer_mla_pf_lf(src, dst, src_indices, dst_indices, *, layer_id: int = 0) -> bool:
    return _transfer(src, dst, None, None, src_indices, dst_indices, src_layout="page_first", dst_layout="layer_first",
                     start_layer=layer_id, num_layers=1, mla=True)


def hicache_transfer_kv_all_layer_mla(src, dst, src_indices, dst_indices) -> bool:
    return _transfer(src, dst, None, None, src_indices, dst_indices, src_layout="layer_first", dst_layout="layer_first",
                     start_layer=0, num_layers=int(src.shape[0]), mla=True)


def hicache_transfer_kv_all_layer_mla_lf_pf(src, dst, src_indices, dst_indices) -> bool:
    """All MLA layers from layer-first to page-first storage."""
    return _transfer(src, dst, None, None, src_indices, dst_indices, src_layout="layer_first", dst_layout="page_first",
                     start_layer=0, num_layers=int(src.shape[0]), mla=True)


# ---------------------------------------------------------------------------
# "direct" page-range variants (reference :480-679)
# ---------------------------------------------------------------------------


def _validate_direct_indices(src_indices, dst_indices, page_size: int) -> tuple[torch.Tensor, torch.Tensor]:
    if not isinstance(src_indices, torch.Tensor) or not isinstance(dst_indices, torch.Tensor):
        raise TypeError("HiCache direct index tables must be torch.Tensor values")
    if src_indices.dim() != 1 or dst_indices.dim() != 1:
        raise ValueError("HiCache direct index tables must be 1-D")
    if src_indices.numel() != dst_indices.numel():
        raise ValueError("source and destination index tables must have the same length")
    if src_indices.dtype not in (torch.int32, torch.int64) or dst_indices.dtype not in (torch.int32, torch.int64):
        raise ValueError("HiCache direct index tables must use int32 or int64")
    if page_size <= 0:
        raise ValueError("HiCache direct page_size must be positive")
    if src_indices.numel() % page_size != 0:
        raise ValueError("HiCache direct index count must be divisible by page_size")
    s = src_indices.detach().to(device="cpu", dtype=torch.long)
    d = dst_indices.detach().to(device="cpu", dtype=torch.long)
    if bool((s < 0).any()) or bool((d < 0).any()):
        raise ValueError("HiCache direct indices must be non-negative")
    return s, d


def _page_rows(values: torch.Tensor, page_size: int) -> torch.Tensor:
    """Each page of ``page_size`` entries copies from its first entry onward (reference run semantics)."""
    n = int(values.numel())
    starts = values.view(-1, page_size)[:, :1]
    return (starts + torch.arange(page_size)).reshape(n)


def _direct_copy(src_planes, dst_planes, s_geo, d_geo, src_rows, dst_rows, item_bytes, dev, name):
    n = int(src_rows.numel())
    si = src_rows.to(dev)
    di = dst_rows.to(dev)
    sd, sa = _native.rows_desc(src_planes, *s_geo)
    dd, da = _native.rows_desc(dst_planes, *d_geo)
    rc = _native.rows_copy(ctypes.byref(sd), ctypes.byref(dd), item_bytes, _native.ptr(si), _native.MAK_DT_I64,
                           _native.ptr(di), _native.MAK_DT_I64, n, int(d_geo[3]), dev, _native.stream_ptr(dev))
    _native.check(rc, name)


def hicache_transfer_kv_direct(src_layers, dst_layers, src_indices, dst_indices, page_size: int) -> bool:
    """Token-range copies ``dst[l][d + j] = src[l][s + j]`` per page (reference :569-580)."""
    if not isinstance(src_layers, (list, tuple)) or not isinstance(dst_layers, (list, tuple)):
        raise TypeError("HiCache direct layers must be tensor lists")
    if not src_layers or len(src_layers) != len(dst_layers):
        raise ValueError("HiCache direct source and destination lists must have equal non-zero length")
    for s, d in zip(src_layers, dst_layers):
        if not isinstance(s, torch.Tensor) or not isinstance(d, torch.Tensor):
            raise TypeError("HiCache direct layer entries must be tensors")
        if s.dim() < 1 or d.dim() < 1:
            raise ValueError("HiCache direct tensors must have at least one dimension")
        if tuple(s.shape[1:]) != tuple(d.shape[1:]):
            raise ValueError("HiCache direct source and destination tails must match")
        if s.dtype != d.dtype:
            raise ValueError("HiCache direct source and destination dtypes must match")
        if not s.is_contiguous() or not d.is_contiguous():
            raise ValueError("HiCache direct tensors must be contiguous")
    sv, dv = _validate_direct_indices(src_indices, dst_indices, int(page_size))
    srows, drows = _page_rows(sv, int(page_size)), _page_rows(dv, int(page_size))
    if srows.numel():
        if int(srows.max()) >= min(int(t.shape[0]) for t in src_layers) or int(drows.max()) >= min(int(t.shape[0]) for t in dst_layers):
            raise ValueError("HiCache direct token range exceeds source or destination")
        dev = _device_of(*src_layers, *dst_layers)
        _check_addressable(*src_layers, *dst_layers)
        s0, d0 = src_layers[0], dst_layers[0]
        item = s0[0].numel() * s0.element_size() if s0.dim() > 1 else s0.element_size()
        if any(t.shape[0] != s0.shape[0] for t in src_layers) or any(t.shape[0] != d0.shape[0] for t in dst_layers):
            for s, d in zip(src_layers, dst_layers):
                _direct_copy([s.data_ptr()], [d.data_ptr()], (1, item, 0, int(s.shape[0])), (1, item, 0, int(d.shape[0])),
                             srows, drows, item, dev, "hicache_transfer_kv_direct")
        else:
            _direct_copy([t.data_ptr() for t in src_layers], [t.data_ptr() for t in dst_layers],
                         (1, item, 0, int(s0.shape[0])), (1, item, 0, int(d0.shape[0])), srows, drows, item, dev,
                         "hicache_transfer_kv_direct")
    emit_native("hicache_transfer_direct", dst_layers[0], "sm100a row engine direct page ranges")
    return True


def hicache_transfer_kv_per_layer_direct_pf_lf(src_ptrs, dst_ptrs, src_indices, dst_indices, layer_id: int, page_size: int) -> bool:
    """Page-first ``[pages, layers, page, item]`` source pages -> one layer-first ``[tokens, item]`` layer."""
    if layer_id < 0:
        raise ValueError("HiCache direct layer_id must be non-negative")
    if len(src_ptrs) not in (1, 2) or len(dst_ptrs) != len(src_ptrs):
        raise ValueError("HiCache per-layer direct expects one MLA plane or K/V plane pairs")
    sv, dv = _validate_direct_indices(src_indices, dst_indices, int(page_size))
    P = int(page_size)
    for s, d in zip(src_ptrs, dst_ptrs):
        if s.dim() != 4 or d.dim() != 2:
            raise ValueError("HiCache per-layer direct expects source [pages,layers,page,item] and destination [tokens,item]")
        if layer_id >= int(s.shape[1]):
            raise ValueError("HiCache direct layer_id exceeds source layers")
        if not s.is_contiguous() or not d.is_contiguous():
            raise ValueError("HiCache direct tensors must be contiguous")
        if s.dtype != d.dtype or tuple(s.shape[3:]) != tuple(d.shape[1:]):
            raise ValueError("HiCache direct source and destination item shapes/dtypes must match")
    starts_s = sv.view(-1, P)[:, 0]
    starts_d = dv.view(-1, P)[:, 0]
    src_page = starts_s // P
    s0 = src_ptrs[0]
    if starts_s.numel() and (int(src_page.max()) >= int(s0.shape[0]) or int((starts_d + P).max()) > int(dst_ptrs[0].shape[0])):
        raise ValueError("HiCache direct page range exceeds source or destination")
    if starts_s.numel():
        dev = _device_of(*src_ptrs, *dst_ptrs)
        _check_addressable(*src_ptrs, *dst_ptrs)
        e = s0.element_size()
        item = int(s0.shape[3]) * e
        srows = (src_page.unsqueeze(1) * P + torch.arange(P)).reshape(-1)
        drows = (starts_d.unsqueeze(1) + torch.arange(P)).reshape(-1)
        planes_s = [t.data_ptr() + layer_id * t.stride(1) * e for t in src_ptrs]
        planes_d = [t.data_ptr() for t in dst_ptrs]
        _direct_copy(planes_s, planes_d, (P, s0.stride(0) * e, s0.stride(2) * e, int(s0.shape[0]) * P),
                     (1, item, 0, int(dst_ptrs[0].shape[0])), srows, drows, item, dev,
                     "hicache_transfer_kv_per_layer_direct_pf_lf")
    emit_native("hicache_transfer_per_layer_direct_pf_lf", dst_ptrs[0], "sm100a row engine direct pages")
    return True


def hicache_transfer_kv_all_layer_direct_lf_pf(src_ptrs, dst_ptrs, src_indices, dst_indices, page_size: int) -> bool:
    """Layer-first ``[tokens, item]`` per-layer sources -> all-layer page-first ``[pages, layers, page, item]``."""
    if len(dst_ptrs) not in (1, 2):
        raise ValueError("HiCache all-layer direct expects one MLA plane or K/V plane pairs")
    is_mla = len(dst_ptrs) == 1
    if len(src_ptrs) == 0 or (not is_mla and len(src_ptrs) % 2 != 0):
        raise ValueError("HiCache all-layer direct source planes do not match destination planes")
    nl = len(src_ptrs) if is_mla else len(src_ptrs) // 2
    _validate_direct_indices(src_indices, dst_indices, int(page_size))
    if not all(isinstance(t, torch.Tensor) for t in list(src_ptrs) + list(dst_ptrs)):
        raise TypeError("HiCache direct layer entries must be tensors")
    for t in src_ptrs:
        if t.dim() != 2 or not t.is_contiguous():
            raise ValueError("HiCache all-layer direct sources must be contiguous [tokens,item] tensors")
    for t in dst_ptrs:
        if t.dim() != 4 or not t.is_contiguous():
            raise ValueError("HiCache all-layer direct destinations must be contiguous [pages,layers,page,item] tensors")
    for i in range(nl):
        if src_ptrs[i].dtype != dst_ptrs[0].dtype or tuple(src_ptrs[i].shape[1:]) != tuple(dst_ptrs[0].shape[3:]):
            raise ValueError("HiCache direct source and destination item shapes/dtypes must match")
    if not is_mla and (src_ptrs[nl].dtype != dst_ptrs[1].dtype or tuple(src_ptrs[nl].shape[1:]) != tuple(dst_ptrs[1].shape[3:])):
        raise ValueError("HiCache direct K/V item shapes/dtypes must match")
    sv, dv = _validate_direct_indices(src_indices, dst_indices, int(page_size))
    P = int(page_size)
    starts_s = sv.view(-1, P)[:, 0]
    dst_page = dv.view(-1, P)[:, 0] // P
    if starts_s.numel():
        if int(dst_page.max()) >= int(dst_ptrs[0].shape[0]):
            raise ValueError("HiCache direct destination page exceeds destination")
        if int((starts_s + P).max()) > min(int(t.shape[0]) for t in src_ptrs):
            raise ValueError("HiCache direct source range exceeds source")
        dev = _device_of(*src_ptrs, *dst_ptrs)
        _check_addressable(*src_ptrs, *dst_ptrs)
        d0 = dst_ptrs[0]
        e = d0.element_size()
        item = int(d0.shape[3]) * e
        srows = (starts_s.unsqueeze(1) + torch.arange(P)).reshape(-1)
        drows = (dst_page.unsqueeze(1) * P + torch.arange(P)).reshape(-1)
        planes_s = [t.data_ptr() for t in src_ptrs]
        planes_d = [d0.data_ptr() + l * d0.stride(1) * e for l in range(nl)]
        if not is_mla:
            d1 = dst_ptrs[1]
            planes_d += [d1.data_ptr() + l * d1.stride(1) * e for l in range(nl)]
        s_rows = min(int(t.shape[0]) for t in src_ptrs)
        _direct_copy(planes_s, planes_d, (1, item, 0, s_rows), (P, d0.stride(0) * e, d0.stride(2) * e, int(d0.shape[0]) * P),
                     srows, drows, item, dev, "hicache_transfer_kv_all_layer_direct_lf_pf")
    emit_native("hicache_transfer_all_layer_direct_lf_pf", dst_ptrs[0], "sm100a row engine direct pages")
    return True
