"""ctypes boundary to ``libmak_kvcache.so`` (the sm_100a kernel library).

The reference loads its JIT-built MUSA library with ctypes and assigns
``argtypes`` on every call (musa_aiter/ops/kv_transfer.py:4193-4206 notes the
~17 us cost).  Here the library is loaded once per process, every prototype
is bound once at load time, and calls go straight through.

There is no fallback: if the library is missing or a call fails, a
``RuntimeError`` carrying the library's own message is raised.
"""

from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, c_int32, c_int64, c_size_t, c_uint64, c_void_p

import torch

from . import _build

ABI_VERSION = 1

MAK_DT_U8, MAK_DT_F16, MAK_DT_BF16, MAK_DT_F32, MAK_DT_I32, MAK_DT_I64 = range(6)
MAK_FP8_E4M3, MAK_FP8_E5M2 = 1, 2
MAK_SCALE_SCALAR, MAK_SCALE_PER_HEAD, MAK_SCALE_PER_LAYER_HEAD = 0, 1, 2
MAK_COPY_AUTO, MAK_COPY_ENGINE, MAK_COPY_KERNEL = 0, 1, 2

_DTYPE_CODES = {
    torch.uint8: MAK_DT_U8,
    torch.float16: MAK_DT_F16,
    torch.bfloat16: MAK_DT_BF16,
    torch.float32: MAK_DT_F32,
    torch.int32: MAK_DT_I32,
    torch.int64: MAK_DT_I64,
}
for _name in ("float8_e4m3fn", "float8_e5m2"):
    if hasattr(torch, _name):
        _DTYPE_CODES[getattr(torch, _name)] = MAK_DT_U8


class PagedDesc(ctypes.Structure):
    """``mak_paged_desc``: block-size-innermost cache ``[L][NB][NH][HD][BS]``."""

    _fields_ = [
        ("k", c_void_p),
        ("v", c_void_p),
        ("num_layers", c_int64),
        ("num_blocks", c_int64),
        ("num_heads", c_int64),
        ("head_dim", c_int64),
        ("block_size", c_int64),
        ("stride_layer", c_int64),
        ("stride_block", c_int64),
        ("stride_head", c_int64),
        ("stride_dim", c_int64),
        ("dtype", c_int32),
        ("reserved", c_int32),
    ]


class LinearDesc(ctypes.Structure):
    """``mak_linear_desc``: token-major ``[L][T][NH][HD]`` buffers."""

    _fields_ = [
        ("k", c_void_p),
        ("v", c_void_p),
        ("num_tokens", c_int64),
        ("stride_layer", c_int64),
        ("stride_token", c_int64),
        ("stride_head", c_int64),
        ("dtype", c_int32),
        ("reserved", c_int32),
    ]


class MlaLinearDesc(ctypes.Structure):
    """``mak_mla_linear_desc``: MLA latent ``[L][T][kv_dim]`` + rope ``[L][T][pe_dim]`` rows."""

    _fields_ = [
        ("kv", c_void_p),
        ("pe", c_void_p),
        ("num_layers", c_int64),
        ("num_tokens", c_int64),
        ("kv_dim", c_int64),
        ("pe_dim", c_int64),
        ("kv_stride_layer", c_int64),
        ("kv_stride_token", c_int64),
        ("pe_stride_layer", c_int64),
        ("pe_stride_token", c_int64),
        ("dtype", c_int32),
        ("reserved", c_int32),
    ]


class CopyEntry(ctypes.Structure):
    """``mak_copy_entry``: one byte copy of a batch."""

    _fields_ = [("dst", c_uint64), ("src", c_uint64), ("size", c_uint64)]


class RowsDesc(ctypes.Structure):
    """``mak_rows_desc``: planes of rows (strides in bytes)."""

    _fields_ = [
        ("plane_ptrs", POINTER(c_uint64)),
        ("num_planes", c_int64),
        ("rows_per_block", c_int64),
        ("block_stride", c_int64),
        ("row_stride", c_int64),
        ("num_rows", c_int64),
    ]


_PROTOTYPES = {
    "mak_abi_version": (c_int32, []),
    "mak_last_error": (ctypes.c_char_p, []),
    "mak_device_sm_count": (c_int32, []),
    "mak_launch_count": (c_uint64, []),
    "mak_slot_max": (c_int32, [c_void_p, c_int32, c_int64, c_void_p, c_void_p]),
    "mak_scatter_workspace_bytes": (c_size_t, [c_int64]),
    "mak_resolve_last_writer": (c_int32, [c_void_p, c_int32, c_int64, c_void_p, c_void_p, c_size_t, c_void_p]),
    "mak_build_slot_mapping": (
        c_int32,
        [c_void_p, c_int32, c_int64, c_void_p, c_int32, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    ),
    "mak_kv_paged_to_linear": (c_int32, [POINTER(PagedDesc), POINTER(LinearDesc), c_void_p, c_int32, c_int32, c_void_p]),
    "mak_kv_linear_to_paged": (
        c_int32,
        [POINTER(LinearDesc), POINTER(PagedDesc), c_void_p, c_int32, c_void_p, c_size_t, c_void_p],
    ),
    "mak_kv_paged_fp8_to_linear": (
        c_int32,
        [POINTER(PagedDesc), POINTER(LinearDesc), c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p],
    ),
    "mak_kv_linear_to_paged_fp8": (
        c_int32,
        [
            POINTER(LinearDesc),
            POINTER(PagedDesc),
            c_void_p,
            c_int32,
            c_void_p,
            c_void_p,
            c_int32,
            c_int32,
            c_void_p,
            c_size_t,
            c_void_p,
        ],
    ),
    "mak_kv_paged_to_linear_mapped": (
        c_int32,
        [POINTER(PagedDesc), POINTER(LinearDesc), c_void_p, c_int32, c_int32, c_void_p, c_int64, ctypes.c_uint32,
         c_void_p],
    ),
    "mak_kv_linear_to_paged_mapped": (
        c_int32,
        [POINTER(LinearDesc), POINTER(PagedDesc), c_void_p, c_int32, c_void_p, c_size_t, c_void_p, c_int64,
         ctypes.c_uint32, c_void_p],
    ),
    "mak_kv_paged_fp8_to_linear_mapped": (
        c_int32,
        [POINTER(PagedDesc), POINTER(LinearDesc), c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p,
         c_int64, ctypes.c_uint32, c_void_p],
    ),
    "mak_kv_linear_to_paged_fp8_mapped": (
        c_int32,
        [POINTER(LinearDesc), POINTER(PagedDesc), c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p,
         c_size_t, c_void_p, c_int64, ctypes.c_uint32, c_void_p],
    ),
    "mak_kv_linear_to_paged_owned": (
        c_int32,
        [POINTER(LinearDesc), POINTER(PagedDesc), c_void_p, c_int32, c_void_p, c_int64, ctypes.c_uint32, c_void_p,
         c_int64, ctypes.c_uint32, c_void_p],
    ),
    "mak_kv_linear_to_paged_fp8_owned": (
        c_int32,
        [POINTER(LinearDesc), POINTER(PagedDesc), c_void_p, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p,
         c_int64, ctypes.c_uint32, c_void_p, c_int64, ctypes.c_uint32, c_void_p],
    ),
    "mak_rows_gather": (
        c_int32,
        [c_void_p, c_void_p, POINTER(c_int64), c_int64, c_void_p, c_int32, c_int64, c_int32, c_void_p],
    ),
    "mak_rows_scatter": (
        c_int32,
        [
            c_void_p,
            c_void_p,
            POINTER(c_int64),
            c_int64,
            c_void_p,
            c_int32,
            c_int64,
            c_int64,
            c_void_p,
            c_size_t,
            c_void_p,
        ],
    ),
    "mak_rows_gatherv": (
        c_int32,
        [c_void_p, c_void_p, c_int32, POINTER(c_int64), c_int64, c_void_p, c_int32, c_int64, c_int32,
         c_void_p],
    ),
    "mak_rows_scatterv": (
        c_int32,
        [c_void_p, c_void_p, c_int32, POINTER(c_int64), c_int64, c_void_p, c_int32, c_int64, c_int64,
         c_void_p, c_size_t, c_void_p],
    ),
    "mak_rows_scatterv_owned": (
        c_int32,
        [c_void_p, c_void_p, c_int32, POINTER(c_int64), c_int64, c_void_p, c_int32, c_int64, c_int64,
         c_void_p, c_int64, ctypes.c_uint32, c_void_p],
    ),
    "mak_rows_scatter_static": (
        c_int32,
        [c_void_p, c_void_p, POINTER(c_int64), c_int64, c_void_p, c_int32, c_int64, c_int64, c_void_p],
    ),
    "mak_build_indexed_slots": (
        c_int32,
        [c_void_p, c_int32, c_void_p, c_int32, c_int64, c_int64, c_int64, c_void_p, c_void_p],
    ),
    "mak_lmcache_strided_block_transfer": (
        c_int32,
        [c_void_p, POINTER(c_uint64), c_void_p] + [c_int64] * 12 + [c_void_p],
    ),
    "mak_memcpy_batch": (c_int32, [POINTER(CopyEntry), c_int64, c_int32, c_int64, c_void_p]),
    "mak_runtime_versions": (c_int32, [POINTER(c_int32), POINTER(c_int32)]),
    "mak_minmax": (c_int32, [c_void_p, c_int32, c_int64, c_void_p, c_void_p]),
    "mak_cachegen_encode": (c_int32, [c_void_p, c_int32, c_int64, c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p]),
    "mak_cachegen_codebook": (c_int32, [c_void_p, c_int32, c_void_p, c_void_p]),
    "mak_cachegen_decode": (c_int32, [c_void_p, c_int64, c_void_p, c_int32, c_int32, c_void_p, c_int32, c_void_p]),
    "mak_mla_fp8_row_bytes": (c_int64, [c_int64, c_int64]),
    "mak_rope_dense": (c_int32, [c_void_p, c_void_p]),
    "mak_rope_key_cache": (c_int32, [c_void_p, c_void_p]),
    "mak_ipc_handle_bytes": (c_int32, []),
    "mak_ipc_export": (c_int32, [c_void_p, c_void_p, POINTER(c_int64)]),
    "mak_ipc_import": (c_int32, [c_void_p, c_int64, POINTER(c_void_p)]),
    "mak_ipc_release": (c_int32, [c_void_p]),
    "mak_mla_fp8_rows_store": (
        c_int32,
        [POINTER(MlaLinearDesc), c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_size_t, c_void_p],
    ),
    "mak_mla_fp8_rows_load": (c_int32, [c_void_p, POINTER(MlaLinearDesc), c_void_p, c_int32, c_int32, c_void_p]),
    "mak_mla_fp8_rows_store_owned": (
        c_int32,
        [POINTER(MlaLinearDesc), c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_int64, ctypes.c_uint32, c_void_p],
    ),
    "mak_fp8_quotient_selfcheck": (c_int32, [c_int32, c_int32, c_int32, c_void_p, c_void_p]),
    "mak_rows_copy_owned": (
        c_int32,
        [c_void_p, c_void_p, POINTER(c_int64), c_int64, c_void_p, c_int32, c_void_p, c_int32, c_int64, c_void_p, c_int64,
         ctypes.c_uint32, c_void_p],
    ),
    "mak_rows_copy": (
        c_int32,
        [
            c_void_p,
            c_void_p,
            POINTER(c_int64),
            c_int64,
            c_void_p,
            c_int32,
            c_void_p,
            c_int32,
            c_int64,
            c_void_p,
            c_size_t,
            c_void_p,
        ],
    ),
}

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None
_LOAD_ERROR: str | None = None


def library_path() -> str:
    return os.environ.get("MUSA_AITER_KVCACHE_LIB", str(_build.LIB_PATH))


def load() -> ctypes.CDLL:
    """Load and bind the kernel library once; raise RuntimeError if it is unavailable."""
    global _LIB, _LOAD_ERROR
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        path = library_path()
        if not os.path.exists(path):
            _LOAD_ERROR = f"{path} not found: build it with musa_aiter.build_native_kv_transfer()"
            raise RuntimeError(f"musa_aiter kvcache native library missing: {_LOAD_ERROR}")
        lib = ctypes.CDLL(path)
        for name, (restype, argtypes) in _PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        version = lib.mak_abi_version()
        if version != ABI_VERSION:
            raise RuntimeError(f"musa_aiter kvcache native library ABI {version} != expected {ABI_VERSION}")
        _LIB = lib
        return lib


def is_available() -> bool:
    try:
        load()
        return True
    except Exception:
        return False


def launch_count() -> int:
    """Kernels launched by the library so far (host-side counter)."""
    return int(load().mak_launch_count())


def exported_symbols() -> list[str]:
    return list(_PROTOTYPES)


def check(rc: int, op: str) -> None:
    if rc != 0:
        msg = load().mak_last_error().decode(errors="replace")
        raise RuntimeError(f"{op}: native kernel library returned {rc}: {msg}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype for the kvcache native library: {dtype}") from None


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_ptr(device: torch.device) -> int:
    """Current CUDA stream of ``device`` as an address (the reference passes
    stream 0 in places; this backend always honours the caller's current stream)."""
    if _RAW_STREAM is not None:
        idx = device.index
        return _RAW_STREAM(idx if idx is not None else torch.cuda.current_device())
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return t.data_ptr() if t is not None else None


def workspace(n_items: int, device: torch.device) -> tuple[torch.Tensor, int]:
    """Scatter workspace from torch's caching allocator (stream-ordered reuse is safe)."""
    nbytes = int(load().mak_scatter_workspace_bytes(int(n_items)))
    return torch.empty(nbytes, dtype=torch.uint8, device=device), nbytes


# Owner tables for the two-launch scatter (mak_rows_scatterv_owned): one zeroed
# int64 vector per (device, stream), grown to the largest destination seen, and
# the next epoch.  The lock makes epoch order equal enqueue order on a stream.
_OWNER_LOCK = threading.Lock()
_OWNERS: dict = {}
_EPOCH_MAX = (1 << 32) - 1
_OWNER_MAX_ROWS = 1 << 27  # 1 GiB of table; larger destinations take the workspace path


def owned_scatter(device: torch.device, stream: int, rows: int, n: int, launch):
    """Call ``launch(owner_ptr, owner_rows, epoch)`` with this stream's owner table and a fresh
    epoch and return its status, or return None when the workspace path must be used instead
    (stream capture: a captured epoch would be replayed; very large destinations or calls)."""
    if rows > _OWNER_MAX_ROWS or n >= _EPOCH_MAX or torch.cuda.is_current_stream_capturing():
        return None
    key = (device.index, stream)
    with _OWNER_LOCK:
        ent = _OWNERS.get(key)
        if ent is None or ent[1] < rows:
            cap = max(rows, 2 * ent[1]) if ent is not None else max(rows, 1 << 16)
            cap = min(cap, _OWNER_MAX_ROWS)
            t = torch.zeros(cap, dtype=torch.int64, device=device)
            ent = _OWNERS[key] = [t, cap, t.data_ptr(), 1]
        epoch = ent[3]
        if epoch > _EPOCH_MAX:
            ent[0].zero_()
            epoch = 1
        ent[3] = epoch + 1
        return launch(ent[2], ent[1], epoch)


# Segment maps for the tile engine's long-run / short-run launch pair
# (mak_kv_*_mapped): one uint32 vector per (device, stream), one entry per 8
# tokens of the largest call seen, and the next epoch.  Every entry the short-run
# launch reads was written by the long-run launch of the same call, so the
# contents never need clearing, and a wrapped epoch may start again at 1.
_SEGMAPS: dict = {}
_SEG_EPOCH_MAX = (1 << 30) - 1
_SEGMAP_MAX_ENTRIES = 1 << 28


def seg_map(device: torch.device, stream: int, n_tokens: int) -> tuple[int | None, int, int]:
    """(map address, entries, epoch) for one tile call of ``n_tokens`` tokens on this stream, or
    (None, 0, 0) where the short-run launch scans every window instead (stream capture: replays
    of a captured epoch could meet on one map; very large calls)."""
    need = (int(n_tokens) + 7) // 8
    if need <= 0 or need > _SEGMAP_MAX_ENTRIES or torch.cuda.is_current_stream_capturing():
        return None, 0, 0
    key = (device.index, stream)
    with _OWNER_LOCK:
        ent = _SEGMAPS.get(key)
        if ent is None or ent[1] < need:
            cap = max(need, 2 * ent[1]) if ent is not None else max(need, 1 << 12)
            cap = min(cap, _SEGMAP_MAX_ENTRIES)
            t = torch.zeros(cap, dtype=torch.int32, device=device)
            ent = _SEGMAPS[key] = [t, cap, t.data_ptr(), 1]
        epoch = ent[3]
        if epoch > _SEG_EPOCH_MAX:
            epoch = 1
        ent[3] = epoch + 1
        return ent[2], ent[1], epoch


def rows_copy(src_desc, dst_desc, row_bytes0: int, si: int, sdt: int, di: int, ddt: int, n: int, dst_rows: int,
              device: torch.device, stream: int) -> int:
    """``mak_rows_copy`` with an indexed destination: duplicate destinations resolved through this
    stream's owner table (``mak_rows_copy_owned``), or through a workspace from torch's caching
    allocator where owner tables do not apply (stream capture, very large destinations)."""
    lib = load()
    rc = owned_scatter(device, stream, dst_rows, n, lambda own, orows, epoch: lib.mak_rows_copy_owned(
        src_desc, dst_desc, None, row_bytes0, si, sdt, di, ddt, n, own, orows, epoch, stream))
    if rc is None:
        ws, nbytes = workspace(n, device)
        rc = lib.mak_rows_copy(src_desc, dst_desc, None, row_bytes0, si, sdt, di, ddt, n, ws.data_ptr(), nbytes, stream)
    return rc


def plane_array(ptrs: list[int]):
    arr = (c_uint64 * max(1, len(ptrs)))(*ptrs)
    return arr


def rows_pack(*sides):
    """One C buffer holding a ``mak_rows_desc`` per side followed by all plane pointer arrays.

    Each side is ``(ptrs, rows_per_block, block_stride, row_stride, num_rows)``;
    descriptor ``i`` starts at byte ``48 * i`` of the buffer (the struct is six
    64-bit words).  Built with one slice assignment: constructing ctypes
    Structures per call costs several microseconds more per launch."""
    n = len(sides)
    words = [0] * (6 * n)
    tail: list[int] = []
    for i, (ptrs, rpb, bstride, rstride, nrows) in enumerate(sides):
        words[6 * i: 6 * i + 6] = (len(tail), len(ptrs), rpb, bstride, rstride, nrows)
        tail += ptrs
    buf = (c_int64 * (6 * n + max(1, len(tail))))()
    pbase = ctypes.addressof(buf) + 48 * n
    for i in range(n):
        words[6 * i] = pbase + 8 * words[6 * i]
    words += tail
    buf[: len(words)] = words
    return buf


_PACK_CACHE: dict = {}
_PACK_CACHE_MAX = 256


def cached(key, build):
    """Memoise a descriptor buffer for long-lived tensors (KV caches).  ``key`` must include every
    pointer, shape and stride the buffer encodes, so a hit is always a valid descriptor."""
    hit = _PACK_CACHE.get(key)
    if hit is None:
        if len(_PACK_CACHE) >= _PACK_CACHE_MAX:
            _PACK_CACHE.clear()
        hit = _PACK_CACHE[key] = build()
    return hit


def rows_desc_array(sides):
    """A C array of ``mak_rows_desc`` (one per group) for the grouped entry points;
    returns ``(array, keepalive)``."""
    buf = rows_pack(*sides)
    return buf, buf


def rows_desc(ptrs: list[int], rows_per_block: int, block_stride: int, row_stride: int, num_rows: int):
    """One ``mak_rows_desc`` (pass it with ``ctypes.byref``); returns ``(desc, keepalive)``."""
    buf = rows_pack((ptrs, rows_per_block, block_stride, row_stride, num_rows))
    return buf, buf
