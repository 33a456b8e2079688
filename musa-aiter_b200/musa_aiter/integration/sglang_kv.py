"""SGLang caller-side routes of the kvcache path on B200.

Mirrors the HiCache and KV-cache routes of the reference adapter
(musa_aiter/integration/sglang_kv.py:187-1262, 1263-1327, 1860-2056): the same
function names, gates (``MUSA_AITER_SGLANG_ADAPTER``,
``MUSA_AITER_NATIVE_CPU_HOST_KV_TRANSFER``), decisions and return contracts
(``True`` / a result when the route ran, ``False`` / ``None`` when the caller
must use its own path).  "Device tensors" here are CUDA tensors.

What changes is how the routes move bytes.  The reference reshapes layer-first
``[tokens, kv_heads, head_dim]`` caches into its paged tile layout, runs its
gather and scatter, and copies the tiles back; here a token row is one row of
the row engine, so a route is one gather (zero rows for negative source
indices) plus one scatter (last writer wins, negative destinations skipped),
K and V together, straight between the caches.  Pinned host caches are read
and written in place by the kernels (zero-copy over PCIe); pageable host
caches go through the same CPU index ops and pinned staging buffers as the
reference.  The attention preload / replacement routes of the reference
adapter belong to the attention kernels, not to this path, and are not built.
"""

from __future__ import annotations

import ctypes
import logging
import os
from dataclasses import dataclass
from importlib.util import find_spec
from typing import Literal

import torch

from .. import _native
from ..ops._common import check_slots_in_bounds, kernel_slots
from ..ops.hicache_transfer import (
    hicache_transfer_kv_all_layer,
    hicache_transfer_kv_all_layer_direct_lf_pf,
    hicache_transfer_kv_all_layer_lf_pf,
    hicache_transfer_kv_all_layer_mla_lf_pf,
    hicache_transfer_kv_direct,
    hicache_transfer_kv_per_layer,
    hicache_transfer_kv_per_layer_direct_pf_lf,
    hicache_transfer_kv_per_layer_mla,
    hicache_transfer_kv_per_layer_mla_pf_lf,
    hicache_transfer_kv_per_layer_pf_lf,
)
from ..ops.kv_transfer import (
    kv_copy_paged_blocks,
    kv_copy_paged_blocks_fp8,
    kv_copy_paged_rows_layer_table,
    kv_load_and_dequantize_fp8_flash,
    kv_load_and_reshape_flash,
)

HiCacheIOBackend = Literal["direct", "kernel"]

logger = logging.getLogger(__name__)

__all__ = [
    "HiCacheIOBackend",
    "SGLangAdapterDecision",
    "SGLangHiCacheBackendDecision",
    "check_kv_copy_paged_blocks",
    "check_kv_load_and_dequantize_fp8_flash",
    "check_kv_load_and_reshape_flash",
    "clear_sglang_cpu_host_staging_cache",
    "is_sglang_cpu_host_staging_cache_enabled",
    "is_sglang_kv_route_logging_enabled",
    "is_sglang_kv_route_profile_enabled",
    "is_sglang_musa_aiter_adapter_enabled",
    "is_sglang_native_cpu_host_kv_transfer_enabled",
    "resolve_hicache_io_backend_for_musa",
    "sglang_integration_import_status",
    "try_kv_copy_paged_blocks",
    "try_kv_copy_paged_blocks_fp8",
    "try_kv_load_and_dequantize_fp8_flash",
    "try_kv_load_and_reshape_flash",
    "try_sglang_hicache_direct_transfer",
    "try_sglang_hicache_flat_paged_transfer",
    "try_sglang_hicache_layer_first_cpu_host_transfer",
    "try_sglang_hicache_layer_first_cpu_host_transfer_multi_layer",
    "try_sglang_hicache_layer_first_transfer",
    "try_sglang_hicache_layout_transfer",
]


# ---------------------------------------------------------------------------
# gates and decisions (reference sglang_kv.py:47-239)
# ---------------------------------------------------------------------------


def is_sglang_kv_route_logging_enabled() -> bool:
    return os.environ.get("MUSA_AITER_SGLANG_KV_LOG", "0") == "1"


def is_sglang_kv_route_profile_enabled() -> bool:
    return os.environ.get("MUSA_AITER_SGLANG_KV_PROFILE", "0") == "1"


def is_sglang_musa_aiter_adapter_enabled() -> bool:
    return os.environ.get("MUSA_AITER_SGLANG_ADAPTER", "0") == "1"


def is_sglang_native_cpu_host_kv_transfer_enabled() -> bool:
    return any(os.environ.get(n, "0") == "1" for n in ("MUSA_AITER_NATIVE_CPU_HOST_KV_TRANSFER", "MUSA_AITER_NATIVE_KV_TRANSFER"))


def is_sglang_cpu_host_staging_cache_enabled() -> bool:
    return os.environ.get("MUSA_AITER_CPU_HOST_STAGING_CACHE", "1") != "0"


def _log_route(message: str, *args) -> None:
    if is_sglang_kv_route_logging_enabled():
        logger.info("musa_aiter SGLang KV route: " + message, *args)


@dataclass(frozen=True)
class SGLangAdapterDecision:
    enabled: bool
    reason: str
    op: str


@dataclass(frozen=True)
class SGLangHiCacheBackendDecision:
    backend: HiCacheIOBackend
    use_musa_aiter_adapter: bool
    reason: str


def sglang_integration_import_status() -> dict[str, bool]:
    modules = ("sglang", "sglang.srt.mem_cache.memory_pool_host", "sglang.srt.managers.cache_controller",
               "sglang.srt.layers.attention.flashattention_backend", "musa_aiter")
    status: dict[str, bool] = {}
    for module in modules:
        try:
            status[module] = find_spec(module) is not None
        except (ImportError, ModuleNotFoundError, ValueError):
            status[module] = False
    return status


def resolve_hicache_io_backend_for_musa(backend: str, *, is_musa: bool, adapter_available: bool,
                                        layout_supported: bool) -> SGLangHiCacheBackendDecision:
    """Reference :219-237; ``is_musa`` means "the accelerator runtime of this build" (CUDA here)."""
    if backend not in ("direct", "kernel"):
        return SGLangHiCacheBackendDecision("direct", False, f"unsupported backend {backend!r}")
    if backend == "direct":
        return SGLangHiCacheBackendDecision("direct", False, "direct is fallback/debug transfer path")
    if not is_musa:
        return SGLangHiCacheBackendDecision("kernel", False, "not a MUSA runtime")
    if not adapter_available:
        return SGLangHiCacheBackendDecision("kernel", False, "musa_aiter adapter is not available")
    if not layout_supported:
        return SGLangHiCacheBackendDecision("kernel", False, "layout is not supported by musa_aiter adapter")
    return SGLangHiCacheBackendDecision("kernel", True, "use internal musa_aiter adapter under kernel backend")


def _is_dev(t) -> bool:
    return isinstance(t, torch.Tensor) and t.is_cuda


def _is_cpu(t) -> bool:
    return isinstance(t, torch.Tensor) and t.device.type == "cpu"


def _is_integer_tensor(t: torch.Tensor) -> bool:
    return t.dtype in (torch.int16, torch.int32, torch.int64)


def _env_decision(op: str, require_env: bool) -> SGLangAdapterDecision | None:
    if require_env and not is_sglang_musa_aiter_adapter_enabled():
        return SGLangAdapterDecision(False, "MUSA_AITER_SGLANG_ADAPTER is not enabled", op)
    return None


def _cpu_host_env_decision(op: str, require_env: bool) -> SGLangAdapterDecision | None:
    env = _env_decision(op, require_env)
    if env is not None:
        return env
    if require_env and not is_sglang_native_cpu_host_kv_transfer_enabled():
        return SGLangAdapterDecision(False, "MUSA_AITER_NATIVE_CPU_HOST_KV_TRANSFER is not enabled", op)
    return None


# ---------------------------------------------------------------------------
# layout-exact HiCache routes (reference :240-372)
# ---------------------------------------------------------------------------


def try_sglang_hicache_layout_transfer(
    src_k: torch.Tensor,
    dst_k: torch.Tensor,
    src_v: torch.Tensor | None,
    dst_v: torch.Tensor | None,
    src_indices: torch.Tensor,
    dst_indices: torch.Tensor,
    *,
    source_layout: Literal["layer_first", "page_first"],
    destination_layout: Literal["layer_first", "page_first"],
    layer_id: int | None = None,
    mla: bool = False,
    require_env: bool = True,
) -> bool:
    """Route exact HiCache layout tensors to the hicache_transfer ops (device tensors only)."""
    op = f"sglang_hicache_{source_layout}_to_{destination_layout}"
    if require_env and not is_sglang_musa_aiter_adapter_enabled():
        _log_route("fallback op=%s reason=adapter_disabled", op)
        return False
    tensors = [src_k, dst_k, src_indices, dst_indices] + [t for t in (src_v, dst_v) if t is not None]
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        _log_route("fallback op=%s reason=non_tensor_input", op)
        return False
    if not all(_is_dev(t) for t in tensors):
        _log_route("fallback op=%s reason=all_inputs_must_be_device_tensors", op)
        return False
    if source_layout not in ("layer_first", "page_first") or destination_layout not in ("layer_first", "page_first"):
        _log_route("fallback op=%s reason=unsupported_layout", op)
        return False
    if source_layout == "page_first" and destination_layout == "layer_first":
        if mla:
            return hicache_transfer_kv_per_layer_mla_pf_lf(src_k, dst_k, src_indices, dst_indices, layer_id=layer_id or 0)
        if layer_id is None:
            _log_route("fallback op=%s reason=page_first_all_layer_requires_explicit_route", op)
            return False
        return hicache_transfer_kv_per_layer_pf_lf(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, layer_id=layer_id)
    if source_layout == "layer_first" and destination_layout == "page_first":
        if mla and layer_id is None:
            return hicache_transfer_kv_all_layer_mla_lf_pf(src_k, dst_k, src_indices, dst_indices)
        if mla or layer_id is not None:
            _log_route("fallback op=%s reason=unsupported_layer_first_to_page_first_contract", op)
            return False
        return hicache_transfer_kv_all_layer_lf_pf(src_k, dst_k, src_v, dst_v, src_indices, dst_indices)
    if source_layout == "layer_first" and destination_layout == "layer_first":
        if mla:
            if layer_id is None:
                _log_route("fallback op=%s reason=MLA_all_layer_not_exposed_by_adapter", op)
                return False
            return hicache_transfer_kv_per_layer_mla(src_k, dst_k, src_indices, dst_indices, layer_id=layer_id)
        if layer_id is None:
            return hicache_transfer_kv_all_layer(src_k, dst_k, src_v, dst_v, src_indices, dst_indices)
        return hicache_transfer_kv_per_layer(src_k, dst_k, src_v, dst_v, src_indices, dst_indices, layer_id=layer_id)
    _log_route("fallback op=%s reason=layout_route_not_implemented", op)
    return False


def try_sglang_hicache_direct_transfer(
    src_layers: list[torch.Tensor],
    dst_layers: list[torch.Tensor],
    src_indices: torch.Tensor,
    dst_indices: torch.Tensor,
    page_size: int,
    *,
    mode: Literal["direct", "per_layer_pf_lf", "all_layer_lf_pf"] = "direct",
    layer_id: int = 0,
    require_env: bool = True,
) -> bool:
    """Execute one of SGLang's three direct HiCache transfer contracts (reference :334-372)."""
    op = f"sglang_hicache_{mode}"
    if require_env and not is_sglang_musa_aiter_adapter_enabled():
        _log_route("fallback op=%s reason=adapter_disabled", op)
        return False
    tensors = list(src_layers) + list(dst_layers) + [src_indices, dst_indices]
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        _log_route("fallback op=%s reason=non_tensor_input", op)
        return False
    if mode == "direct":
        return hicache_transfer_kv_direct(src_layers, dst_layers, src_indices, dst_indices, page_size)
    if mode == "per_layer_pf_lf":
        return hicache_transfer_kv_per_layer_direct_pf_lf(src_layers, dst_layers, src_indices, dst_indices, layer_id,
                                                          page_size)
    if mode == "all_layer_lf_pf":
        return hicache_transfer_kv_all_layer_direct_lf_pf(src_layers, dst_layers, src_indices, dst_indices, page_size)
    raise ValueError(f"unsupported SGLang direct mode={mode!r}")


# ---------------------------------------------------------------------------
# token-row moves between layer-first caches (the row engine)
# ---------------------------------------------------------------------------


def _token_rows_move(src: list[torch.Tensor], dst: list[torch.Tensor], src_idx: torch.Tensor, dst_idx: torch.Tensor,
                     *, device: torch.device, op: str) -> None:
    """``dst[p][dst_idx[i]] = src[p][src_idx[i]]`` for every plane p, a token row being
    ``[kv_heads, head_dim]``: zero rows where ``src_idx[i] < 0`` (the reference gathers with
    zero fill), destinations ``< 0`` skipped, last writer wins.  Planes may live in pinned host
    memory (addressed in place) or on the device."""
    n = int(src_idx.numel())
    if n == 0 or not src:
        return
    s0, d0 = src[0], dst[0]
    e = s0.element_size()
    row = int(s0[0].numel()) * e
    # The reference raises on out-of-range slots through kv_paged_to_linear / kv_linear_to_paged.
    check_slots_in_bounds(src_idx, int(s0.shape[0]), 1, "kv_paged_to_linear")
    check_slots_in_bounds(dst_idx, int(d0.shape[0]), 1, "kv_linear_to_paged")
    lib = _native.load()
    stream = _native.stream_ptr(device)
    staging = torch.empty((len(src), n, row), dtype=torch.uint8, device=device)
    si, sc = kernel_slots(src_idx)
    di, dc = kernel_slots(dst_idx)
    paged = ([t.data_ptr() for t in src], 1, s0.stride(0) * e, 0, int(s0.shape[0]))
    lin = ([staging[p].data_ptr() for p in range(len(src))], 1, row, 0, n)
    buf = _native.rows_pack(paged, lin)
    base = ctypes.addressof(buf)
    _native.check(lib.mak_rows_gather(base, base + 48, None, row, si.data_ptr(), sc, n, 1, stream), op)
    dpaged = ([t.data_ptr() for t in dst], 1, d0.stride(0) * e, 0, int(d0.shape[0]))
    buf2 = _native.rows_pack(lin, dpaged)
    base2 = ctypes.addressof(buf2)
    ws, nbytes = _native.workspace(n, device)
    _native.check(lib.mak_rows_scatter(base2, base2 + 48, None, row, di.data_ptr(), dc, n, 0, ws.data_ptr(), nbytes,
                                       stream), op)


def _rows_ok(t: torch.Tensor) -> bool:
    return t.dim() >= 2 and t[0].is_contiguous()


def _can_route_sglang_layer_first_hicache(host_cache, device_cache, host_indices, device_indices, *, page_size: int,
                                          op: str, require_env: bool) -> SGLangAdapterDecision:
    env = _env_decision(op, require_env)
    if env is not None:
        return env
    tensors = (host_cache, device_cache, host_indices, device_indices)
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        return SGLangAdapterDecision(False, "all inputs must be torch.Tensor", op)
    if not _is_dev(host_cache) or not _is_dev(device_cache):
        return SGLangAdapterDecision(False, "host and device cache tensors must both be MUSA tensors", op)
    if not _is_dev(host_indices) or not _is_dev(device_indices):
        return SGLangAdapterDecision(False, "host/device indices must both be MUSA tensors", op)
    return _common_layer_first_checks(host_cache, device_cache, host_indices, device_indices, page_size=page_size, op=op)


def _common_layer_first_checks(host_cache, device_cache, host_indices, device_indices, *, page_size: int,
                               op: str) -> SGLangAdapterDecision:
    if host_cache.dtype != device_cache.dtype:
        return SGLangAdapterDecision(False, "host and device cache dtypes must match", op)
    if host_cache.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        return SGLangAdapterDecision(False, "cache dtype must be float32, float16, or bfloat16", op)
    if host_cache.dim() != 3 or device_cache.dim() != 3:
        return SGLangAdapterDecision(False, "layer cache tensors must be [tokens, kv_heads, head_dim]", op)
    if host_cache.shape[1:] != device_cache.shape[1:]:
        return SGLangAdapterDecision(False, "host/device cache inner shapes must match", op)
    if page_size <= 0:
        return SGLangAdapterDecision(False, "page_size must be positive", op)
    if int(host_cache.shape[0]) % page_size != 0 or int(device_cache.shape[0]) % page_size != 0:
        return SGLangAdapterDecision(False, "token dimension must be divisible by page_size", op)
    if not _is_integer_tensor(host_indices) or not _is_integer_tensor(device_indices):
        return SGLangAdapterDecision(False, "host/device indices must use integer dtype", op)
    if host_indices.numel() != device_indices.numel():
        return SGLangAdapterDecision(False, "host/device indices must have the same length", op)
    if host_indices.dim() != 1 or device_indices.dim() != 1:
        return SGLangAdapterDecision(False, "host/device indices must be 1-D", op)
    if not _rows_ok(host_cache) or not _rows_ok(device_cache):
        return SGLangAdapterDecision(False, "token rows [kv_heads, head_dim] must be contiguous", op)
    return SGLangAdapterDecision(True, "supported", op)


def try_sglang_hicache_layer_first_transfer(
    host_key_cache: torch.Tensor,
    host_value_cache: torch.Tensor,
    device_key_cache: torch.Tensor,
    device_value_cache: torch.Tensor,
    host_indices: torch.Tensor,
    device_indices: torch.Tensor,
    *,
    page_size: int,
    direction: Literal["host_to_device", "device_to_host"],
    require_env: bool = True,
) -> bool:
    """Layer-first ``[tokens, kv_heads, head_dim]`` K/V caches, both on the device (reference :443-589)."""
    op = f"sglang_hicache_layer_first_{direction}"
    if direction not in ("host_to_device", "device_to_host"):
        _log_route("fallback op=%s reason=unsupported_direction direction=%s", op, direction)
        return False
    for hc, dc, gate in ((host_key_cache, device_key_cache, require_env), (host_value_cache, device_value_cache, False)):
        d = _can_route_sglang_layer_first_hicache(hc, dc, host_indices, device_indices, page_size=page_size, op=op,
                                                  require_env=gate)
        if not d.enabled:
            _log_route("fallback op=%s reason=%s", op, d.reason)
            return False
    if host_key_cache.shape != host_value_cache.shape or device_key_cache.shape != device_value_cache.shape:
        _log_route("fallback op=%s stage=kv_shape_check reason=kv_shape_mismatch", op)
        return False
    if direction == "host_to_device":
        _token_rows_move([host_key_cache, host_value_cache], [device_key_cache, device_value_cache], host_indices,
                         device_indices, device=device_key_cache.device, op=op)
    else:
        _token_rows_move([device_key_cache, device_value_cache], [host_key_cache, host_value_cache], device_indices,
                         host_indices, device=device_key_cache.device, op=op)
    _log_route("success op=%s tokens=%s", op, int(host_indices.numel()))
    return True


# ---------------------------------------------------------------------------
# DSV4 flat byte-row pools (reference :606-699)
# ---------------------------------------------------------------------------


def _can_route_sglang_flat_paged_hicache(host_pool, device_pool, *, op: str, require_env: bool) -> SGLangAdapterDecision:
    env = _env_decision(op, require_env)
    if env is not None:
        return env
    if host_pool is None or device_pool is None:
        return SGLangAdapterDecision(False, "host/device pools must be objects", op)
    if getattr(host_pool, "layout", None) != "layer_first":
        return SGLangAdapterDecision(False, "host pool layout must be layer_first", op)
    host_kv = getattr(host_pool, "kv_buffer", None)
    device_kv = getattr(device_pool, "kv_buffer", None)
    if not isinstance(host_kv, torch.Tensor) or not isinstance(device_kv, torch.Tensor):
        return SGLangAdapterDecision(False, "host/device pools must expose kv_buffer tensors", op)
    if host_kv.dtype is not torch.uint8 or device_kv.dtype is not torch.uint8:
        return SGLangAdapterDecision(False, f"kv_buffer must be uint8 byte rows, got host={host_kv.dtype}, device={device_kv.dtype}", op)
    if host_kv.dim() != 3 or device_kv.dim() != 3:
        return SGLangAdapterDecision(False, "kv_buffer must be [layers, pages, item_bytes]", op)
    if host_kv.shape[0] != device_kv.shape[0] or host_kv.shape[2] != device_kv.shape[2]:
        return SGLangAdapterDecision(False, f"kv_buffer layer/item_bytes mismatch: host={tuple(host_kv.shape)}, device={tuple(device_kv.shape)}", op)
    return SGLangAdapterDecision(True, "supported", op)


def try_sglang_hicache_flat_paged_transfer(host_pool, device_pool, host_indices: torch.Tensor, device_indices: torch.Tensor,
                                           *, direction: Literal["load_to_device", "backup_from_device"],
                                           require_env: bool = True) -> bool:
    """DSV4 flat uint8 ``kv_buffer[layers, pages, item_bytes]`` pools -> ``kv_copy_paged_rows_layer_table``."""
    op = f"sglang_hicache_flat_paged_{direction}"
    if direction not in ("load_to_device", "backup_from_device"):
        _log_route("fallback op=%s reason=unsupported_direction direction=%s", op, direction)
        return False
    decision = _can_route_sglang_flat_paged_hicache(host_pool, device_pool, op=op, require_env=require_env)
    if not decision.enabled:
        _log_route("fallback op=%s reason=%s", op, decision.reason)
        return False
    if not _is_integer_tensor(host_indices) or not _is_integer_tensor(device_indices):
        _log_route("fallback op=%s reason=indices_not_integer", op)
        return False
    if host_indices.numel() != device_indices.numel() or host_indices.dim() != 1:
        _log_route("fallback op=%s reason=indices_shape", op)
        return False
    host_kv, device_kv = host_pool.kv_buffer, device_pool.kv_buffer
    src = host_kv.unbind(0) if direction == "load_to_device" else device_kv.unbind(0)
    dst = device_kv.unbind(0) if direction == "load_to_device" else host_kv.unbind(0)
    si, di = (host_indices, device_indices) if direction == "load_to_device" else (device_indices, host_indices)
    kv_copy_paged_rows_layer_table(list(src), list(dst), si, di)
    _log_route("success op=%s layers=%s rows=%s", op, int(host_kv.shape[0]), int(host_indices.numel()))
    return True


# ---------------------------------------------------------------------------
# host caches on the CPU side (reference :700-1261)
# ---------------------------------------------------------------------------

_STAGING_CACHE_MAX_ENTRIES = 32
_staging: dict[tuple, torch.Tensor] = {}


def clear_sglang_cpu_host_staging_cache() -> None:
    _staging.clear()


def _staging_tensor(name: str, *, like: torch.Tensor, shape: tuple[int, ...], device: torch.device, pin: bool) -> torch.Tensor:
    if not is_sglang_cpu_host_staging_cache_enabled():
        return torch.empty(shape, dtype=like.dtype, device=device, pin_memory=pin)
    key = (name, str(like.dtype), shape, str(device))
    t = _staging.get(key)
    if t is None:
        if len(_staging) >= _STAGING_CACHE_MAX_ENTRIES:
            _staging.clear()
        t = _staging[key] = torch.empty(shape, dtype=like.dtype, device=device, pin_memory=pin)
    return t


def _pinned(t: torch.Tensor) -> bool:
    try:
        return bool(t.is_pinned())
    except (AttributeError, RuntimeError):
        return False


def _can_route_cpu_host(host_cache, device_cache, host_indices, device_indices, *, page_size: int, op: str,
                        require_env: bool) -> SGLangAdapterDecision:
    env = _cpu_host_env_decision(op, require_env)
    if env is not None:
        return env
    tensors = (host_cache, device_cache, host_indices, device_indices)
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        return SGLangAdapterDecision(False, "all inputs must be torch.Tensor", op)
    if not _is_cpu(host_cache):
        return SGLangAdapterDecision(False, "host cache tensor must be a CPU tensor", op)
    if not _is_dev(device_cache):
        return SGLangAdapterDecision(False, "device cache tensor must be a MUSA tensor", op)
    return _common_layer_first_checks(host_cache, device_cache, host_indices, device_indices, page_size=page_size, op=op)


def _cpu_host_move(host: list[torch.Tensor], device: list[torch.Tensor], host_indices: torch.Tensor,
                   device_indices: torch.Tensor, *, direction: str, op: str) -> None:
    """Token rows between host planes ``[tokens, ...]`` (CPU) and device planes.  Pinned host planes
    are addressed in place by the kernels; pageable ones go through CPU index ops and pinned staging."""
    dev = device[0].device
    hidx_dev = host_indices.to(dev)
    didx_dev = device_indices.to(dev)
    if all(_pinned(h) for h in host):
        if direction == "host_to_device":
            _token_rows_move(host, device, hidx_dev, didx_dev, device=dev, op=op)
        else:
            _token_rows_move(device, host, didx_dev, hidx_dev, device=dev, op=op)
        torch.cuda.current_stream(dev).synchronize()  # the host rows are the caller's on return
        return
    hidx = host_indices.to("cpu", torch.long)
    n = int(hidx.numel())
    if direction == "host_to_device":
        for p, (h, d) in enumerate(zip(host, device)):
            rows = h.index_select(0, hidx.clamp(min=0))
            rows[hidx < 0] = 0
            stage = _staging_tensor(f"{op}_h2d_{p}", like=h, shape=tuple(rows.shape), device=torch.device("cpu"), pin=True)
            stage.copy_(rows)
            dev_rows = _staging_tensor(f"{op}_h2d_dev_{p}", like=h, shape=tuple(rows.shape), device=dev, pin=False)
            dev_rows.copy_(stage, non_blocking=True)
            ident = torch.arange(n, device=dev)
            _token_rows_move([dev_rows], [d], ident, didx_dev, device=dev, op=op)
        return
    for p, (h, d) in enumerate(zip(host, device)):
        dev_rows = _staging_tensor(f"{op}_d2h_dev_{p}", like=d, shape=(n,) + tuple(d.shape[1:]), device=dev, pin=False)
        ident = torch.arange(n, device=dev)
        _token_rows_move([d], [dev_rows], didx_dev, ident, device=dev, op=op)
        stage = _staging_tensor(f"{op}_d2h_{p}", like=d, shape=tuple(dev_rows.shape), device=torch.device("cpu"), pin=True)
        stage.copy_(dev_rows, non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        keep = hidx >= 0
        # last writer wins for repeated host rows: index_copy_ applies rows in order on the CPU
        h.index_copy_(0, hidx[keep], stage[keep])


def try_sglang_hicache_layer_first_cpu_host_transfer(
    host_key_cache: torch.Tensor,
    host_value_cache: torch.Tensor,
    device_key_cache: torch.Tensor,
    device_value_cache: torch.Tensor,
    host_indices: torch.Tensor,
    device_indices: torch.Tensor,
    *,
    page_size: int,
    direction: Literal["host_to_device", "device_to_host"],
    require_env: bool = True,
) -> bool:
    """Host K/V caches on the CPU side, device caches layer-first (reference :1088-1261)."""
    op = f"sglang_hicache_layer_first_cpu_host_{direction}"
    if direction not in ("host_to_device", "device_to_host"):
        return False
    for hc, dc, gate in ((host_key_cache, device_key_cache, require_env), (host_value_cache, device_value_cache, False)):
        d = _can_route_cpu_host(hc, dc, host_indices, device_indices, page_size=page_size, op=op, require_env=gate)
        if not d.enabled:
            _log_route("fallback op=%s reason=%s", op, d.reason)
            return False
    if host_key_cache.shape != host_value_cache.shape or device_key_cache.shape != device_value_cache.shape:
        return False
    _cpu_host_move([host_key_cache, host_value_cache], [device_key_cache, device_value_cache], host_indices,
                   device_indices, direction=direction, op=op)
    return True


def try_sglang_hicache_layer_first_cpu_host_transfer_multi_layer(
    host_key_cache: torch.Tensor,
    host_value_cache: torch.Tensor,
    device_key_cache: torch.Tensor,
    device_value_cache: torch.Tensor,
    host_indices: torch.Tensor,
    device_indices: torch.Tensor,
    *,
    page_size: int,
    direction: Literal["host_to_device", "device_to_host"],
    require_env: bool = True,
) -> bool:
    """``[layers, tokens, kv_heads, head_dim]`` host / device caches, all layers (reference :1003-1086)."""
    op = f"sglang_hicache_layer_first_cpu_host_multi_layer_{direction}"
    if direction not in ("host_to_device", "device_to_host"):
        return False
    env = _cpu_host_env_decision(op, require_env)
    if env is not None:
        return False
    tensors = (host_key_cache, host_value_cache, device_key_cache, device_value_cache, host_indices, device_indices)
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        return False
    if any(t.dim() != 4 for t in tensors[:4]):
        return False
    if host_key_cache.shape != host_value_cache.shape or device_key_cache.shape != device_value_cache.shape:
        return False
    if host_key_cache.shape[0] != device_key_cache.shape[0] or host_key_cache.shape[2:] != device_key_cache.shape[2:]:
        return False
    for hc, dc in ((host_key_cache[0], device_key_cache[0]), (host_value_cache[0], device_value_cache[0])):
        if not _can_route_cpu_host(hc, dc, host_indices, device_indices, page_size=page_size, op=op,
                                   require_env=False).enabled:
            return False
    nl = int(host_key_cache.shape[0])
    host = [host_key_cache[l] for l in range(nl)] + [host_value_cache[l] for l in range(nl)]
    dev = [device_key_cache[l] for l in range(nl)] + [device_value_cache[l] for l in range(nl)]
    _cpu_host_move(host, dev, host_indices, device_indices, direction=direction, op=op)
    return True


# ---------------------------------------------------------------------------
# kvcache routes with explicit checks (reference :1263-1327, 1860-2056)
# ---------------------------------------------------------------------------


def check_kv_load_and_reshape_flash(key_cache, value_cache, block_tables, seq_lens, *, require_env: bool = True) -> SGLangAdapterDecision:
    op = "kv_load_and_reshape_flash"
    env = _env_decision(op, require_env)
    if env is not None:
        return env
    tensors = (key_cache, value_cache, block_tables, seq_lens)
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        return SGLangAdapterDecision(False, "all inputs must be torch.Tensor", op)
    if not all(_is_dev(t) for t in tensors):
        return SGLangAdapterDecision(False, "all inputs must be MUSA tensors", op)
    if key_cache.dim() != 4 or value_cache.dim() != 4:
        return SGLangAdapterDecision(False, "key/value cache must be [blocks, kv_heads, head_dim, block_size]", op)
    if key_cache.shape != value_cache.shape:
        return SGLangAdapterDecision(False, "key/value cache shapes must match", op)
    if key_cache.dtype != value_cache.dtype:
        return SGLangAdapterDecision(False, "key/value cache dtypes must match", op)
    if not key_cache.is_contiguous() or not value_cache.is_contiguous():
        return SGLangAdapterDecision(False, "key/value cache must be contiguous", op)
    if block_tables.dim() != 2:
        return SGLangAdapterDecision(False, "block_tables must be [batch, max_blocks]", op)
    if seq_lens.dim() != 1 or seq_lens.shape[0] != block_tables.shape[0]:
        return SGLangAdapterDecision(False, "seq_lens must be [batch]", op)
    if not _is_integer_tensor(block_tables) or not _is_integer_tensor(seq_lens):
        return SGLangAdapterDecision(False, "block_tables and seq_lens must be integer tensors", op)
    return SGLangAdapterDecision(True, "supported", op)


def try_kv_load_and_reshape_flash(key_cache, value_cache, block_tables, seq_lens, *, max_seq_len: int | None = None,
                                  out_k=None, out_v=None, require_env: bool = True):
    if not check_kv_load_and_reshape_flash(key_cache, value_cache, block_tables, seq_lens, require_env=require_env).enabled:
        return None
    return kv_load_and_reshape_flash(key_cache, value_cache, block_tables, seq_lens, max_seq_len=max_seq_len,
                                     out_k=out_k, out_v=out_v)


def check_kv_load_and_dequantize_fp8_flash(key_cache_fp8, value_cache_fp8, block_tables, seq_lens, k_scale, v_scale, *,
                                           require_env: bool = True) -> SGLangAdapterDecision:
    op = "kv_load_and_dequantize_fp8_flash"
    base = check_kv_load_and_reshape_flash(key_cache_fp8, value_cache_fp8, block_tables, seq_lens, require_env=require_env)
    if not base.enabled:
        return SGLangAdapterDecision(False, base.reason, op)
    if key_cache_fp8.dtype is not torch.uint8 and str(key_cache_fp8.dtype) not in ("torch.float8_e4m3fn", "torch.float8_e5m2"):
        return SGLangAdapterDecision(False, "FP8 cache must be torch.uint8 or Torch FP8 dtype", op)
    for scale in (k_scale, v_scale):
        if isinstance(scale, torch.Tensor):
            if not _is_dev(scale):
                return SGLangAdapterDecision(False, "scale tensors must be on MUSA", op)
            if scale.dtype is not torch.float32:
                return SGLangAdapterDecision(False, "scale tensors must be float32", op)
            if not scale.is_contiguous():
                return SGLangAdapterDecision(False, "scale tensors must be contiguous", op)
    return SGLangAdapterDecision(True, "supported", op)


def try_kv_load_and_dequantize_fp8_flash(key_cache_fp8, value_cache_fp8, block_tables, seq_lens, k_scale, v_scale, *,
                                         max_seq_len: int | None = None, out_dtype: torch.dtype = torch.bfloat16,
                                         fp8_format: Literal["e4m3", "e5m2"] = "e4m3", out_k=None, out_v=None,
                                         require_env: bool = True):
    if not check_kv_load_and_dequantize_fp8_flash(key_cache_fp8, value_cache_fp8, block_tables, seq_lens, k_scale, v_scale,
                                                  require_env=require_env).enabled:
        return None
    return kv_load_and_dequantize_fp8_flash(key_cache_fp8, value_cache_fp8, block_tables, seq_lens, k_scale, v_scale,
                                            max_seq_len=max_seq_len, out_dtype=out_dtype, fp8_format=fp8_format,
                                            out_k=out_k, out_v=out_v)


def check_kv_copy_paged_blocks(src_key_cache, src_value_cache, dst_key_cache, dst_value_cache, block_mapping, *,
                               fp8: bool = False, require_env: bool = True) -> SGLangAdapterDecision:
    op = "kv_copy_paged_blocks_fp8" if fp8 else "kv_copy_paged_blocks"
    env = _env_decision(op, require_env)
    if env is not None:
        return env
    tensors = (src_key_cache, src_value_cache, dst_key_cache, dst_value_cache, block_mapping)
    if not all(isinstance(t, torch.Tensor) for t in tensors):
        return SGLangAdapterDecision(False, "all inputs must be torch.Tensor", op)
    if not all(_is_dev(t) for t in tensors):
        return SGLangAdapterDecision(False, "all inputs must be MUSA tensors", op)
    if not _is_integer_tensor(block_mapping):
        return SGLangAdapterDecision(False, "block_mapping must use integer dtype", op)
    if block_mapping.dim() != 2 or block_mapping.shape[1] != 2:
        return SGLangAdapterDecision(False, "block_mapping must be [num_pairs, 2]", op)
    caches = (src_key_cache, src_value_cache, dst_key_cache, dst_value_cache)
    if not all(t.is_contiguous() for t in caches):
        return SGLangAdapterDecision(False, "cache tensors must be contiguous", op)
    if src_key_cache.shape != src_value_cache.shape or dst_key_cache.shape != dst_value_cache.shape:
        return SGLangAdapterDecision(False, "K/V cache shapes must match", op)
    if src_key_cache.dim() not in (4, 5) or dst_key_cache.dim() != src_key_cache.dim():
        return SGLangAdapterDecision(False, "cache tensors must be single-layer or multi-layer paged layout", op)
    si = src_key_cache.shape[1:] if src_key_cache.dim() == 4 else src_key_cache.shape[2:]
    di = dst_key_cache.shape[1:] if dst_key_cache.dim() == 4 else dst_key_cache.shape[2:]
    if si != di:
        return SGLangAdapterDecision(False, "source/destination cache inner shapes must match", op)
    if fp8:
        if src_key_cache.dtype is not torch.uint8 and str(src_key_cache.dtype) not in ("torch.float8_e4m3fn", "torch.float8_e5m2"):
            return SGLangAdapterDecision(False, "FP8 cache must be torch.uint8 or Torch FP8 dtype", op)
    elif src_key_cache.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        return SGLangAdapterDecision(False, "cache dtype must be float32, float16, or bfloat16", op)
    if not (src_key_cache.dtype == src_value_cache.dtype == dst_key_cache.dtype == dst_value_cache.dtype):
        return SGLangAdapterDecision(False, "all cache dtypes must match", op)
    return SGLangAdapterDecision(True, "supported", op)


def try_kv_copy_paged_blocks(src_key_cache, src_value_cache, dst_key_cache, dst_value_cache, block_mapping, *,
                             require_env: bool = True) -> int | None:
    if not check_kv_copy_paged_blocks(src_key_cache, src_value_cache, dst_key_cache, dst_value_cache, block_mapping,
                                      require_env=require_env).enabled:
        return None
    return kv_copy_paged_blocks(src_key_cache, src_value_cache, dst_key_cache, dst_value_cache, block_mapping)


def try_kv_copy_paged_blocks_fp8(src_key_cache_fp8, src_value_cache_fp8, dst_key_cache_fp8, dst_value_cache_fp8,
                                 block_mapping, *, require_env: bool = True) -> int | None:
    if not check_kv_copy_paged_blocks(src_key_cache_fp8, src_value_cache_fp8, dst_key_cache_fp8, dst_value_cache_fp8,
                                      block_mapping, fp8=True, require_env=require_env).enabled:
        return None
    return kv_copy_paged_blocks_fp8(src_key_cache_fp8, src_value_cache_fp8, dst_key_cache_fp8, dst_value_cache_fp8,
                                    block_mapping)
