"""Operator capability registry for the ``kvcache`` family.

Keeps the reference's record type and query functions (musa_aiter/registry.py:7-56)
and the 36 ``kvcache`` operator names (musa_aiter/registry.py:87-122, pinned by
op_tests/test_kvcache_registry.py:4-44).  Every entry lists one backend,
``cuda-sm100a`` (the hand-written sm_100a kernels), and one device, ``cuda``:
there is no reference/CPU backend in this build.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Iterable

from .dispatch import BACKEND


@dataclass(frozen=True)
class OperatorCapability:
    name: str
    family: str
    status: str
    dtypes: tuple[str, ...]
    devices: tuple[str, ...]
    backends: tuple[str, ...]
    description: str
    notes: tuple[str, ...] = field(default_factory=tuple)
    vendor_backends: tuple[str, ...] = field(default_factory=tuple)


_REGISTRY: dict[str, OperatorCapability] = {}


def register(capability: OperatorCapability) -> OperatorCapability:
    if capability.name in _REGISTRY:
        raise ValueError(f"duplicate operator capability: {capability.name}")
    _REGISTRY[capability.name] = capability
    return capability


def get(name: str) -> OperatorCapability:
    return _REGISTRY[name]


def list_capabilities(family: str | None = None) -> list[OperatorCapability]:
    values: Iterable[OperatorCapability] = _REGISTRY.values()
    if family is not None:
        values = [cap for cap in values if cap.family == family]
    return sorted(values, key=lambda cap: (cap.family, cap.name))


def as_dict() -> dict[str, dict]:
    return {
        name: {
            "name": cap.name,
            "family": cap.family,
            "status": cap.status,
            "dtypes": list(cap.dtypes),
            "devices": list(cap.devices),
            "backends": list(cap.backends),
            "description": cap.description,
            "notes": list(cap.notes),
            "vendor_backends": list(cap.vendor_backends),
        }
        for name, cap in sorted(_REGISTRY.items())
    }


_FLOAT = ("float32", "float16", "bfloat16")
_HALF = ("float16", "bfloat16")
_FP8_STORE = ("float16", "bfloat16", "float32", "uint8")
_FP8_LOAD = ("uint8", "float16", "bfloat16", "float32")
_FP8_RAW = ("uint8", "float8_e4m3fn", "float8_e5m2")

# name, status, dtypes, description, notes
_KVCACHE = [
    ("kv_cachegen_encode", "b200", _FLOAT, "CacheGen-style uniform-bin KV tensor encode with empirical CDF metadata.", ()),
    ("kv_cachegen_decode", "b200", ("uint8",), "CacheGen-style uint8 codebook decode.", ()),
    ("kv_copy_paged_blocks", "b200", _FLOAT, "Copy selected paged KV cache blocks between same-layout caches.", ()),
    ("kv_copy_paged_blocks_fp8", "b200", _FP8_RAW, "Raw FP8 paged KV cache block copy.", ()),
    ("kv_load_and_reshape_flash", "b200", _FLOAT, "Paged KV caches -> dense Flash-style [batch, seq, kv_heads, head_dim].", ()),
    ("kv_load_and_dequantize_fp8_flash", "b200", _FP8_RAW, "Paged FP8 KV caches -> dense dequantized Flash-style tensors.", ()),
    ("kv_reshape_and_cache_back_flash", "b200", _FLOAT, "Dense Flash-style KV -> paged KV caches.", ()),
    ("kv_paged_to_linear", "b200", _FLOAT, "Paged KV -> token-major linear gather (single layer).", ()),
    ("kv_paged_fp8_to_linear", "b200", _FP8_LOAD, "Paged FP8 KV cache -> linear dequantize gather.", ()),
    ("kv_linear_to_paged", "b200", _FLOAT, "Token-major KV -> paged scatter (single layer).", ()),
    ("kv_linear_to_paged_fp8", "b200", _FP8_STORE, "Linear KV -> paged FP8 cache quantize scatter.", ()),
    ("kv_paged_to_linear_multi_layer", "b200", _FLOAT, "Paged KV -> linear gather (multi-layer stack, one launch).", ()),
    ("kv_paged_fp8_to_linear_multi_layer", "b200", _FP8_LOAD, "Paged FP8 KV -> linear dequantize gather (multi-layer).", ()),
    ("kv_paged_fp8_to_merged_linear", "b200", _FP8_LOAD, "Paged FP8 KV -> merged linear dequantize gather.", ()),
    ("kv_paged_fp8_to_merged_linear_multi_layer", "b200", _FP8_LOAD, "Paged FP8 KV -> merged linear dequantize gather (multi-layer).", ()),
    ("kv_linear_to_paged_multi_layer", "b200", _FLOAT, "Linear -> paged scatter (multi-layer stack, one launch).", ()),
    ("kv_linear_to_paged_fp8_multi_layer", "b200", _FP8_STORE, "Linear KV -> paged FP8 quantize scatter (multi-layer).", ()),
    ("kv_merged_linear_to_paged_fp8", "b200", _FP8_STORE, "Merged linear KV -> paged FP8 quantize scatter.", ()),
    ("kv_merged_linear_to_paged_fp8_multi_layer", "b200", _FP8_STORE, "Merged linear KV -> paged FP8 quantize scatter (multi-layer).", ()),
    ("kv_paged_to_merged_linear", "b200", _FLOAT, "Paged KV -> merged token-major [T, 2, kv_heads, head_dim].", ()),
    ("kv_merged_linear_to_paged", "b200", _FLOAT, "Merged token-major [T, 2, kv_heads, head_dim] -> paged.", ()),
    ("kv_paged_to_merged_linear_multi_layer", "b200", _FLOAT, "Paged KV -> merged [L, T, 2, kv_heads, head_dim].", ()),
    ("kv_merged_linear_to_paged_multi_layer", "b200", _FLOAT, "Merged [L, T, 2, kv_heads, head_dim] -> paged.", ()),
    ("kv_paged_to_mla_linear", "b200", _FLOAT, "MLA asymmetric flat paged caches -> [T, kv_dim] and [T, pe_dim].", ()),
    ("kv_mla_linear_to_paged", "b200", _FLOAT, "MLA asymmetric linear -> flat paged caches.", ()),
    ("kv_paged_to_mla_linear_multi_layer", "b200", _FLOAT, "Stacked MLA flat caches -> layer-major linear buffers.", ()),
    ("kv_mla_linear_to_paged_multi_layer", "b200", _FLOAT, "Layer-major MLA linear buffers -> stacked flat caches.", ()),
    ("hicache_transfer_kv_per_layer", "b200", _HALF, "SGLang HiCache per-layer layer-first transfer.", ()),
    ("hicache_transfer_kv_per_layer_pf_lf", "b200", _HALF, "SGLang HiCache per-layer page-first -> layer-first transfer.", ()),
    ("hicache_transfer_kv_all_layer", "b200", _HALF, "SGLang HiCache all-layer layer-first transfer.", ()),
    ("hicache_transfer_kv_all_layer_lf_pf", "b200", _HALF, "SGLang HiCache all-layer layer-first -> page-first transfer.", ()),
    ("hicache_transfer_kv_per_layer_mla", "b200", _HALF, "SGLang HiCache per-layer MLA layer-first transfer.", ()),
    ("hicache_transfer_kv_per_layer_mla_pf_lf", "b200", _HALF, "SGLang HiCache per-layer MLA page-first -> layer-first transfer.", ()),
    ("lmcache_kv_paged_to_buffer_two_x_nl", "b200", _FLOAT, "Gather SGLang MP 2 x NL x [NB, BS, NH, HS] caches into an LMCache [2, NL, T, NH*HS] buffer.", ()),
    ("lmcache_kv_buffer_to_paged_two_x_nl", "b200", _FLOAT, "Scatter an LMCache [2, NL, T, NH*HS] buffer into SGLang MP caches.", ()),
    ("lmcache_musa_memcpy_batch_async", "b200", ("uint8",), "Asynchronous host/device byte-copy batch for LMCache direct transfer.", ()),
]

for _name, _status, _dtypes, _desc, _notes in _KVCACHE:
    register(OperatorCapability(_name, "kvcache", _status, _dtypes, ("cuda",), (BACKEND,), _desc, _notes, ("handwritten-cuda-sm100a",)))

# The `cache` family entries the reference registers (musa_aiter/registry.py:85-86), the write-side
# producers of the kvcache path.
_CACHE = [
    ("apply_rope", "b200", _FLOAT, "RoPE with the reference's per-operation rounding.", ()),
    ("apply_rope_to_key_cache", "b200", _FLOAT, "Apply RoPE in place to selected paged key-cache slots.", ()),
]
for _name, _status, _dtypes, _desc, _notes in _CACHE:
    register(OperatorCapability(_name, "cache", _status, _dtypes, ("cuda",), (BACKEND,), _desc, _notes, ("handwritten-cuda-sm100a",)))
