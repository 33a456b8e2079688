"""musa_aiter — B200-native (sm_100a) drop-in for the musa-aiter ``kvcache`` operator family.

The public names below keep the reference's signatures (musa_aiter/__init__.py:31-133
of musa-aiter v0.5.0).  Every data-moving call runs hand-written CUDA kernels from
``lib/libmak_kvcache.so`` on the caller's current CUDA stream; CPU tensors are
rejected (there is no CPU fallback).
"""

from .version import __version__
from . import registry, dispatch
from .ops.cache import apply_rope, apply_rope_to_key_cache, copy_to_kv_cache
from .ops.kv_layout import KVFormatFacts, KVLayoutKind, KVLayoutSpec, KVOrganization, KVScaleKind
from .ops.kv_transfer_plan import (
    KVTransferEntry,
    KVTransferPlan,
    assess_direct_eligibility,
    build_slot_mapping,
    build_transfer_plan,
    plan_slot_runs,
    validate_transfer_plan,
)
from .ops.kv_backend import KVBackend, KVBackendCapabilities, KVBackendDecision, native_capabilities, select_kv_backend
from .ops.lmcache_format import LMCacheFormat, LMCacheFormatFacts, describe_lmcache_format, describe_sglang_split_list
from .ops.hicache_transfer import (
    build_native_hicache_transfer,
    hicache_transfer_kv_all_layer,
    hicache_transfer_kv_all_layer_direct_lf_pf,
    hicache_transfer_kv_all_layer_lf_pf,
    hicache_transfer_kv_all_layer_mla,
    hicache_transfer_kv_all_layer_mla_lf_pf,
    hicache_transfer_kv_direct,
    hicache_transfer_kv_per_layer,
    hicache_transfer_kv_per_layer_direct_pf_lf,
    hicache_transfer_kv_per_layer_mla,
    hicache_transfer_kv_per_layer_mla_pf_lf,
    hicache_transfer_kv_per_layer_pf_lf,
    is_native_hicache_transfer_available,
    native_hicache_transfer_abi_version,
)
from .ops.kv_transfer import (
    InterleavedFp8Layout,
    PoolSpec,
    kv_cachegen_decode,
    kv_cachegen_encode,
    kv_copy_paged_blocks,
    kv_copy_paged_blocks_fp8,
    kv_copy_paged_rows,
    kv_copy_paged_rows_layer_table,
    kv_copy_paged_rows_multi_pool,
    kv_load_and_dequantize_fp8_flash,
    kv_load_and_reshape_flash,
    kv_reshape_and_cache_back_flash,
    kv_transfer_stats,
    kv_triton_indexed_to_dense,
    reset_kv_transfer_stats,
    build_native_fp8_kv_cache,
    build_native_kv_transfer,
    is_native_fp8_kv_cache_available,
    is_native_fp8_kv_vectorized_available,
    is_native_kv_transfer_available,
    kv_linear_to_paged,
    kv_linear_to_paged_fp8,
    kv_linear_to_paged_fp8_multi_layer,
    kv_linear_to_paged_multi_layer,
    kv_merged_linear_to_paged,
    kv_merged_linear_to_paged_fp8,
    kv_merged_linear_to_paged_fp8_multi_layer,
    kv_merged_linear_to_paged_multi_layer,
    kv_mla_linear_to_paged,
    kv_mla_linear_to_paged_fp8_rows,
    kv_mla_linear_to_paged_multi_layer,
    kv_paged_fp8_rows_to_mla_linear,
    kv_paged_fp8_to_linear,
    kv_paged_fp8_to_linear_multi_layer,
    kv_paged_fp8_to_merged_linear,
    kv_paged_fp8_to_merged_linear_multi_layer,
    kv_paged_to_linear,
    kv_paged_to_linear_multi_layer,
    kv_paged_to_merged_linear,
    kv_paged_to_merged_linear_multi_layer,
    kv_paged_to_mla_linear,
    kv_paged_to_mla_linear_multi_layer,
    mla_fp8_row_bytes,
    native_fp8_kv_cache_abi_version,
    native_kv_transfer_abi_version,
)
from .ops.lmcache_musa_batch_copy import (
    is_native_lmcache_musa_batch_copy_available,
    lmcache_musa_memcpy_batch_async,
    native_lmcache_musa_batch_copy_abi_version,
    native_lmcache_musa_batch_copy_runtime_versions,
)
from .ops.lmcache_kv_transfer import (
    clear_native_lmcache_kv_transfer_cache,
    is_native_lmcache_kv_transfer_available,
    is_native_lmcache_two_x_nl_kv_transfer_available,
    lmcache_kv_buffer_to_paged,
    lmcache_kv_buffer_to_paged_mla,
    lmcache_kv_buffer_to_paged_two_x_nl,
    lmcache_kv_paged_to_buffer,
    lmcache_kv_paged_to_buffer_two_x_nl,
    lmcache_kv_strided_block_transfer,
    lmcache_mla_buffer_to_paged,
    lmcache_mla_paged_to_buffer,
    lmcache_paged_to_kv_buffer,
    lmcache_paged_to_kv_buffer_mla,
    native_lmcache_kv_transfer_abi_version,
)

__all__ = [name for name in dir() if not name.startswith("_") and name not in ("registry", "dispatch", "ops", "version")]
