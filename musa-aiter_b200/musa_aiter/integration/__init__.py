"""Caller-side integration routes (SGLang HiCache / kvcache) on the B200 kvcache path."""

from .sglang_kv import (  # noqa: F401
    SGLangAdapterDecision,
    SGLangHiCacheBackendDecision,
    check_kv_copy_paged_blocks,
    check_kv_load_and_dequantize_fp8_flash,
    check_kv_load_and_reshape_flash,
    clear_sglang_cpu_host_staging_cache,
    is_sglang_cpu_host_staging_cache_enabled,
    is_sglang_kv_route_logging_enabled,
    is_sglang_kv_route_profile_enabled,
    is_sglang_musa_aiter_adapter_enabled,
    is_sglang_native_cpu_host_kv_transfer_enabled,
    resolve_hicache_io_backend_for_musa,
    sglang_integration_import_status,
    try_kv_copy_paged_blocks,
    try_kv_copy_paged_blocks_fp8,
    try_kv_load_and_dequantize_fp8_flash,
    try_kv_load_and_reshape_flash,
    try_sglang_hicache_direct_transfer,
    try_sglang_hicache_flat_paged_transfer,
    try_sglang_hicache_layer_first_cpu_host_transfer,
    try_sglang_hicache_layer_first_cpu_host_transfer_multi_layer,
    try_sglang_hicache_layer_first_transfer,
    try_sglang_hicache_layout_transfer,
)
from .sglang_kv import __all__  # noqa: F401
