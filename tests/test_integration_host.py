"""SGLang caller-side routes: gates, decisions and fallbacks (host logic, no GPU)."""

from __future__ import annotations

import types

import pytest
import torch

from musa_aiter import integration as I


def test_resolve_backend_decisions():
    assert I.resolve_hicache_io_backend_for_musa("mmap", is_musa=True, adapter_available=True, layout_supported=True).backend == "direct"
    d = I.resolve_hicache_io_backend_for_musa("direct", is_musa=True, adapter_available=True, layout_supported=True)
    assert (d.backend, d.use_musa_aiter_adapter) == ("direct", False)
    assert not I.resolve_hicache_io_backend_for_musa("kernel", is_musa=False, adapter_available=True, layout_supported=True).use_musa_aiter_adapter
    assert not I.resolve_hicache_io_backend_for_musa("kernel", is_musa=True, adapter_available=False, layout_supported=True).use_musa_aiter_adapter
    assert I.resolve_hicache_io_backend_for_musa("kernel", is_musa=True, adapter_available=True, layout_supported=True).use_musa_aiter_adapter


def test_routes_need_the_adapter_gate(monkeypatch):
    monkeypatch.delenv("MUSA_AITER_SGLANG_ADAPTER", raising=False)
    t = torch.zeros((8, 2, 4))
    idx = torch.arange(2)
    assert I.try_sglang_hicache_layout_transfer(t, t, t, t, idx, idx, source_layout="layer_first",
                                                destination_layout="layer_first") is False
    assert I.try_sglang_hicache_layer_first_transfer(t, t, t, t, idx, idx, page_size=4, direction="host_to_device") is False
    assert I.check_kv_copy_paged_blocks(t, t, t, t, torch.zeros((1, 2), dtype=torch.int64)).reason == \
        "MUSA_AITER_SGLANG_ADAPTER is not enabled"
    assert I.try_kv_load_and_reshape_flash(t, t, torch.zeros((1, 1), dtype=torch.int64), torch.ones(1, dtype=torch.int64)) is None


def test_decisions_with_the_gate_on(monkeypatch):
    monkeypatch.setenv("MUSA_AITER_SGLANG_ADAPTER", "1")
    t = torch.zeros((8, 2, 4))
    idx = torch.arange(2)
    # CPU tensors are not device tensors: routes decline instead of raising
    assert I.try_sglang_hicache_layout_transfer(t, t, t, t, idx, idx, source_layout="layer_first",
                                                destination_layout="layer_first") is False
    assert I.check_kv_copy_paged_blocks(t, t, t, t, torch.zeros((1, 2), dtype=torch.int64)).reason == \
        "all inputs must be MUSA tensors"
    assert I.try_sglang_hicache_layer_first_transfer(t, t, t, t, idx, idx, page_size=4, direction="sideways") is False
    # CPU-host routes need their own gate
    assert I.try_sglang_hicache_layer_first_cpu_host_transfer(t, t, t, t, idx, idx, page_size=4,
                                                              direction="host_to_device") is False
    monkeypatch.setenv("MUSA_AITER_NATIVE_CPU_HOST_KV_TRANSFER", "1")
    # host cache on CPU but device cache also on CPU -> declined with the reference's reason
    assert I.try_sglang_hicache_layer_first_cpu_host_transfer(t, t, t, t, idx, idx, page_size=4,
                                                              direction="host_to_device") is False


def test_flat_pool_decisions(monkeypatch):
    monkeypatch.setenv("MUSA_AITER_SGLANG_ADAPTER", "1")
    good = types.SimpleNamespace(layout="layer_first", kv_buffer=torch.zeros((2, 4, 16), dtype=torch.uint8))
    other = types.SimpleNamespace(layout="page_first", kv_buffer=torch.zeros((2, 4, 16), dtype=torch.uint8))
    wrong = types.SimpleNamespace(layout="layer_first", kv_buffer=torch.zeros((2, 4, 8), dtype=torch.uint8))
    idx = torch.arange(2)
    assert I.try_sglang_hicache_flat_paged_transfer(other, good, idx, idx, direction="load_to_device") is False
    assert I.try_sglang_hicache_flat_paged_transfer(good, wrong, idx, idx, direction="load_to_device") is False
    assert I.try_sglang_hicache_flat_paged_transfer(good, good, idx, idx, direction="nowhere") is False


def test_direct_transfer_rejects_unknown_mode(monkeypatch):
    monkeypatch.setenv("MUSA_AITER_SGLANG_ADAPTER", "1")
    t = torch.zeros(4)
    with pytest.raises(ValueError, match="unsupported SGLang direct mode"):
        I.try_sglang_hicache_direct_transfer([t], [t], torch.arange(1), torch.arange(1), 1, mode="sideways")
