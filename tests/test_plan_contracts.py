"""Host-side contracts of the plan builder and layout descriptors (no GPU).

Follows the reference's contract tests (op_tests/test_kv_layout_contract.py,
test_kv_transfer_plan.py, test_kv_backend.py, test_lmcache_format_matrix.py,
test_lmcache_musa_batch_copy.py:75-189) case by case, plus this backend's
run planner."""

from __future__ import annotations

import pytest
import torch

import musa_aiter as ma
from musa_aiter.ops.kv_backend import KVBackend, KVBackendCapabilities, KVBackendDecision, select_kv_backend
from musa_aiter.ops.kv_layout import KVLayoutKind, KVLayoutSpec, KVOrganization, KVScaleKind
from musa_aiter.ops.kv_transfer_plan import (
    KVTransferEntry,
    KVTransferPlan,
    assess_direct_eligibility,
    build_transfer_plan,
    plan_slot_runs,
    validate_transfer_plan,
)
from musa_aiter.ops.lmcache_format import LMCacheFormat, describe_lmcache_format, describe_sglang_split_list
from musa_aiter.ops.lmcache_musa_batch_copy_plan import build_batch_copy_plan, chunk_batch_copy_plan


def paged(**kw):
    base = dict(num_layers=1, num_blocks=4, block_size=16, num_heads=2, head_size=8, dtype_name="float16",
                row_bytes=32, block_stride_bytes=512)
    base.update(kw)
    return KVLayoutSpec.standard_paged(**base)


def linear(**kw):
    base = dict(num_layers=1, num_tokens=32, num_heads=2, head_size=8, dtype_name="float16")
    base.update(kw)
    return KVLayoutSpec.linear(**base)


def test_layout_spec_facts_and_rejections():
    s = paged(num_layers=2, num_heads=8, head_size=64, row_bytes=128, block_stride_bytes=2048)
    assert s.kind is KVLayoutKind.STANDARD_PAGED and s.organization is KVOrganization.SEPARATE
    assert s.hidden_size == 512 and s.is_paged
    with pytest.raises(ValueError, match="row_bytes"):
        paged(row_bytes=0)
    with pytest.raises(ValueError, match="block_stride_bytes"):
        paged(row_bytes=32, block_stride_bytes=16)
    with pytest.raises(ValueError, match="scale_bytes"):
        KVLayoutSpec.dsv4(num_layers=1, num_blocks=4, block_size=16, row_bytes=132, block_stride_bytes=8640,
                          dtype_name="uint8", scale_kind=KVScaleKind.BLOCKED, value_bytes=128, scale_bytes=0)
    pf = KVLayoutSpec.page_first(num_layers=2, num_blocks=8, block_size=16, num_heads=4, head_size=32,
                                 dtype_name="bfloat16", row_bytes=64, block_stride_bytes=1024)
    assert pf.kind is KVLayoutKind.PAGE_FIRST and not pf.is_contiguous and pf.requires_layout_transform
    d = KVLayoutSpec.dsv4(num_layers=1, num_blocks=8, block_size=64, row_bytes=132, block_stride_bytes=8640,
                          dtype_name="uint8", scale_kind=KVScaleKind.BLOCKED, value_bytes=128, scale_bytes=4)
    f = d.format_facts()
    assert d.kind is KVLayoutKind.DSV4_BLOCKED_SCALE and f.value_bytes == 128 and f.scale_bytes == 4 and f.requires_transform
    assert ma.KVLayoutSpec is KVLayoutSpec and ma.KVLayoutKind is KVLayoutKind


def test_transfer_plan_validation_and_direct_eligibility():
    plan = KVTransferPlan(paged(), linear(), "d2h", 32, 0, (KVTransferEntry(0, 0, 64), KVTransferEntry(64, 64, 64)),
                          None, True, None)
    assert validate_transfer_plan(plan) is plan
    bad = KVTransferPlan(paged(), linear(), "d2h", 32, 0, (KVTransferEntry(0, 0, 64), KVTransferEntry(0, 32, 64)),
                         None, True, None)
    with pytest.raises(ValueError, match="overlap"):
        validate_transfer_plan(bad)
    with pytest.raises(ValueError, match="skip_prefix"):
        validate_transfer_plan(KVTransferPlan(paged(), linear(), "d2h", 4, 5, (), None, True, None))
    pf = KVLayoutSpec.page_first(num_layers=1, num_blocks=4, block_size=16, num_heads=2, head_size=8,
                                 dtype_name="float16", row_bytes=32, block_stride_bytes=512)
    ok, why = assess_direct_eligibility(pf, linear())
    assert not ok and "transform" in why
    assert assess_direct_eligibility(paged(), linear()) == (True, None)


def test_backend_selection_rules():
    plan = KVTransferPlan(linear(num_tokens=4), linear(num_tokens=4), "d2d", 4, 0, (KVTransferEntry(0, 0, 16),), None,
                          True, None)
    d = select_kv_backend(plan, capabilities=KVBackendCapabilities(True, True, True, True))
    assert d == KVBackendDecision(KVBackend.SPECIALIZED_NATIVE, True, "exact specialized native capability is available", False)
    assert select_kv_backend(plan, capabilities=KVBackendCapabilities(direct_batch=True)).backend is KVBackend.DIRECT_BATCH
    nd = KVTransferPlan(plan.source, plan.destination, "d2d", 4, 0, plan.entries, None, False, "layout transform is required")
    r = select_kv_backend(nd, capabilities=KVBackendCapabilities(direct_batch=True, reference=True))
    assert r.backend is KVBackend.REFERENCE and "layout transform is required" in r.reason
    rej = select_kv_backend(plan, capabilities=KVBackendCapabilities(reference=True), require_native=True)
    assert rej.backend is KVBackend.REJECTED and not rej.accepted


def test_lmcache_format_descriptions():
    f = describe_lmcache_format(torch.zeros(2, 3, 5, 16))
    assert f.format is LMCacheFormat.KV_2LTD and f.spec.num_layers == 3 and f.spec.num_tokens == 5
    assert describe_lmcache_format(torch.zeros(7, 2, 16)).format is LMCacheFormat.KV_T2D
    assert describe_lmcache_format(torch.zeros(2, 7, 16)).format is LMCacheFormat.KV_2TD
    with pytest.raises(ValueError, match="ambiguous"):
        describe_lmcache_format(torch.zeros(2, 2, 16))
    with pytest.raises(ValueError, match="rank"):
        describe_lmcache_format(torch.zeros(16))
    split = describe_sglang_split_list([[torch.zeros(4, 16, 2, 8)] * 3, [torch.zeros(4, 16, 2, 8)] * 3])
    assert split.format is LMCacheFormat.SGLANG_SPLIT_LIST
    assert split.spec.num_layers == 3 and split.spec.pointer_table_length == 6 and split.spec.row_bytes == 64
    with pytest.raises(ValueError, match="non-empty"):
        describe_sglang_split_list([[], []])


def test_slot_run_planner_and_byte_plan():
    slots = torch.tensor([16, 17, 18, 19, -1, 5, 6, 40, 41, 42, 43, 44, 45, 46, 47, 48])
    assert plan_slot_runs(slots) == [(0, 16, 4), (5, 5, 2), (7, 40, 9)]
    p = build_transfer_plan(paged(num_blocks=8), linear(num_tokens=16), slots, direction="d2d")
    validate_transfer_plan(p)
    # run (7, 40, 9) crosses a block at slot 48 -> split into 8 + 1 rows
    sizes = [e.nbytes for e in p.entries]
    assert sizes == [4 * 32, 2 * 32, 8 * 32, 1 * 32]
    assert p.entries[3].src_offset_bytes == 3 * 512 and p.entries[3].dst_offset_bytes == 15 * 32


def test_batch_copy_plan_contract():
    plan = build_batch_copy_plan(direction="h2d", sizes=[100, 10], source_capacities=[100, 50],
                                 destination_capacities=[200, 10], source_offsets=[0, 40],
                                 host_registration_offsets=[60, 0], pin_chunk_size=64)
    assert [(e.input_index, e.source_offset, e.size) for e in plan.entries] == [(0, 0, 4), (0, 4, 64), (0, 68, 32), (1, 40, 10)]
    assert plan.total_bytes == 110
    for kwargs, msg in [
        (dict(direction="d2d"), "direction"),
        (dict(sizes=[0]), "positive"),
        (dict(source_offsets=[-1]), "non-negative"),
        (dict(destination_capacities=[5]), "destination range"),
        (dict(source_capacities=[5]), "source range"),
        (dict(pin_chunk_size=0), "pin_chunk_size"),
    ]:
        base = dict(direction="h2d", sizes=[8], source_capacities=[8], destination_capacities=[8])
        base.update(kwargs)
        with pytest.raises(ValueError, match=msg):
            build_batch_copy_plan(**base)
    with pytest.raises(ValueError, match="overlapping"):
        build_batch_copy_plan(direction="h2d", sizes=[8, 8], source_capacities=[16, 16], destination_capacities=[16, 16],
                              destination_offsets=[0, 4], destination_keys=["a", "a"])
    chunks = chunk_batch_copy_plan(plan, 3)
    assert [len(c) for c in chunks] == [3, 1] and chunks[0][0] == plan.entries[0]
    with pytest.raises(ValueError, match="max_batch_entries"):
        chunk_batch_copy_plan(plan, 0)


def test_batch_copy_api_host_rules():
    assert ma.lmcache_musa_memcpy_batch_async([], [], []) is True
    # host <-> host is not a pairing this path serves: the caller keeps its own path
    assert ma.lmcache_musa_memcpy_batch_async([torch.zeros(4)], [torch.ones(4)], [16]) is False
    with pytest.raises(ValueError, match="same length"):
        ma.lmcache_musa_memcpy_batch_async([torch.zeros(4)], [], [16])
    with pytest.raises(TypeError):
        ma.lmcache_musa_memcpy_batch_async([1], [2], [3])
    with pytest.raises(ValueError, match="boundary"):
        from musa_aiter.ops.lmcache_musa_batch_copy import lmcache_musa_memcpy_batch_async_internal

        lmcache_musa_memcpy_batch_async_internal([], [], [], host_registration_offsets=None, pin_chunk_size=None)
    assert ma.native_lmcache_musa_batch_copy_abi_version() == 1
