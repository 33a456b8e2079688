"""Host-side API behaviour with CPU tensors: reference validation messages, and
no CPU fallback (CPU tensors are rejected once the arguments are valid)."""

from __future__ import annotations

import pytest
import torch

import musa_aiter as ma


def test_cpu_tensors_are_rejected_not_computed():
    kc = torch.zeros(2, 2, 4, 4)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ma.kv_paged_to_linear(kc, kc.clone(), torch.tensor([0, 1]))


def test_out_of_bounds_slot_message():
    # op_tests/test_kv_transfer.py:520-560: OOB slots raise ValueError before any data moves
    kc = torch.zeros(2, 2, 4, 4)
    with pytest.raises(ValueError, match="out of bounds"):
        ma.kv_paged_to_linear(kc, kc.clone(), torch.tensor([0, 8]))
    with pytest.raises(ValueError, match="out of bounds"):
        ma.kv_linear_to_paged_multi_layer(torch.zeros(1, 1, 2, 4), torch.zeros(1, 1, 2, 4), torch.zeros(1, 2, 2, 4, 4),
                                          torch.zeros(1, 2, 2, 4, 4), torch.tensor([8]))


def test_shape_and_dtype_messages():
    kc = torch.zeros(2, 2, 4, 4)
    with pytest.raises(ValueError, match="4-D"):
        ma.kv_paged_to_linear(torch.zeros(2, 2, 4), kc, torch.tensor([0]))
    with pytest.raises(ValueError, match="integer-valued"):
        ma.kv_paged_to_linear(kc, kc.clone(), torch.tensor([0.0]))
    with pytest.raises(ValueError, match="preserve requires"):
        ma.kv_paged_to_linear(kc, kc.clone(), torch.tensor([0]), fill_skipped="preserve")
    with pytest.raises(ValueError, match="unsupported FP8"):
        ma.kv_linear_to_paged_fp8(torch.zeros(1, 2, 4), torch.zeros(1, 2, 4), torch.zeros(2, 2, 4, 4, dtype=torch.uint8),
                                  torch.zeros(2, 2, 4, 4, dtype=torch.uint8), torch.tensor([0]), 1.0, 1.0, fp8_format="e3m4")
    with pytest.raises(ValueError, match="positive and finite"):
        ma.kv_linear_to_paged_fp8(torch.zeros(1, 2, 4), torch.zeros(1, 2, 4), torch.zeros(2, 2, 4, 4, dtype=torch.uint8),
                                  torch.zeros(2, 2, 4, 4, dtype=torch.uint8), torch.tensor([0]), 0.0, 1.0)
    # Python numbers are checked on the host, tensors through their values
    for bad in (float("nan"), float("inf"), -1.0, -2, torch.tensor(0.0), torch.tensor([1.0, float("nan")])):
        with pytest.raises(ValueError, match="positive and finite"):
            ma.kv_linear_to_paged_fp8(torch.zeros(1, 2, 4), torch.zeros(1, 2, 4), torch.zeros(2, 2, 4, 4, dtype=torch.uint8),
                                      torch.zeros(2, 2, 4, 4, dtype=torch.uint8), torch.tensor([0]), 1.0, bad)
    with pytest.raises(ValueError, match="FP8 cache storage"):
        ma.kv_linear_to_paged_fp8(torch.zeros(1, 2, 4), torch.zeros(1, 2, 4), torch.zeros(2, 2, 4, 4),
                                  torch.zeros(2, 2, 4, 4), torch.tensor([0]), 1.0, 1.0)


def test_lmcache_contract_messages():
    # op_tests/test_lmcache_kv_transfer.py:118-170, 278-295
    slots = torch.tensor([0, 8], dtype=torch.int32)
    with pytest.raises(ValueError, match="out of range"):
        ma.lmcache_kv_buffer_to_paged(torch.zeros(2, 1, 2, 4), torch.zeros(1, 2, 1, 4, 1, 4), slots)
    with pytest.raises(ValueError, match="rank"):
        ma.lmcache_kv_buffer_to_paged(torch.zeros(1, 2, 3), torch.zeros(1, 2, 1, 4, 1, 4), torch.tensor([0]))
    memory = torch.zeros(2, 2, 2, 4)
    mismatched = [[torch.zeros(1, 2, 1, 4), torch.zeros(1, 2, 1, 4)], [torch.zeros(1, 2, 1, 4)]]
    with pytest.raises(ValueError, match="layer"):
        ma.lmcache_kv_paged_to_buffer(mismatched, memory, torch.tensor([0, 1]), 2, 1, 4)
    valid = [[torch.zeros(1, 2, 1, 4) for _ in range(2)] for _ in range(2)]
    with pytest.raises(ValueError, match="int32 or int64"):
        ma.lmcache_kv_paged_to_buffer(valid, memory, torch.tensor([0.0, 1.0]), 2, 1, 4)
    with pytest.raises(ValueError, match="transfer range"):
        ma.lmcache_kv_buffer_to_paged_two_x_nl(memory, valid, torch.tensor([0, 1]), 1, 2, 1, 4)
    with pytest.raises(TypeError):
        ma.lmcache_kv_buffer_to_paged(memory, [torch.zeros(2, 1, 2, 1, 4)], torch.tensor([0, 1]))


def test_dispatch_trace_line(monkeypatch, capsys):
    from musa_aiter import dispatch

    monkeypatch.setenv("MUSA_AITER_TRACE_DISPATCH", "1")
    dispatch.emit_native("kv_paged_to_linear", torch.zeros(1), "unit test")
    err = capsys.readouterr().err
    assert "[MUSA_AITER DISPATCH] op=kv_paged_to_linear backend=cuda-sm100a" in err


def test_flash_cache_back_checks_in_sequence_order():
    """kv_reshape_and_cache_back_flash raises the reference's error of the first offending
    sequence: length outside [0, S], too few block-table columns, or an invalid block id."""
    kc = torch.zeros((8, 2, 4, 4))
    vc = torch.zeros_like(kc)
    dk = torch.zeros((3, 10, 2, 4))
    dv = torch.zeros_like(dk)
    bt = torch.tensor([[0, 1, 2], [3, 4, 5], [6, 7, 0]])
    name = "kv_reshape_and_cache_back_flash"
    cases = [
        (torch.tensor([4, 11, 4]), bt, "seq_lens exceeds dense sequence length"),
        (torch.tensor([4, -1, 4]), bt, "seq_lens exceeds dense sequence length"),
        (torch.tensor([4, 4, 10]), bt[:, :2], "block_tables does not contain enough columns"),
        (torch.tensor([4, 9, 11]), torch.tensor([[0, 1, 2], [3, 9, 5], [6, 7, 0]]), "invalid block id 9"),
        (torch.tensor([4, 3, 9]), torch.tensor([[0, 1, 2], [3, -2, 5], [6, 7, 8]]), "invalid block id 8"),
    ]
    for lens, table, msg in cases:
        with pytest.raises(ValueError, match=f"{name}: {msg}"):
            ma.kv_reshape_and_cache_back_flash(dk, dv, kc, vc, table, lens)
    # the block -2 of sequence 1 lies past that sequence's blocks, so it is not checked: only the
    # device requirement remains
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ma.kv_reshape_and_cache_back_flash(dk, dv, kc, vc, torch.tensor([[0, 1, 2], [3, -2, 5], [6, 7, 0]]),
                                           torch.tensor([4, 3, 9]))
