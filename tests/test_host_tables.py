"""Host logic of the per-stream tables the native calls take (no GPU needed): segment maps for
the tile engine's launch pair and owner tables for last-writer-wins scatters — growth, epoch
sequence and wrap, and the cases that hand back None (stream capture, empty or oversized calls)."""

from __future__ import annotations

import torch

from musa_aiter import _native

CPU = torch.device("cpu")


def _no_capture(monkeypatch, capturing=False):
    monkeypatch.setattr(torch.cuda, "is_current_stream_capturing", lambda: capturing)


def test_seg_map_epochs_growth_and_wrap(monkeypatch):
    _no_capture(monkeypatch)
    stream = 0x5E6A
    _native._SEGMAPS.pop((CPU.index, stream), None)
    ptr0, cap0, e0 = _native.seg_map(CPU, stream, 100)
    assert ptr0 and cap0 >= 13 and e0 == 1
    ptr1, cap1, e1 = _native.seg_map(CPU, stream, 100)
    assert (ptr1, cap1, e1) == (ptr0, cap0, 2)  # same map, next epoch
    _, cap2, e2 = _native.seg_map(CPU, stream, 8 * cap0 + 1)  # needs more entries than the map has
    assert cap2 >= cap0 + 1 and e2 == 1  # a new map starts its own epoch sequence
    assert _native.seg_map(CPU, stream, 100)[1:] == (cap2, 2)
    ent = _native._SEGMAPS[(CPU.index, stream)]
    assert ent[0].numel() == cap2 and ent[0].dtype == torch.int32
    ent[3] = _native._SEG_EPOCH_MAX + 1  # epochs stay below 2^30: the next one starts again at 1
    assert _native.seg_map(CPU, stream, 100)[2] == 1
    _native._SEGMAPS.pop((CPU.index, stream), None)


def test_seg_map_declines_capture_empty_and_oversized(monkeypatch):
    _no_capture(monkeypatch)
    assert _native.seg_map(CPU, 7, 0) == (None, 0, 0)
    assert _native.seg_map(CPU, 7, 8 * _native._SEGMAP_MAX_ENTRIES + 8) == (None, 0, 0)
    _no_capture(monkeypatch, capturing=True)
    assert _native.seg_map(CPU, 7, 100) == (None, 0, 0)


def test_owner_table_epochs_growth_and_wrap(monkeypatch):
    _no_capture(monkeypatch)
    stream = 0x0A11
    _native._OWNERS.pop((CPU.index, stream), None)
    seen = []
    launch = lambda own, rows, epoch: seen.append((own, rows, epoch)) or 0  # noqa: E731
    assert _native.owned_scatter(CPU, stream, 1000, 10, launch) == 0
    assert _native.owned_scatter(CPU, stream, 1000, 10, launch) == 0
    assert seen[0][2] == 1 and seen[1][2] == 2 and seen[0][:2] == seen[1][:2]
    assert _native.owned_scatter(CPU, stream, seen[0][1] + 1, 10, launch) == 0  # grows: a new zeroed table
    assert seen[2][1] > seen[0][1] and seen[2][2] == 1
    ent = _native._OWNERS[(CPU.index, stream)]
    ent[0].fill_(123)
    ent[3] = _native._EPOCH_MAX + 1  # wrap: the table is cleared and epochs restart at 1
    assert _native.owned_scatter(CPU, stream, 10, 10, launch) == 0
    assert seen[3][2] == 1 and int(ent[0].abs().sum()) == 0
    _native._OWNERS.pop((CPU.index, stream), None)
    _no_capture(monkeypatch, capturing=True)
    assert _native.owned_scatter(CPU, stream, 10, 10, launch) is None
