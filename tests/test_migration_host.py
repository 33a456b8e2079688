"""Host logic of the paged-block migration: layer ownership and argument agreement across
ranks (world_size 2 over gloo on CPU; no GPU needed)."""

from __future__ import annotations

import socket

import pytest
import torch.multiprocessing as mp

from musa_aiter.ops.kv_migration import layer_owners

from . import _mp_workers


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_layer_owners_split():
    assert layer_owners(61, list(range(1, 8))) == [1] * 9 + [2] * 9 + [3] * 9 + [4] * 9 + [5] * 9 + [6] * 8 + [7] * 8
    assert layer_owners(61, [1]) == [1] * 61
    assert layer_owners(3, [1, 2, 3, 4]) == [1, 2, 3]
    with pytest.raises(ValueError):
        layer_owners(4, [])


def test_bad_arguments_raise_on_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mp_workers.gloo_bad_arguments, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank in (0, 1):
        msg = results[rank]
        assert "rank 1 must pass layers [0, 1, 2]" in msg, msg
        assert "CUDA tensors" in msg, msg
