"""Paged-block migration between two GPUs (NCCL for the block tables, the row engine's peer
stores for the payload): the owner's blocks equal the prefill rank's blocks byte for byte, and
untouched blocks keep their contents.  Needs 2 GPUs; skipped otherwise."""

from __future__ import annotations

import socket

import pytest
import torch
import torch.multiprocessing as mp

from . import _mp_workers

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_migration():
    world = min(torch.cuda.device_count(), 4)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_mp_workers.nccl_migration, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, ok, moved = q.get(timeout=300)
        results[rank] = (ok, moved)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(ok for ok, _ in results.values()), results
    assert results[0][1] == sum(m for r, (_, m) in results.items() if r != 0)
