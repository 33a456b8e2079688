"""Worker functions for the multi-process tests (importable by spawned children)."""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def _init(rank: int, world: int, port: int, backend: str, device=None) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    kw = {"device_id": device} if device is not None else {}
    dist.init_process_group(backend, rank=rank, world_size=world, timeout=timedelta(seconds=60), **kw)


def gloo_bad_arguments(rank: int, world: int, port: int, q) -> None:
    """Rank 0 passes CPU caches, rank 1 the wrong layers: every rank must raise, none may hang."""
    from musa_aiter.ops.kv_migration import PagedBlockMigration, layer_owners

    _init(rank, world, port, "gloo")
    try:
        owners = layer_owners(3, [1])
        caches = {l: torch.zeros((4, 16), dtype=torch.uint8) for l in range(3)} if rank == 0 else \
            {0: torch.zeros((4, 16), dtype=torch.uint8)}
        try:
            PagedBlockMigration(caches, owners)
            q.put((rank, "no error"))
        except ValueError as exc:
            q.put((rank, str(exc)))
    finally:
        dist.destroy_process_group()


def _pattern(layer: int, blocks: torch.Tensor, row: int) -> torch.Tensor:
    j = torch.arange(row, device=blocks.device)
    return ((layer * 131 + blocks[:, None] * 7 + j[None, :] * 3) % 251).to(torch.uint8)


def nccl_migration(rank: int, world: int, port: int, q) -> None:
    """Prefill rank 0 holds 5 layers; ranks 1.. own them; two migrations with different block tables."""
    from musa_aiter.ops.kv_migration import PagedBlockMigration, layer_owners

    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    _init(rank, world, port, "nccl", dev)
    try:
        nl, nb_src, nb_dst, bs, tok = 5, 96, 128, 16, 72
        row = bs * tok
        owners = layer_owners(nl, list(range(1, world)))
        if rank == 0:
            caches = {l: _pattern(l, torch.arange(nb_src, device=dev), row).view(nb_src, bs, tok) for l in range(nl)}
        else:
            caches = {l: torch.full((nb_dst, bs, tok), 0xAA, dtype=torch.uint8, device=dev)
                      for l in range(nl) if owners[l] == rank}
        mig = PagedBlockMigration(caches, owners)
        ok = True
        moved_total = 0
        for trial in range(2):
            n = 40 + 10 * trial
            g_src = torch.Generator().manual_seed(11 + trial)
            src_ids = torch.randperm(nb_src, generator=g_src)[:n]
            g_dst = torch.Generator().manual_seed(100 * rank + trial)
            dst_ids = torch.randperm(nb_dst, generator=g_dst)[:n]
            ids = src_ids if rank == 0 else dst_ids
            moved_total += mig.run(ids.to(dev))
            if rank != 0:
                for l, c in caches.items():
                    got = c.view(nb_dst, row)[dst_ids.to(dev)]
                    want = _pattern(l, src_ids.to(dev), row)
                    ok = ok and bool(torch.equal(got, want))
        if rank != 0:
            touched = torch.zeros(nb_dst, dtype=torch.bool)
            for trial in range(2):
                touched[torch.randperm(nb_dst, generator=torch.Generator().manual_seed(100 * rank + trial))[:40 + 10 * trial]] = True
            for c in caches.values():
                ok = ok and bool(torch.all(c.view(nb_dst, row)[(~touched).to(dev)] == 0xAA))
        mig.close()
        q.put((rank, ok, moved_total))
    finally:
        dist.destroy_process_group()
