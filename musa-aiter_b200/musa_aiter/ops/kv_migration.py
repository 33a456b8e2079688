"""Paged-block migration between the GPUs of one node.

A prefill rank holds every layer of a request's KV cache; each layer has an
owner rank that will decode with it.  The migration moves the request's blocks
of every layer to its owner, where they land at blocks the owner allocated
(its own block table).  There is no reference API for this step: the
reference's communication layer raises for ``world_size != 1``
(musa_aiter/communication.py:55-56); correctness follows the block-copy
semantics of ``kv_copy_paged_blocks`` (musa_aiter/ops/kv_transfer.py:2081-2091):
after the call, ``owner_cache[dst_blocks[i]] == prefill_cache[src_blocks[i]]``
byte for byte, for every layer.

Data path: no staging and no library collective for the payload.  Each owner
exports its cache allocations once as CUDA IPC handles
(``mak_ipc_export``); the prefill rank maps them (``mak_ipc_import``) and
moves every block of every layer with ONE row-engine launch per owner
(``mak_rows_copy``: a block is one row, the source index is the prefill block
table, the destination index the owner's), so the gather from scattered blocks
and the NVLink transfer are the same 16-byte stores, and the owner does no work.
Only the per-migration block tables travel through a collective
(``all_gather_into_tensor``, on the device), plus one barrier that publishes
completion.  Plain peer stores only, no waits inside kernels.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from .. import _native
from ..dispatch import emit_native

__all__ = ["layer_owners", "PagedBlockMigration"]


def layer_owners(num_layers: int, receivers: list[int]) -> list[int]:
    """Owner rank of each layer: contiguous runs, the first ``num_layers % R`` receivers get one more
    layer (61 layers over ranks 1-7 -> 9,9,9,9,9,8,8)."""
    if num_layers < 0 or not receivers:
        raise ValueError("layer_owners: need a non-negative layer count and at least one receiver")
    r = len(receivers)
    base, extra = divmod(num_layers, r)
    owners: list[int] = []
    for k, rank in enumerate(receivers):
        owners += [rank] * (base + (1 if k < extra else 0))
    return owners


def _block_geometry(cache: torch.Tensor, name: str) -> tuple[int, int, int]:
    """(num_blocks, block_stride_bytes, block_bytes) of a cache whose leading dim is the block id
    and whose blocks are contiguous byte ranges."""
    if cache.dim() < 1 or cache.shape[0] == 0:
        raise ValueError(f"{name}: caches must be [num_blocks, ...] with num_blocks > 0")
    e = cache.element_size()
    inner = cache[0]
    if not inner.is_contiguous():
        raise ValueError(f"{name}: each block must be one contiguous byte range")
    return int(cache.shape[0]), int(cache.stride(0)) * e, int(inner.numel()) * e


@dataclass
class _Remote:
    rank: int
    layers: list[int]
    ptrs: list[int]
    handles: list[bytes]
    num_blocks: int
    block_stride: int


class PagedBlockMigration:
    """Set up once per set of caches (collective over ``group``), then ``run`` per migration.

    ``layer_caches`` maps layer index -> cache tensor on this rank: on ``src_rank`` every layer
    ``0 .. len(owners)-1``; on a receiver exactly the layers ``owners`` assigns to it; other ranks
    pass ``{}``.  Caches are ``[num_blocks, ...]`` with contiguous blocks and the same block size in
    bytes on every rank (the block count may differ).
    """

    def __init__(self, layer_caches: dict[int, torch.Tensor], owners: list[int], *, src_rank: int = 0,
                 group: dist.ProcessGroup | None = None) -> None:
        name = "PagedBlockMigration"
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.src_rank = src_rank
        self.owners = list(owners)
        self.layer_caches = dict(layer_caches)
        self.device: torch.device | None = None
        self.remotes: list[_Remote] = []
        self._closed = True
        # Every rank checks its own arguments, then all ranks learn every verdict in the same
        # collective that carries the handles: a bad argument on one rank raises on all of them
        # instead of leaving the others waiting in a collective.
        problem = None
        info = None
        try:
            info = self._local_setup(name)
        except Exception as exc:  # reported to every rank below, then raised everywhere
            problem = f"{type(exc).__name__}: {exc}"
        gathered: list = [None] * self.world
        dist.all_gather_object(gathered, {"problem": problem, "info": info}, group=group)
        problems = [f"rank {r}: {g['problem']}" for r, g in enumerate(gathered) if g["problem"]]
        if problems:
            raise ValueError(f"{name}: " + "; ".join(problems))
        if self.rank == src_rank:
            lib = _native.load()
            for r, g in enumerate(gathered):
                rinfo = g["info"]
                if r == src_rank or rinfo is None or not rinfo["planes"]:
                    continue
                if rinfo["block_bytes"] != self.block_bytes:
                    self._release_imports()
                    raise ValueError(f"{name}: rank {r} caches hold {rinfo['block_bytes']}-byte blocks, "
                                     f"the prefill rank {self.block_bytes}")
                ptrs, handles = [], []
                for h, off in rinfo["planes"]:
                    p = ctypes.c_void_p()
                    _native.check(lib.mak_ipc_import(h, off, ctypes.byref(p)), name)
                    ptrs.append(int(p.value))
                    handles.append(h)
                self.remotes.append(_Remote(r, rinfo["layers"], ptrs, handles, rinfo["nb"], rinfo["stride"]))
        self._closed = False

    def _local_setup(self, name: str) -> dict | None:
        """Validate this rank's caches; on an owner, export them.  Raises ValueError."""
        if self.src_rank in self.owners:
            raise ValueError("the prefill rank cannot own a layer")
        mine = sorted(self.layer_caches)
        if self.rank == self.src_rank:
            expect = list(range(len(self.owners)))
        else:
            expect = [l for l, o in enumerate(self.owners) if o == self.rank]
        if mine != expect:
            raise ValueError(f"rank {self.rank} must pass layers {expect}, got {mine}")
        geo = {l: _block_geometry(c, name) for l, c in self.layer_caches.items()}
        if len({g for g in geo.values()}) > 1:
            raise ValueError("the caches of one rank must share block count, stride and block size")
        if any(c.device.type != "cuda" for c in self.layer_caches.values()):
            raise ValueError("caches must be CUDA tensors (there is no CPU path)")
        self.device = next(iter(self.layer_caches.values())).device if self.layer_caches else None
        if not self.layer_caches:
            return None
        nb, stride, bbytes = next(iter(geo.values()))
        if self.rank == self.src_rank:
            self.src_nb, self.src_stride, self.block_bytes = nb, stride, bbytes
            return None
        lib = _native.load()
        hbytes = int(lib.mak_ipc_handle_bytes())
        info = {"layers": mine, "nb": nb, "stride": stride, "block_bytes": bbytes, "planes": []}
        for l in mine:
            h = ctypes.create_string_buffer(hbytes)
            off = ctypes.c_int64(0)
            _native.check(lib.mak_ipc_export(self.layer_caches[l].data_ptr(), h, ctypes.byref(off)), name)
            info["planes"].append((h.raw, int(off.value)))
        return info

    def _release_imports(self) -> None:
        lib = _native.load()
        for rem in self.remotes:
            for h in rem.handles:
                lib.mak_ipc_release(h)
        self.remotes = []

    def run(self, block_ids: torch.Tensor) -> int:
        """One migration (collective).  ``block_ids`` (int64, device, same length on every rank): the
        source blocks in order on the prefill rank, the destination blocks on a receiver (any value on
        other ranks).  Returns the bytes this rank moved (prefill) or received (owners)."""
        name = "PagedBlockMigration.run"
        if self._closed:
            raise RuntimeError(f"{name}: migration already closed")
        device = self.device if self.device is not None else torch.device("cuda", torch.cuda.current_device())
        ids = block_ids.to(device=device, dtype=torch.int64).contiguous()
        table = torch.empty((self.world, ids.numel()), dtype=torch.int64, device=device)
        dist.all_gather_into_tensor(table, ids, group=self.group)
        moved = 0
        if self.rank == self.src_rank:
            lib = _native.load()
            stream = _native.stream_ptr(self.device)
            src_ids = table[self.src_rank]
            n = int(ids.numel())
            ws, nbytes = _native.workspace(n, self.device)
            for rem in self.remotes:
                src_ptrs = [self.layer_caches[l].data_ptr() for l in rem.layers]
                buf = _native.rows_pack((src_ptrs, 1, self.src_stride, 0, self.src_nb),
                                        (rem.ptrs, 1, rem.block_stride, 0, rem.num_blocks))
                base = ctypes.addressof(buf)
                dst_ids = table[rem.rank]
                _native.check(lib.mak_rows_copy(base, base + 48, None, self.block_bytes, src_ids.data_ptr(),
                                                _native.MAK_DT_I64, dst_ids.data_ptr(), _native.MAK_DT_I64, n,
                                                ws.data_ptr(), nbytes, stream), name)
                moved += n * len(rem.layers) * self.block_bytes
            # The owners read their caches after this barrier: finish the peer stores first.
            torch.cuda.current_stream(self.device).synchronize()
            emit_native("kv_migrate_paged_blocks", ids, "sm100a row copy into peer memory (IPC, NVLink)")
        else:
            moved = int(ids.numel()) * len(self.layer_caches) * (
                _block_geometry(next(iter(self.layer_caches.values())), name)[2] if self.layer_caches else 0)
        dist.barrier(group=self.group)
        return moved

    def close(self) -> None:
        """Collective: the prefill rank unmaps the owners' caches before anyone frees them."""
        if self._closed:
            return
        if self.rank == self.src_rank:
            self._release_imports()
        self._closed = True
        dist.barrier(group=self.group)
