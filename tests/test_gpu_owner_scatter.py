"""The two-launch scatter (``mak_rows_scatterv_owned``): last-writer resolution through a
per-stream owner table that persists across calls, tagged with a growing epoch.

Checked against the oracle: scatters with repeated slots into several caches that share
one table (entries left by earlier calls must never win), an epoch wrap (the table is
zeroed and the epochs restart), table growth for a larger destination, a second stream
(its own table), and CUDA graph capture (a captured epoch would be replayed, so capture
takes the workspace path)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import musa_aiter as ma
from musa_aiter import _native
from oracle import kv_oracle as O

from ._util import first_diff, same_bits, to_np

pytestmark = pytest.mark.gpu


def eq(got, want, what):
    assert same_bits(got, want), f"{what}: {first_diff(got, want)}"


def _case(g, nl, nb, bs, nh, hs, t, dup_every=5):
    mem = torch.randn((2, nl, t, nh * hs), generator=g).to(torch.bfloat16)
    slots = torch.randint(-1, nb * bs, (t,), generator=g, dtype=torch.int64)
    slots[::dup_every] = slots[1]  # many tokens fight for one slot; the last must win
    return mem, slots


def _scatter_and_check(mem, caches, ref, slots, what):
    assert ma.lmcache_kv_buffer_to_paged_two_x_nl(mem.cuda(), caches, slots.cuda(), 0, caches[0][0].shape[1],
                                                  caches[0][0].shape[2], caches[0][0].shape[3]) is True
    O.lmcache_two_x_nl_buffer_to_paged(to_np(mem), ref, slots.numpy())
    for kv in range(2):
        for layer in range(len(caches[0])):
            eq(caches[kv][layer], ref[kv][layer], f"{what} kv{kv} layer{layer}")


def _fresh(nl, nb, bs, nh, hs):
    dev = [[torch.zeros((nb, bs, nh, hs), dtype=torch.bfloat16, device="cuda") for _ in range(nl)] for _ in range(2)]
    ref = [[np.zeros((nb, bs, nh, hs), np.uint16) for _ in range(nl)] for _ in range(2)]
    return dev, ref


def test_shared_table_across_caches_and_calls(cuda_device):
    g = torch.Generator().manual_seed(21)
    geo = (2, 24, 16, 2, 32)
    a, ra = _fresh(*geo)
    b, rb = _fresh(*geo)
    for step in range(6):  # alternate caches; later calls reuse rows earlier calls owned
        mem, slots = _case(g, 2, 24, 16, 2, 32, 200)
        if step % 2:
            _scatter_and_check(mem, a, ra, slots, f"cache a, call {step}")
        else:
            _scatter_and_check(mem, b, rb, slots, f"cache b, call {step}")


def test_epoch_wrap_zeroes_the_table(cuda_device):
    g = torch.Generator().manual_seed(22)
    geo = (1, 16, 16, 2, 32)
    c, r = _fresh(*geo)
    mem, slots = _case(g, 1, 16, 16, 2, 32, 150)
    _scatter_and_check(mem, c, r, slots, "before the wrap")
    key = (torch.cuda.current_device(), _native.stream_ptr(torch.device("cuda")))
    ent = _native._OWNERS[key]
    ent[3] = _native._EPOCH_MAX - 1  # the next two calls use the last epochs, the third restarts at 1
    for step in range(3):
        mem, slots = _case(g, 1, 16, 16, 2, 32, 150)
        _scatter_and_check(mem, c, r, slots, f"wrap call {step}")
    assert ent[3] == 2


def test_table_grows_and_streams_are_separate(cuda_device):
    g = torch.Generator().manual_seed(23)
    small, rs = _fresh(1, 8, 16, 2, 32)
    mem, slots = _case(g, 1, 8, 16, 2, 32, 64)
    _scatter_and_check(mem, small, rs, slots, "small destination")
    rows = 1 << 17  # above the initial table size
    big, rbig = _fresh(1, rows // 16, 16, 1, 8)
    mem, slots = _case(g, 1, rows // 16, 16, 1, 8, 3000)
    _scatter_and_check(mem, big, rbig, slots, "grown table")
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        mem, slots = _case(g, 1, 8, 16, 2, 32, 64)
        _scatter_and_check(mem, small, rs, slots, "second stream")
    torch.cuda.synchronize()
    assert len({k for k in _native._OWNERS if k[0] == torch.cuda.current_device()}) >= 2
    mem, slots = _case(g, 1, 8, 16, 2, 32, 64)
    _scatter_and_check(mem, small, rs, slots, "default stream again")


def test_graph_capture_takes_the_workspace_path(cuda_device):
    g = torch.Generator().manual_seed(24)
    nl, nb, bs, nh, hs = 1, 16, 16, 2, 32
    caches, ref = _fresh(nl, nb, bs, nh, hs)
    mem, slots = _case(g, nl, nb, bs, nh, hs, 120)
    dmem, dslots = mem.cuda(), slots.cuda()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up outside capture
        ma.lmcache_kv_buffer_to_paged_two_x_nl(dmem, caches, dslots, 0, bs, nh, hs)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ma.lmcache_kv_buffer_to_paged_two_x_nl(dmem, caches, dslots, 0, bs, nh, hs)
    for step in range(3):
        new_mem, _ = _case(g, nl, nb, bs, nh, hs, 120)
        dmem.copy_(new_mem.cuda())
        # an eager scatter between replays moves the owner table's epochs past anything captured
        other, _ = _case(g, nl, nb, bs, nh, hs, 120)
        ma.lmcache_kv_buffer_to_paged_two_x_nl(other.cuda(), caches, dslots, 0, bs, nh, hs)
        O.lmcache_two_x_nl_buffer_to_paged(to_np(other), ref, slots.numpy())
        graph.replay()
        torch.cuda.synchronize()
        O.lmcache_two_x_nl_buffer_to_paged(to_np(new_mem), ref, slots.numpy())
        for kv in range(2):
            eq(caches[kv][0], ref[kv][0], f"graph replay {step} kv{kv}")
    del graph


def test_mla_pair_scatter_owner_path(cuda_device):
    g = torch.Generator().manual_seed(25)
    nl, nb, bs = 3, 20, 64
    kvc = torch.zeros((nl, nb, bs, 512), dtype=torch.bfloat16, device="cuda")
    pec = torch.zeros((nl, nb, bs, 64), dtype=torch.bfloat16, device="cuda")
    rkv = np.zeros((nl, nb * bs, 512), np.uint16)
    rpe = np.zeros((nl, nb * bs, 64), np.uint16)
    for step in range(4):
        t = 300
        kv = torch.randn((nl, t, 512), generator=g).to(torch.bfloat16)
        pe = torch.randn((nl, t, 64), generator=g).to(torch.bfloat16)
        slots = torch.randint(-1, nb * bs, (t,), generator=g)
        slots[::7] = slots[3]
        assert ma.kv_mla_linear_to_paged_multi_layer(kv.cuda(), pe.cuda(), kvc, pec, slots.cuda()) is True
        keep = O.last_writer_mask(slots.numpy())
        ok = keep & (slots.numpy() >= 0)
        rkv[:, slots.numpy()[ok]] = to_np(kv)[:, ok]
        rpe[:, slots.numpy()[ok]] = to_np(pe)[:, ok]
        eq(kvc.view(nl, nb * bs, 512), rkv, f"latent, call {step}")
        eq(pec.view(nl, nb * bs, 64), rpe, f"rope, call {step}")
