"""GPU parity for the grouped row entry points (``mak_rows_gatherv`` /
``mak_rows_scatterv``) and for the pointer-arithmetic plane descriptors the
LMCache / SGLang-MP / MLA forms use, including the layouts that fall back to the
per-plane path (non-uniform cache lists, padded memory tensors).  All
comparisons are bit-exact against the CPU oracle."""

from __future__ import annotations

import ctypes

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


def _side(planes: list[torch.Tensor], paged: bool):
    """(ptrs, rows_per_block, block_stride, row_stride, num_rows) of uint8 planes [NB, BS, W] or [T, W]."""
    p0 = planes[0]
    if paged:
        return [p.data_ptr() for p in planes], p0.shape[1], p0.stride(0), p0.stride(1), p0.shape[0] * p0.shape[1]
    return [p.data_ptr() for p in planes], 1, p0.stride(0), 0, p0.shape[0]


def test_rows_gatherv_scatterv_two_geometries(cuda_device):
    """Two plane groups with different widths, strides and row counts in one call."""
    g = torch.Generator().manual_seed(11)
    nb, bs = 8, 4
    # group 0: 3 planes, 40-byte rows in 48-byte slots; group 1: 2 planes, 24-byte rows, padded blocks
    big0 = torch.randint(0, 256, (3, nb, bs, 48), generator=g, dtype=torch.uint8)
    big1 = torch.randint(0, 256, (2, nb + 1, bs, 32), generator=g, dtype=torch.uint8)
    caches0 = [big0[i, :, :, :40] for i in range(3)]
    caches1 = [big1[i, :nb, :, :24] for i in range(2)]
    slots = torch.tensor([5, -1, 31, 0, 30, 7, 7, 12, 3, -4], dtype=torch.int64)
    t0, t1 = 12, 7  # group 1 buffer is shorter: its rows 7.. are outside its buffer
    big0d, big1d = big0.cuda(), big1.cuda()  # slice on the device so the planes keep their padded strides
    dev0 = [big0d[i, :, :, :40] for i in range(3)]
    dev1 = [big1d[i, :nb, :, :24] for i in range(2)]
    lin0 = torch.full((3, t0, 48), 0xAB, dtype=torch.uint8, device="cuda")
    lin1 = torch.full((2, t1, 24), 0xCD, dtype=torch.uint8, device="cuda")
    lib = _native.load()
    pd, pk = _native.rows_desc_array([_side(dev0, True), _side(dev1, True)])
    ld, lk = _native.rows_desc_array([_side([lin0[i, :, :40] for i in range(3)], False), _side(list(lin1.unbind(0)), False)])
    rb = (ctypes.c_int64 * 2)(40, 24)
    ks = slots.cuda()
    rc = lib.mak_rows_gatherv(pd, ld, 2, rb, 0, ctypes.c_void_p(ks.data_ptr()), 5, ks.numel(), 1,
                              _native.stream_ptr(ks.device))
    _native.check(rc, "gatherv")
    torch.cuda.synchronize()
    for i in range(3):
        want = np.full((t0, 48), 0xAB, np.uint8)
        want[:, :40] = O.rows_gather(caches0[i].contiguous().numpy().reshape(nb * bs, 40), slots.numpy(), t0)
        eq(lin0[i], want, f"group 0 plane {i}")
    for i in range(2):
        want = O.rows_gather(caches1[i].contiguous().numpy().reshape(nb * bs, 24), slots.numpy(), t1)
        eq(lin1[i], want, f"group 1 plane {i}")

    # scatter back with duplicates (last writer wins) and a skipped prefix of 1 row
    sslots = torch.tensor([9, 2, 9, 30, -1, 2], dtype=torch.int32)
    ref0 = [c.contiguous().numpy().reshape(nb * bs, 40).copy() for c in caches0]
    ref1 = [c.contiguous().numpy().reshape(nb * bs, 24).copy() for c in caches1]
    src0 = to_np(lin0[:, :, :40])
    src1 = to_np(lin1)
    # group 1 buffer has 7 rows: source rows 1..6 exist
    for i in range(3):
        O.rows_scatter(src0[i], ref0[i], sslots.numpy(), skip_prefix=1)
    for i in range(2):
        O.rows_scatter(src1[i], ref1[i], sslots.numpy(), skip_prefix=1)
    ks = sslots.cuda()
    ws, nbytes = _native.workspace(ks.numel(), ks.device)
    rc = lib.mak_rows_scatterv(ld, pd, 2, rb, 0, ctypes.c_void_p(ks.data_ptr()), 4, ks.numel(), 1,
                               ctypes.c_void_p(ws.data_ptr()), nbytes, _native.stream_ptr(ks.device))
    _native.check(rc, "scatterv")
    torch.cuda.synchronize()
    for i in range(3):
        eq(dev0[i].contiguous().view(nb * bs, 40), ref0[i], f"scatter group 0 plane {i}")
    for i in range(2):
        eq(dev1[i].contiguous().view(nb * bs, 24), ref1[i], f"scatter group 1 plane {i}")
    # bytes outside the rows are untouched
    assert torch.equal(big0d[:, :, :, 40:].cpu(), big0[:, :, :, 40:])
    assert torch.equal(big1d[:, nb:].cpu(), big1[:, nb:]) and torch.equal(big1d[..., 24:].cpu(), big1[..., 24:])


def test_rows_gatherv_rejects_bad_groups(cuda_device):
    lib = _native.load()
    t = torch.zeros((4, 16), dtype=torch.uint8, device="cuda")
    sides = [([t.data_ptr()], 1, 16, 0, 4)] * 5
    pd, pk = _native.rows_desc_array(sides)
    ld, lk = _native.rows_desc_array(sides)
    s = torch.zeros(2, dtype=torch.int64, device="cuda")
    rc = lib.mak_rows_gatherv(pd, ld, 5, None, 16, ctypes.c_void_p(s.data_ptr()), 5, 2, 1, _native.stream_ptr(s.device))
    assert rc != 0 and b"plane groups" in lib.mak_last_error()


def _rand(shape, g, dt=torch.bfloat16):
    return torch.randn(shape, generator=g).to(dt)


def test_two_x_nl_fallback_layouts_vs_oracle(cuda_device):
    """Non-uniform cache lists and padded memory tensors (per-plane path) and the fast path agree with the oracle."""
    g = torch.Generator().manual_seed(5)
    nl, nb, bs, nh, hs = 3, 16, 8, 2, 32
    slots = torch.randperm(nb * bs, generator=g)[:50].to(torch.int64)
    slots[7] = -1
    caches = [[_rand((nb, bs, nh, hs), g) for _ in range(nl)] for _ in range(2)]
    # one cache lives inside a wider allocation: its token rows are not contiguous -> per-plane path
    wide = _rand((nb, bs, nh, hs + 8), g)
    caches[1][2] = wide[..., :hs]
    dcaches = [[c.cuda() for c in kv] for kv in caches]
    dcaches[1][2] = wide.cuda()[..., :hs]
    assert not dcaches[1][2].is_contiguous()
    t = 64
    mem_big = torch.full((2, nl, t + 3, nh * hs + 16), 3.0, dtype=torch.bfloat16, device="cuda")
    mem = mem_big[:, :, :t, : nh * hs]  # padded in T and in the row: strided buffer, rows still contiguous
    assert ma.lmcache_kv_paged_to_buffer_two_x_nl(dcaches, mem, slots.cuda(), bs, nh, hs) is True
    ref = np.zeros((2, nl, t, nh * hs), np.uint16)
    O.lmcache_two_x_nl_paged_to_buffer([[to_np(c.contiguous()) for c in kv] for kv in caches], ref, slots.numpy())
    eq(mem, ref, "two_x_nl gather (mixed layouts)")
    assert torch.all(mem_big[:, :, t:] == 3.0) and torch.all(mem_big[..., nh * hs:] == 3.0)

    # uniform caches, strided memory tensor: fast path
    ucaches = [[c.contiguous().cuda() for c in kv] for kv in caches]
    mem2 = torch.zeros_like(mem_big)[:, :, :t, : nh * hs]
    assert ma.lmcache_kv_paged_to_buffer_two_x_nl(ucaches, mem2, slots.cuda(), bs, nh, hs) is True
    eq(mem2, ref, "two_x_nl gather (fast path, strided memory)")

    # scatter into fresh uniform caches from the strided memory tensor, skip 2 tokens
    sl = slots[:40].clone()
    fresh = [[torch.zeros((nb, bs, nh, hs), dtype=torch.bfloat16, device="cuda") for _ in range(nl)] for _ in range(2)]
    assert ma.lmcache_kv_buffer_to_paged_two_x_nl(mem, fresh, sl.cuda(), 2, bs, nh, hs) is True
    rc = [[np.zeros((nb, bs, nh, hs), np.uint16) for _ in range(nl)] for _ in range(2)]
    O.lmcache_two_x_nl_buffer_to_paged(ref, rc, sl.numpy(), skip_prefix=2)
    for kv in range(2):
        for layer in range(nl):
            eq(fresh[kv][layer], rc[kv][layer], f"two_x_nl scatter kv{kv} layer{layer}")


def test_layer_list_and_six_d_strided_vs_oracle(cuda_device):
    g = torch.Generator().manual_seed(8)
    nl, nb, bs, nh, hs = 2, 12, 4, 2, 16
    slots = torch.randint(-1, nb * bs, (32,), generator=g, dtype=torch.int64)
    six = _rand((nl, 2, nb, bs, nh, hs), g, torch.float16)
    buf_big = torch.full((2, nl, 33, nh * hs + 8), 1.0, dtype=torch.float16, device="cuda")
    buf = buf_big[:, :, :32, : nh * hs]
    assert ma.lmcache_paged_to_kv_buffer(six.cuda(), buf, slots.cuda()) is True
    ref = np.full((2, nl, 32, nh * hs), 7, np.float16)
    O.lmcache_paged_to_kv_buffer(six.numpy(), ref, slots.numpy())
    eq(buf, ref, "6-D gather into strided buffer")
    dst = torch.zeros_like(six).cuda()
    sl = torch.randint(0, nb * bs, (32,), generator=g, dtype=torch.int64)
    assert ma.lmcache_kv_buffer_to_paged(buf, dst, sl.cuda()) is True
    want = np.zeros_like(six.numpy())
    O.lmcache_kv_buffer_to_paged(ref, want, sl.numpy())
    eq(dst, want, "6-D scatter from strided buffer")

    lst = [_rand((2, nb, bs, nh, hs), g, torch.float32) for _ in range(nl)]
    mem = torch.empty((2, nl, 32, nh * hs), dtype=torch.float32, device="cuda")
    assert ma.lmcache_kv_paged_to_buffer([c.cuda() for c in lst], mem, slots.cuda(), bs, nh, hs) is True
    refm = np.zeros((2, nl, 32, nh * hs), np.float32)
    O.lmcache_list_paged_to_buffer([c.numpy() for c in lst], refm, slots.numpy())
    eq(mem, refm, "layer list gather")
    out = [torch.zeros((2, nb, bs, nh, hs), device="cuda") for _ in range(nl)]
    assert ma.lmcache_kv_buffer_to_paged(mem, out, sl[:20].cuda(), 3, bs, nh, hs) is True
    wl = [np.zeros((2, nb, bs, nh, hs), np.float32) for _ in range(nl)]
    O.lmcache_list_buffer_to_paged(refm, wl, sl[:20].numpy(), 3)
    for i in range(nl):
        eq(out[i], wl[i], f"layer list scatter {i}")


def test_mla_pair_one_launch_vs_oracle(cuda_device, monkeypatch):
    """Latent + rope caches move in one launch per direction (gather and scatter)."""
    monkeypatch.setenv("MUSA_AITER_SKIP_VALIDATION", "1")  # no slot-bound reduction launch
    g = torch.Generator().manual_seed(9)
    nl, nb, bs, kvd, ped = 3, 10, 16, 96, 16
    kvc = _rand((nl, nb, bs, kvd), g)
    pec = _rand((nl, nb, bs, ped), g)
    slots = torch.randint(-2, nb * bs, (70,), generator=g, dtype=torch.int64)
    dk, dp = kvc.cuda(), pec.cuda()
    n0 = _native.launch_count()
    okv, ope = ma.kv_paged_to_mla_linear_multi_layer(dk, dp, slots.cuda())
    assert _native.launch_count() - n0 == 1
    for layer in range(nl):
        rk, rp = O.kv_paged_to_mla_linear(to_np(kvc[layer]), to_np(pec[layer]), slots.numpy())
        eq(okv[layer], rk, f"mla gather kv {layer}")
        eq(ope[layer], rp, f"mla gather pe {layer}")
    sl = torch.randint(0, nb * bs, (70,), generator=g, dtype=torch.int64)
    sl[5] = sl[60]  # duplicate: the later row wins in both caches
    tk, tp = torch.zeros_like(dk), torch.zeros_like(dp)
    assert ma.kv_mla_linear_to_paged_multi_layer(okv, ope, tk, tp, sl.cuda()) is True
    for layer in range(nl):
        wk = np.zeros((nb, bs, kvd), np.uint16)
        wp = np.zeros((nb, bs, ped), np.uint16)
        O.kv_mla_linear_to_paged(to_np(okv[layer]), to_np(ope[layer]), wk, wp, sl.numpy())
        eq(tk[layer], wk, f"mla scatter kv {layer}")
        eq(tp[layer], wp, f"mla scatter pe {layer}")


@pytest.mark.parametrize("n", (1, 777, 12288, 12289, 40000))
@pytest.mark.parametrize("dt", (torch.int32, torch.int64))
def test_resolve_last_writer_both_paths(cuda_device, n, dt):
    """Last-writer resolution over sizes from one slot to several hash-table growths agrees with the oracle."""
    g = torch.Generator().manual_seed(n)
    slots = torch.randint(-3, max(2, n // 3), (n,), generator=g).to(dt)  # many duplicates and negatives
    d = slots.cuda()
    lib = _native.load()
    ws, nbytes = _native.workspace(n, d.device)
    eff = torch.empty(n, dtype=torch.int64, device="cuda")
    rc = lib.mak_resolve_last_writer(d.data_ptr(), _native.dtype_code(dt), n, eff.data_ptr(), ws.data_ptr(), nbytes,
                                     _native.stream_ptr(d.device))
    _native.check(rc, "resolve")
    keep = O.last_writer_mask(slots.numpy())
    want = np.where(keep, slots.numpy().astype(np.int64), -1)
    assert np.array_equal(eff.cpu().numpy(), want)
