"""GPU runs of the SGLang caller-side routes: layer-first token-row transfers (device caches,
pinned and pageable host caches, single and multi layer), DSV4 flat pools, block copies, and the
layout-exact HiCache route, each checked byte for byte against a plain restatement of the
reference's semantics (gather with zero rows for negative sources, scatter skipping negative
destinations, last writer wins)."""

from __future__ import annotations

import types

import numpy as np
import pytest
import torch

from musa_aiter import integration as I
from oracle import kv_oracle as O

from ._util import same_bits, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gates(monkeypatch):
    monkeypatch.setenv("MUSA_AITER_SGLANG_ADAPTER", "1")
    monkeypatch.setenv("MUSA_AITER_NATIVE_CPU_HOST_KV_TRANSFER", "1")


def _expect(src: np.ndarray, dst: np.ndarray, sidx, didx) -> np.ndarray:
    out = dst.copy()
    sidx = np.asarray(sidx, dtype=np.int64)
    didx = np.asarray(didx, dtype=np.int64)
    rows = np.zeros((len(sidx),) + src.shape[1:], dtype=src.dtype)
    ok = sidx >= 0
    rows[ok] = src[sidx[ok]]
    keep = O.last_writer_mask(didx)
    out[didx[keep]] = rows[keep]
    return out


def _case(seed, ts=64, td=96, n=40):
    g = torch.Generator().manual_seed(seed)
    src = torch.randn((ts, 4, 32), generator=g).to(torch.bfloat16)
    dst = torch.randn((td, 4, 32), generator=g).to(torch.bfloat16)
    sidx = torch.randint(-1, ts, (n,), generator=g)
    didx = torch.randint(-1, td, (n,), generator=g)
    didx[3] = didx[30]
    return src, dst, sidx, didx


@pytest.mark.parametrize("direction", ("host_to_device", "device_to_host"))
def test_layer_first_device_caches(cuda_device, direction):
    hk, dk, hidx, didx = _case(1)
    hv, dv, _, _ = _case(2)
    hk_d, hv_d, dk_d, dv_d = hk.cuda(), hv.cuda(), dk.cuda(), dv.cuda()
    assert I.try_sglang_hicache_layer_first_transfer(hk_d, hv_d, dk_d, dv_d, hidx.cuda(), didx.cuda(), page_size=16,
                                                     direction=direction)
    torch.cuda.synchronize()
    if direction == "host_to_device":
        assert same_bits(dk_d, _expect(to_np(hk), to_np(dk), hidx, didx))
        assert same_bits(dv_d, _expect(to_np(hv), to_np(dv), hidx, didx))
    else:
        assert same_bits(hk_d, _expect(to_np(dk), to_np(hk), didx, hidx))
        assert same_bits(hv_d, _expect(to_np(dv), to_np(hv), didx, hidx))


@pytest.mark.parametrize("pinned", (True, False))
@pytest.mark.parametrize("direction", ("host_to_device", "device_to_host"))
def test_layer_first_cpu_host(cuda_device, direction, pinned):
    hk, dk, hidx, didx = _case(3)
    hv, dv, _, _ = _case(4)
    hidx[hidx < 0] = 0  # the reference's CPU index ops take no negative host rows
    if pinned:
        hk, hv = hk.pin_memory(), hv.pin_memory()
    hk0, hv0 = hk.clone(), hv.clone()
    dk_d, dv_d = dk.cuda(), dv.cuda()
    assert I.try_sglang_hicache_layer_first_cpu_host_transfer(hk, hv, dk_d, dv_d, hidx, didx.cuda(), page_size=16,
                                                              direction=direction)
    torch.cuda.synchronize()
    if direction == "host_to_device":
        assert same_bits(dk_d, _expect(to_np(hk0), to_np(dk), hidx, didx))
        assert same_bits(dv_d, _expect(to_np(hv0), to_np(dv), hidx, didx))
    else:
        assert same_bits(hk, _expect(to_np(dk), to_np(hk0), didx, hidx))
        assert same_bits(hv, _expect(to_np(dv), to_np(hv0), didx, hidx))


def test_layer_first_cpu_host_multi_layer(cuda_device):
    g = torch.Generator().manual_seed(5)
    hk = torch.randn((3, 64, 2, 16), generator=g).half().pin_memory()
    hv = torch.randn((3, 64, 2, 16), generator=g).half().pin_memory()
    dk = torch.zeros((3, 80, 2, 16), dtype=torch.float16, device="cuda")
    dv = torch.zeros_like(dk)
    hidx = torch.randperm(64, generator=g)[:20]
    didx = torch.randperm(80, generator=g)[:20]
    assert I.try_sglang_hicache_layer_first_cpu_host_transfer_multi_layer(hk, hv, dk, dv, hidx, didx.cuda(),
                                                                          page_size=16, direction="host_to_device")
    torch.cuda.synchronize()
    for l in range(3):
        assert same_bits(dk[l], _expect(to_np(hk[l]), np.zeros((80, 2, 16), np.float16), hidx, didx))
        assert same_bits(dv[l], _expect(to_np(hv[l]), np.zeros((80, 2, 16), np.float16), hidx, didx))


def test_flat_pool_and_block_copy_routes(cuda_device):
    g = torch.Generator().manual_seed(6)
    host = types.SimpleNamespace(layout="layer_first",
                                 kv_buffer=torch.randint(0, 256, (2, 16, 24), generator=g, dtype=torch.uint8).pin_memory())
    dev = types.SimpleNamespace(layout="layer_first", kv_buffer=torch.zeros((2, 20, 24), dtype=torch.uint8, device="cuda"))
    hidx, didx = torch.tensor([3, 0, 15, 7]), torch.tensor([19, 2, 5, 0])
    assert I.try_sglang_hicache_flat_paged_transfer(host, dev, hidx.cuda(), didx.cuda(), direction="load_to_device")
    torch.cuda.synchronize()
    for l in range(2):
        want = np.zeros((20, 24), np.uint8)
        want[didx.numpy()] = host.kv_buffer[l].numpy()[hidx.numpy()]
        assert same_bits(dev.kv_buffer[l], want)
    kc = torch.randn((6, 2, 8, 4), generator=g).cuda()
    vc = torch.randn((6, 2, 8, 4), generator=g).cuda()
    dk, dv = torch.zeros_like(kc), torch.zeros_like(vc)
    pairs = torch.tensor([[0, 5], [3, 1], [-1, 2]], device="cuda")
    assert I.try_kv_copy_paged_blocks(kc, vc, dk, dv, pairs) == 2
    assert torch.equal(dk[5], kc[0]) and torch.equal(dk[1], kc[3]) and torch.equal(dv[1], vc[3])
    assert int(torch.count_nonzero(dk[2])) == 0


def test_layout_route_all_layer(cuda_device):
    g = torch.Generator().manual_seed(7)
    nl, pages, item = 2, 12, 64
    src_k = torch.randn((nl, pages, item), generator=g).half().cuda()
    src_v = torch.randn((nl, pages, item), generator=g).half().cuda()
    dst_k = torch.zeros_like(src_k)
    dst_v = torch.zeros_like(src_v)
    si = torch.tensor([0, 5, 7], device="cuda")
    di = torch.tensor([11, 1, 6], device="cuda")
    assert I.try_sglang_hicache_layout_transfer(src_k, dst_k, src_v, dst_v, si, di, source_layout="layer_first",
                                                destination_layout="layer_first")
    assert torch.equal(dst_k[:, di], src_k[:, si]) and torch.equal(dst_v[:, di], src_v[:, si])
