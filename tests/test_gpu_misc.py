"""GPU parity for the rest of the kvcache family: Flash dense layouts, the
Triton-indexed dense gather, block copies, DSV4 byte rows, HiCache transfers,
the CacheGen codec and the DSV4 strided block transfer — against the
reference's golden vectors and the CPU oracle, bit for bit."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import musa_aiter as ma
from oracle import kv_oracle as O

from ._util import TORCH_OF, first_diff, same_bits, to_np, to_torch

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
DTYPES = ("float32", "float16", "bfloat16")


@pytest.fixture(scope="module")
def misc():
    return np.load(GOLDEN / "misc.npz")


def T(a, dt=None):
    return to_torch(a, dt)


def eq(a, b, what=""):
    assert same_bits(a, b), f"{what}: {first_diff(a, b)}"


@pytest.mark.parametrize("dt", DTYPES)
def test_golden_flash_triton_blocks(cuda_device, misc, dt):
    p = f"flash/{dt}"
    kc, vc = T(misc[f"{p}/k_cache"], dt), T(misc[f"{p}/v_cache"], dt)
    bt, lens = T(misc["flash/block_tables"]), T(misc["flash/seq_lens"])
    ok, ov = ma.kv_load_and_reshape_flash(kc, vc, bt, lens, max_seq_len=15)
    eq(ok, misc[f"{p}/out_k"], "flash load k")
    eq(ov, misc[f"{p}/out_v"], "flash load v")
    kd, vd = kc.clone(), vc.clone()
    assert ma.kv_reshape_and_cache_back_flash(T(misc[f"{p}/dense_k"], dt), T(misc[f"{p}/dense_v"], dt), kd, vd, bt, lens) is True
    eq(kd, misc[f"{p}/back_k"], "flash back k")
    eq(vd, misc[f"{p}/back_v"], "flash back v")

    q = f"triton/{dt}"
    tk, tv = ma.kv_triton_indexed_to_dense(T(misc[f"{q}/pool_k"], dt), T(misc[f"{q}/pool_v"], dt), T(misc["triton/indptr"]),
                                           T(misc[f"{q}/indices"]), max_seq_len=9)
    eq(tk, misc[f"{q}/out_k"], "triton k")
    eq(tv, misc[f"{q}/out_v"], "triton v")

    r = f"blocks/{dt}"
    sk, sv = T(misc[f"{r}/src_k"], dt), T(misc[f"{r}/src_v"], dt)
    dk = torch.zeros(misc[f"{r}/dst_k"].shape, dtype=TORCH_OF[dt], device="cuda")
    dv = torch.zeros_like(dk)
    n = ma.kv_copy_paged_blocks(sk, sv, dk, dv, T(misc["blocks/pairs"]))
    assert n == int(misc[f"{r}/count"])
    eq(dk, misc[f"{r}/dst_k"], "blocks ml k")
    eq(dv, misc[f"{r}/dst_v"], "blocks ml v")
    dk1 = torch.zeros(misc[f"{r}/dst1_k"].shape, dtype=TORCH_OF[dt], device="cuda")
    dv1 = torch.zeros_like(dk1)
    n1 = ma.kv_copy_paged_blocks(sk[0], sv[0], dk1, dv1, torch.from_numpy(misc["blocks/pairs"]))  # host mapping
    assert n1 == int(misc[f"{r}/count1"])
    eq(dk1, misc[f"{r}/dst1_k"], "blocks k")
    eq(dv1, misc[f"{r}/dst1_v"], "blocks v")


@pytest.mark.parametrize("fp8", (False, True))
def test_block_copy_device_mapping_without_validation(cuda_device, misc, monkeypatch, fp8):
    """Validation off and a device mapping: the count comes back behind an event after the copy
    is queued; copies and count equal the golden ones (negative pairs included)."""
    monkeypatch.setenv("MUSA_AITER_SKIP_VALIDATION", "1")
    r = "blocks/bfloat16"
    sk, sv = T(misc[f"{r}/src_k"], "bfloat16"), T(misc[f"{r}/src_v"], "bfloat16")
    dk = torch.zeros(misc[f"{r}/dst_k"].shape, dtype=torch.bfloat16, device="cuda")
    dv = torch.zeros_like(dk)
    if fp8:  # the same bytes as raw FP8 blocks
        sk, sv, dk, dv = (t.view(torch.uint8) for t in (sk, sv, dk, dv))
    copy = ma.kv_copy_paged_blocks_fp8 if fp8 else ma.kv_copy_paged_blocks
    for _ in range(2):  # a repeated call waits on its own count only
        n = copy(sk, sv, dk, dv, T(misc["blocks/pairs"]))
        assert n == int(misc[f"{r}/count"])
    want_k, want_v = misc[f"{r}/dst_k"], misc[f"{r}/dst_v"]
    if fp8:
        want_k, want_v = want_k.view(np.uint8), want_v.view(np.uint8)
    eq(dk, want_k, "blocks k (no validation)")
    eq(dv, want_v, "blocks v (no validation)")
    assert copy(sk, sv, dk, dv, torch.empty((0, 2), dtype=torch.int64, device="cuda")) == 0


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
def test_golden_fp8_flash(cuda_device, misc, fmt):
    ok, ov = ma.kv_load_and_dequantize_fp8_flash(T(misc["fp8flash/k8"]), T(misc["fp8flash/v8"]), T(misc["fp8flash/bt"]),
                                                 T(misc["fp8flash/lens"]), 0.03, [0.5, 0.25], out_dtype=torch.bfloat16,
                                                 fp8_format=fmt)
    eq(ok, misc[f"fp8flash/{fmt}/out_k"], "fp8 flash k")
    eq(ov, misc[f"fp8flash/{fmt}/out_v"], "fp8 flash v")


def test_golden_rows_and_hicache(cuda_device, misc):
    for width in (1, 24, 1729):
        d = T(misc[f"rows/{width}/dst"])
        ma.kv_copy_paged_rows(T(misc[f"rows/{width}/src"]), d, T(misc["rows/si"]), T(misc["rows/di"]))
        eq(d, misc[f"rows/{width}/out"], f"rows {width}")
    lf_k, lf_v = T(misc["hicache/lf_k"]), T(misc["hicache/lf_v"])
    pf_k, pf_v = T(misc["hicache/pf_k"]), T(misc["hicache/pf_v"])
    si, di = T(misc["hicache/si"]), T(misc["hicache/di"])
    z = torch.zeros_like
    dk, dv = z(lf_k), z(lf_v)
    ma.hicache_transfer_kv_per_layer(lf_k, dk, lf_v, dv, si, di, layer_id=1)
    eq(dk, misc["hicache/out/per_layer/0"], "per_layer k")
    eq(dv, misc["hicache/out/per_layer/1"], "per_layer v")
    dk, dv = z(lf_k), z(lf_v)
    ma.hicache_transfer_kv_per_layer_pf_lf(pf_k, dk, pf_v, dv, si, di, layer_id=2)
    eq(dk, misc["hicache/out/per_layer_pf_lf/0"], "pf_lf k")
    eq(dv, misc["hicache/out/per_layer_pf_lf/1"], "pf_lf v")
    dk, dv = z(lf_k), z(lf_v)
    ma.hicache_transfer_kv_all_layer(lf_k, dk, lf_v, dv, si, di)
    eq(dk, misc["hicache/out/all_layer/0"], "all k")
    dk, dv = z(pf_k), z(pf_v)
    ma.hicache_transfer_kv_all_layer_lf_pf(lf_k, dk, lf_v, dv, si, di)
    eq(dk, misc["hicache/out/all_layer_lf_pf/0"], "lf_pf k")
    eq(dv, misc["hicache/out/all_layer_lf_pf/1"], "lf_pf v")
    dm = z(lf_k)
    ma.hicache_transfer_kv_per_layer_mla(lf_k, dm, si, di, layer_id=0)
    eq(dm, misc["hicache/out/mla_per_layer/0"], "mla per layer")
    dm = z(lf_k)
    ma.hicache_transfer_kv_per_layer_mla_pf_lf(pf_k, dm, si, di, layer_id=1)
    eq(dm, misc["hicache/out/mla_pf_lf/0"], "mla pf_lf")
    dm = z(lf_k)
    ma.hicache_transfer_kv_all_layer_mla(lf_k, dm, si, di)
    eq(dm, misc["hicache/out/mla_all/0"], "mla all")
    dm = z(pf_k)
    ma.hicache_transfer_kv_all_layer_mla_lf_pf(lf_k, dm, si, di)
    eq(dm, misc["hicache/out/mla_all_lf_pf/0"], "mla lf_pf")
    src = [t.contiguous() for t in T(misc["hicache/direct/src"], "bfloat16").unbind(0)]
    dst = [torch.zeros((20, 2, 8), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    ma.hicache_transfer_kv_direct(src, dst, T(misc["hicache/direct/si"]), T(misc["hicache/direct/di"]), 4)
    eq(torch.stack(dst), misc["hicache/direct/out"], "direct")


def test_hicache_pinned_host_pool(cuda_device):
    """Device pages -> pinned host pool and back (the HiCache offload direction), one launch each."""
    g = torch.Generator(device="cuda").manual_seed(4)
    dev_k = torch.randn((4, 64, 128), device="cuda", generator=g).to(torch.bfloat16)
    dev_v = torch.randn((4, 64, 128), device="cuda", generator=g).to(torch.bfloat16)
    host_k = torch.zeros((4, 80, 128), dtype=torch.bfloat16, pin_memory=True)
    host_v = torch.zeros((4, 80, 128), dtype=torch.bfloat16, pin_memory=True)
    si = torch.randperm(64, device="cuda")[:40]
    di = torch.randperm(80, device="cuda")[:40]
    ma.hicache_transfer_kv_all_layer(dev_k, host_k, dev_v, host_v, si, di)
    torch.cuda.synchronize()
    assert torch.equal(host_k[:, di.cpu()].view(torch.int16), dev_k[:, si].cpu().view(torch.int16))
    back_k, back_v = torch.zeros_like(dev_k), torch.zeros_like(dev_v)
    ma.hicache_transfer_kv_all_layer(host_k, back_k, host_v, back_v, di, si)
    torch.cuda.synchronize()
    assert torch.equal(back_v[:, si].view(torch.int16), dev_v[:, si].view(torch.int16))


def test_golden_cachegen(cuda_device, misc):
    for name, dt in (("f32_256", "float32"), ("bf16_256", "bfloat16"), ("f16_16", "float16"), ("f32_2", "float32"), ("const", "float32")):
        p = f"cachegen/{name}"
        x = T(misc[f"{p}/x"], dt)
        bins = misc[f"{p}/codebook"].shape[0]
        enc, cb, cdf = ma.kv_cachegen_encode(x, num_bins=bins)
        eq(enc, misc[f"{p}/enc"], name + " codes")
        eq(cb, misc[f"{p}/codebook"], name + " codebook")
        eq(cdf, misc[f"{p}/cdf"], name + " cdf")
        if f"{p}/dec" in misc:
            eq(ma.kv_cachegen_decode(enc, cb, dtype=TORCH_OF[dt]), misc[f"{p}/dec"], name + " decode")


def test_cachegen_large_vs_oracle(cuda_device):
    g = torch.Generator().manual_seed(9)
    x = (torch.randn((3, 1000, 257), generator=g) * 5.0).to(torch.bfloat16)
    enc, cb, cdf = ma.kv_cachegen_encode(x.cuda(), num_bins=256)
    renc, rcb, rcdf = O.kv_cachegen_encode(O.to_f32(to_np(x), "bfloat16"), 256)
    eq(enc, renc, "codes")
    eq(cdf, rcdf, "cdf")
    eq(cb, rcb, "codebook")


@pytest.mark.parametrize("bins", (2, 17, 256))
@pytest.mark.parametrize("dt", ("bfloat16", "float32"))
def test_cachegen_constant_and_two_valued_slabs_vs_oracle(cuda_device, dt, bins):
    """max == min (every code 0, CDF [0, 1, ..., 1], codebook filled with the value) and a slab
    of two values (codes 0 and bins - 1 only), through the same device launches as any slab."""
    const = torch.full((5, 333), -2.75).to(TORCH_OF[dt])
    two = torch.where(torch.rand((7, 129), generator=torch.Generator().manual_seed(3)) < 0.3, 1.5, -0.5).to(TORCH_OF[dt])
    for x in (const, two):
        enc, cb, cdf = ma.kv_cachegen_encode(x.cuda(), num_bins=bins)
        renc, rcb, rcdf = O.kv_cachegen_encode(O.to_f32(to_np(x), dt), bins)
        eq(enc, renc, "codes")
        eq(cdf, rcdf, "cdf")
        eq(cb, rcb, "codebook")


@pytest.mark.parametrize("vec", (16, 8, 4))
@pytest.mark.parametrize("mode", (0, 1))
def test_strided_block_transfer_vs_oracle(cuda_device, mode, vec):
    """DSV4 staging <-> padded pages, both directions, vs the restated kernel semantics; row,
    value and scale sizes that allow 16-, 8- and 4-byte vectors, and blocks split over several
    warp items."""
    g = torch.Generator().manual_seed(12 + mode + vec)
    nl, nb, bs = 3, 20, 8 if vec == 16 else 37
    value_bytes, scale_bytes = (0, 0) if mode == 0 else {16: (576, 16), 8: (584, 8), 4: (652, 4)}[vec]
    row = {16: 592, 8: 600, 4: 604}[vec] if mode == 0 else value_bytes + scale_bytes
    stride = bs * row + 64  # padded pages
    stt = max(50, 9 + 4 * bs + 3)  # staging tokens: the batch's blocks start at token 9
    pages = [torch.randint(0, 256, (nb * stride,), generator=g, dtype=torch.int32).to(torch.uint8) for _ in range(nl)]
    staging = torch.randint(0, 256, (nl, stt, row), generator=g, dtype=torch.int32).to(torch.uint8)
    block_ids = torch.tensor([7, 3, -1, 12, 0, 19], dtype=torch.int64)
    idx_start, n_valid, offset = 1, 4, 9
    dpages = [p.cuda() for p in pages]
    dstaging = staging.cuda()
    ok = ma.lmcache_kv_strided_block_transfer(dstaging, [p.data_ptr() for p in dpages], block_ids.cuda(), 0, nl, idx_start,
                                              n_valid, offset, stt, bs, row, stride, mode, value_bytes, scale_bytes)
    assert ok is True
    rpages = [p.numpy().copy() for p in pages]
    O.strided_block_transfer(staging.numpy(), rpages, block_ids.numpy(), 0, idx_start, n_valid, offset, bs, row, stride,
                             mode, value_bytes, scale_bytes)
    for a, b in zip(dpages, rpages):
        eq(a, b, "staging->paged")
    out = torch.zeros_like(dstaging)
    ok = ma.lmcache_kv_strided_block_transfer(out, [p.data_ptr() for p in dpages], block_ids.cuda(), 1, nl, idx_start,
                                              n_valid, offset, stt, bs, row, stride, mode, value_bytes, scale_bytes)
    assert ok is True
    rout = np.zeros(out.shape, np.uint8)
    O.strided_block_transfer(rout, rpages, block_ids.numpy(), 1, idx_start, n_valid, offset, bs, row, stride, mode,
                             value_bytes, scale_bytes)
    eq(out, rout, "paged->staging")
    assert ma.lmcache_kv_strided_block_transfer(out, [0] * 2, block_ids.cuda(), 1, nl, 0, 1, 0, stt, bs, row, stride, mode) is False


def test_flash_random_vs_oracle(cuda_device):
    g = torch.Generator().manual_seed(21)
    nb, nh, hd, bs = 64, 4, 64, 16
    kc = torch.randn((nb, nh, hd, bs), generator=g).to(torch.float16)
    vc = torch.randn((nb, nh, hd, bs), generator=g).to(torch.float16)
    lens = torch.tensor([0, 17, 130, 64, 5])
    bt = torch.stack([torch.randperm(nb, generator=g)[:12] for _ in range(5)]).to(torch.int32)
    ok, ov = ma.kv_load_and_reshape_flash(kc.cuda(), vc.cuda(), bt.cuda(), lens.cuda())
    rk, rv = O.kv_load_and_reshape_flash(kc.numpy(), vc.numpy(), bt.numpy(), lens.numpy())
    eq(ok, rk, "flash k")
    eq(ov, rv, "flash v")


def test_kv_copy_paged_rows_layer_table_and_oob(cuda_device):
    g = torch.Generator().manual_seed(30)
    layers = 5
    srcs = [torch.randint(0, 256, (100, 1728), generator=g, dtype=torch.int32).to(torch.uint8).cuda() for _ in range(layers)]
    dsts = [torch.zeros((90, 1728), dtype=torch.uint8, device="cuda") for _ in range(layers)]
    si = torch.tensor([1, 50, 99, 3, 150], device="cuda")  # 150 is out of range: skipped on the device path
    di = torch.tensor([0, 89, 10, 11, 12], device="cuda")
    ma.kv_copy_paged_rows_layer_table(srcs, dsts, si, di)
    for s, d in zip(srcs, dsts):
        assert torch.equal(d[di[:4]], s[si[:4]])
        assert torch.count_nonzero(d[12]) == 0
    with pytest.raises(IndexError):
        ma.kv_copy_paged_rows(srcs[0], dsts[0], torch.tensor([150]), torch.tensor([0]))


def test_memcpy_batch_h2d_d2h(cuda_device):
    """Small entries go through the batch kernel, large ones through the copy engines; offsets and
    registration-boundary splits land every byte where the plan says."""
    g = torch.Generator().manual_seed(40)
    host = torch.randint(0, 256, (9 << 20,), generator=g, dtype=torch.int32).to(torch.uint8).pin_memory()
    dev = torch.zeros(10 << 20, dtype=torch.uint8, device="cuda")
    sizes = [100, 4096, 3, 8 << 20, 1000]
    src_off = [0, 128, 7, 5000, (8 << 20) + 6000]
    dst_off = [16, 4096, 9000, 1 << 20, (9 << 20) + 5]
    assert ma.lmcache_musa_memcpy_batch_async([dev] * 5, [host] * 5, sizes, source_offsets=src_off,
                                              destination_offsets=dst_off, pin_chunk_size=1 << 16) is True
    torch.cuda.synchronize()
    expect = torch.zeros_like(dev).cpu()
    for s, so, do in zip(sizes, src_off, dst_off):
        expect[do: do + s] = host[so: so + s]
    assert torch.equal(dev.cpu(), expect)
    back = torch.zeros(10 << 20, dtype=torch.uint8).pin_memory()
    assert ma.lmcache_musa_memcpy_batch_async([back] * 5, [dev] * 5, sizes, source_offsets=dst_off,
                                              destination_offsets=dst_off, prefer_overlap_with_compute=True,
                                              max_batch_entries=2) is True
    torch.cuda.synchronize()
    for s, do in zip(sizes, dst_off):
        assert torch.equal(back[do: do + s], expect[do: do + s])
    with pytest.raises(ValueError, match="pinned"):
        ma.lmcache_musa_memcpy_batch_async([dev], [torch.zeros(16, dtype=torch.uint8)], [16])
    assert ma.lmcache_musa_memcpy_batch_async([dev], [dev], [16]) is False
    assert ma.native_lmcache_musa_batch_copy_runtime_versions()[0] >= 12000


def test_python_number_fp8_scales_are_placed_once(cuda_device):
    """FP8 scales given as Python numbers go to the device once per value and device: the same
    read-only tensor serves later calls on any stream, and results equal tensor scales'."""
    from musa_aiter.ops import kv_transfer as kt

    dev = torch.device("cuda", torch.cuda.current_device())
    a = kt._device_scalar_scale(0.0173, dev)
    assert a is kt._device_scalar_scale(0.0173, dev) and a.dtype == torch.float32 and a.dim() == 0
    assert float(a) == float(torch.tensor(0.0173, dtype=torch.float32))
    g = torch.Generator().manual_seed(5)
    nb, nh, hd, bs = 64, 2, 128, 16
    kl = torch.randn((300, nh, hd), generator=g).to(torch.bfloat16).cuda()
    vl = torch.randn((300, nh, hd), generator=g).to(torch.bfloat16).cuda()
    slots = torch.randperm(nb * bs, generator=g)[:300].cuda()
    outs = []
    for scales, stream in (((0.0173, 0.031), None), ((0.0173, 0.031), torch.cuda.Stream()),
                           ((torch.tensor(0.0173).cuda(), torch.tensor(0.031).cuda()), None)):
        k8 = torch.zeros((nb, nh, hd, bs), dtype=torch.uint8, device="cuda")
        v8 = torch.zeros_like(k8)
        with torch.cuda.stream(stream or torch.cuda.current_stream()):
            ma.kv_linear_to_paged_fp8(kl, vl, k8, v8, slots, *scales)
            ok, ov = ma.kv_paged_fp8_to_linear(k8, v8, slots, *scales)
        torch.cuda.synchronize()
        outs.append((k8, v8, ok, ov))
    for other in outs[1:]:
        assert all(torch.equal(x, y) for x, y in zip(outs[0], other))


def test_hicache_device_indices_without_validation(cuda_device, monkeypatch):
    """With device page indices and validation off, a HiCache transfer reads nothing back to the
    host: pages whose index is -1 or out of range on either side are skipped by the kernel (the
    rest move exactly as torch indexing moves them), where validation on raises like the
    reference."""
    g = torch.Generator().manual_seed(13)
    L, P, W = 3, 40, 64
    src_k = torch.randn((L, P, W), generator=g).to(torch.bfloat16).cuda()
    src_v = torch.randn((L, P, W), generator=g).to(torch.bfloat16).cuda()
    si = torch.tensor([3, 7, -1, 39, 41, 12, 5, 0], dtype=torch.int64)
    di = torch.tensor([0, 9, 4, 100, 2, -1, 39, 20], dtype=torch.int64)
    with pytest.raises(ValueError):
        ma.hicache_transfer_kv_all_layer(src_k, torch.zeros_like(src_k), src_v, torch.zeros_like(src_v), si.cuda(),
                                         di.cuda())
    monkeypatch.setenv("MUSA_AITER_SKIP_VALIDATION", "1")
    dst_k, dst_v = torch.zeros_like(src_k), torch.zeros_like(src_v)
    ma.hicache_transfer_kv_all_layer(src_k, dst_k, src_v, dst_v, si.cuda(), di.cuda())
    want_k, want_v = torch.zeros_like(src_k), torch.zeros_like(src_v)
    for s, d in zip(si.tolist(), di.tolist()):
        if 0 <= s < P and 0 <= d < P:
            want_k[:, d] = src_k[:, s]
            want_v[:, d] = src_v[:, s]
    assert torch.equal(dst_k.view(torch.int16), want_k.view(torch.int16))
    assert torch.equal(dst_v.view(torch.int16), want_v.view(torch.int16))


def test_cachegen_codebook_matches_torch_linspace(cuda_device):
    """The device codebook (mak_cachegen_codebook) equals torch.linspace(min, max, bins) in float32
    on the GPU, bit for bit, for bounds spread over many magnitudes and every bin count the encode
    takes at its ends and in between; max == min fills min, signed zero included, as the
    reference's torch.full does."""
    from musa_aiter import _native

    lib = _native.load()
    g = torch.Generator().manual_seed(17)
    lo = torch.randn(600, generator=g) * torch.exp(torch.randn(600, generator=g) * 4)
    hi = lo + torch.rand(600, generator=g) * torch.exp(torch.randn(600, generator=g) * 4)
    pairs = [(float(a), float(b)) for a, b in zip(lo.float(), hi.float())] + [(-0.0, -0.0), (3.5, 3.5), (-1.0, 1.0), (0.0, 1e-30)]
    stream = _native.stream_ptr(torch.device("cuda", torch.cuda.current_device()))
    for bins in (2, 3, 17, 128, 255, 256):
        for a, b in pairs:
            mm = torch.tensor([a, b], dtype=torch.float32, device="cuda")
            out = torch.empty(bins, dtype=torch.float32, device="cuda")
            _native.check(lib.mak_cachegen_codebook(_native.ptr(mm), bins, _native.ptr(out), stream), "codebook")
            a32, b32 = float(mm[0]), float(mm[1])
            want = torch.full((bins,), a32, dtype=torch.float32, device="cuda") if a32 == b32 else \
                torch.linspace(a32, b32, bins, dtype=torch.float32, device="cuda")
            assert torch.equal(out.view(torch.int32), want.view(torch.int32)), (a, b, bins)
