"""GPU parity for the MLA FP8 row kernels (per-128 group scales, fused quantise +
scatter and gather + dequantise) against the reference's FP8 element codec
(golden vectors) and the CPU oracle.  Bit-exact: the scales come from the same
fp32 division and every value goes through the same encode / decode rule."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import musa_aiter as ma
from oracle import kv_oracle as O

from ._util import first_diff, same_bits, to_np, to_torch

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
TORCH = {"bfloat16": torch.bfloat16, "float16": torch.float16}


def eq(got, want, what):
    assert same_bits(got, want), f"{what}: {first_diff(got, want)}"


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN / "mla_fp8.npz")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", ("bfloat16", "float16"))
def test_golden_group_codec(cuda_device, golden, dt, fmt):
    p = f"{dt}/{fmt}"
    x = to_torch(golden[f"{p}/x"], dt)
    t = x.shape[0]
    pe = torch.randn((t, 64), device="cuda").to(TORCH[dt])
    row = ma.mla_fp8_row_bytes(512, 64)
    cache = torch.full((4, 8, row), 0xEE, dtype=torch.uint8, device="cuda")
    slots = torch.arange(t, device="cuda") + 3
    assert ma.kv_mla_linear_to_paged_fp8_rows(x, pe, cache, slots, fp8_format=fmt) is True
    rows = cache.view(32, row)[3: 3 + t]
    eq(rows[:, :512], golden[f"{p}/codes"], "codes")
    eq(rows[:, 512:528].contiguous().view(torch.float32), golden[f"{p}/scale"], "scales")
    eq(rows[:, 528:].contiguous().view(TORCH[dt]), to_np(pe), "rope")
    assert torch.all(cache.view(32, row)[:3] == 0xEE) and torch.all(cache.view(32, row)[3 + t:] == 0xEE)
    okv, ope = ma.kv_paged_fp8_rows_to_mla_linear(cache, slots, out_dtype=TORCH[dt], fp8_format=fmt)
    eq(okv, golden[f"{p}/dec"], "decoded latent")
    eq(ope, to_np(pe), "rope round trip")


def _oracle_cache(cache: torch.Tensor) -> np.ndarray:
    c = cache.cpu().numpy()
    return c.reshape(c.shape[0], -1, c.shape[-1]).copy()


@pytest.mark.parametrize("kvd,ped", ((512, 64), (256, 32), (1024, 128), (512, 0), (512, 8), (512, 24), (512, 72)))
@pytest.mark.parametrize("dt", ("bfloat16", "float16"))
def test_random_multi_layer_vs_oracle(cuda_device, kvd, ped, dt):
    g = torch.Generator().manual_seed(kvd + ped)
    nl, nb, bs, t = 3, 12, 16, 90
    x = (torch.randn((nl, t, kvd), generator=g) * torch.exp2(torch.randint(-8, 8, (nl, t, 1), generator=g).float()))
    x = x.to(TORCH[dt])
    pe = torch.randn((nl, t, ped), generator=g).to(TORCH[dt])
    slots = torch.randint(-2, nb * bs, (t,), generator=g, dtype=torch.int64)
    slots[10] = slots[70]  # duplicate: token 70 wins
    row = ma.mla_fp8_row_bytes(kvd, ped)
    cache0 = torch.randint(0, 256, (nl, nb, bs, row), generator=g, dtype=torch.uint8)
    cache = cache0.cuda()
    xs = x.cuda()
    pes = pe.cuda()
    assert ma.kv_mla_linear_to_paged_fp8_rows(xs, pes, cache, slots.cuda()) is True
    want = _oracle_cache(cache0)
    O.mla_fp8_rows_store(to_np(x), to_np(pe), want, slots.numpy(), in_dtype=dt)
    eq(cache.view(nl, nb * bs, row), want, "store")
    # load back from written rows (untouched rows hold random bytes, not FP8 rows), plus misses
    lslots = torch.cat([slots[torch.randperm(t, generator=g)], torch.tensor([-1, -5])]).to(torch.int32)
    okv, ope = ma.kv_paged_fp8_rows_to_mla_linear(cache, lslots.cuda(), kv_dim=kvd, pe_dim=ped, out_dtype=TORCH[dt])
    rk, rp = O.mla_fp8_rows_load(want, lslots.numpy(), kv_dim=kvd, pe_dim=ped, out_dtype=dt)
    eq(okv, rk, "load latent")
    eq(ope, rp, "load rope")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", ("bfloat16", "float16"))
def test_pair_kernels_odd_counts_int32_and_workspace_path(cuda_device, dt, fmt, monkeypatch):
    """kv_dim 512 moves two tokens per warp: odd token counts (the last pair has one token),
    single tokens, int32 and int64 slots with negatives and duplicates, rope rows of 0 to 144
    bytes, and the workspace last-writer path that CUDA graph capture takes next to the owner
    table path of eager calls."""
    g = torch.Generator().manual_seed(91)
    for ped, t in ((64, 91), (8, 1), (24, 33), (72, 77), (0, 5), (64, 2)):
        nl, nb, bs = 2, 7, 64
        x = (torch.randn((nl, t, 512), generator=g) * 3).to(TORCH[dt])
        pe = torch.randn((nl, t, ped), generator=g).to(TORCH[dt])
        slots = torch.randint(-3, nb * bs, (t,), generator=g, dtype=torch.int64)
        if t > 4:
            slots[t - 1] = slots[1]  # duplicate: the last token wins
        row = ma.mla_fp8_row_bytes(512, ped)
        cache0 = torch.randint(0, 256, (nl, nb, bs, row), generator=g, dtype=torch.uint8)
        want = _oracle_cache(cache0)
        O.mla_fp8_rows_store(to_np(x), to_np(pe), want, slots.numpy(), in_dtype=dt, fp8_format=fmt)
        xs, pes, ss = x.cuda(), pe.cuda(), slots.cuda()
        cache = cache0.cuda()
        assert ma.kv_mla_linear_to_paged_fp8_rows(xs, pes, cache, ss.to(torch.int32), fp8_format=fmt) is True
        eq(cache.view(nl, nb * bs, row), want, f"store, owner table, int32 slots {ped, t}")
        # the workspace path: a captured call replayed onto the original cache
        cache2 = cache0.cuda()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):  # warm-up outside capture
            ma.kv_mla_linear_to_paged_fp8_rows(xs, pes, cache2, ss, fp8_format=fmt)
        torch.cuda.current_stream().wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with monkeypatch.context() as m:
            m.setenv("MUSA_AITER_SKIP_VALIDATION", "1")  # the bounds check reads back: not capturable
            with torch.cuda.graph(graph):
                ma.kv_mla_linear_to_paged_fp8_rows(xs, pes, cache2, ss, fp8_format=fmt)
        cache2.copy_(cache0.cuda())
        graph.replay()
        torch.cuda.synchronize()
        del graph
        eq(cache2.view(nl, nb * bs, row), want, f"store, workspace path (graph replay) {ped, t}")
        for idx_dt in (torch.int64, torch.int32):
            lslots = torch.cat([slots.flip(0), torch.tensor([-1])]).to(idx_dt)
            okv, ope = ma.kv_paged_fp8_rows_to_mla_linear(cache, lslots.cuda(), kv_dim=512, pe_dim=ped,
                                                          out_dtype=TORCH[dt], fp8_format=fmt)
            rk, rp = O.mla_fp8_rows_load(want, lslots.numpy(), kv_dim=512, pe_dim=ped, out_dtype=dt, fp8_format=fmt)
            eq(okv, rk, f"load latent {ped, t, idx_dt}")
            eq(ope, rp, f"load rope {ped, t, idx_dt}")


def test_flat_cache_strided_inputs_and_e5m2(cuda_device):
    """Single-layer caches, latent rows read through a strided view, E5M2 codes."""
    g = torch.Generator().manual_seed(77)
    nb, bs, t = 9, 64, 200
    big = (torch.randn((t, 640), generator=g) * 50).to(torch.bfloat16)
    x = big[:, 64:576]  # 16-byte aligned rows with a 1280-byte token stride
    pe = torch.randn((t, 64), generator=g).to(torch.bfloat16)
    slots = torch.randperm(nb * bs, generator=g)[:t].to(torch.int64)
    row = ma.mla_fp8_row_bytes()
    cache = torch.zeros((nb, bs, row), dtype=torch.uint8, device="cuda")
    assert ma.kv_mla_linear_to_paged_fp8_rows(big.cuda()[:, 64:576], pe.cuda(), cache, slots.cuda(), fp8_format="e5m2")
    want = np.zeros((1, nb * bs, row), np.uint8)
    O.mla_fp8_rows_store(to_np(x)[None], to_np(pe)[None], want, slots.numpy(), in_dtype="bfloat16", fp8_format="e5m2")
    eq(cache.view(1, nb * bs, row), want, "store e5m2")
    out_big = torch.full((t, 700), 9.0, dtype=torch.bfloat16, device="cuda")
    okv, ope = ma.kv_paged_fp8_rows_to_mla_linear(cache, slots.cuda(), fp8_format="e5m2", out_kv=out_big[:, 8:520])
    rk, rp = O.mla_fp8_rows_load(want, slots.numpy(), kv_dim=512, pe_dim=64, out_dtype="bfloat16", fp8_format="e5m2")
    eq(okv, rk[0], "load e5m2 into a strided output")
    eq(ope, rp[0], "rope")
    assert torch.all(out_big[:, :8] == 9.0) and torch.all(out_big[:, 520:] == 9.0)


def test_rejects_bad_rows(cuda_device):
    x = torch.zeros((4, 512), dtype=torch.bfloat16, device="cuda")
    pe = torch.zeros((4, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="row is"):
        ma.kv_mla_linear_to_paged_fp8_rows(x, pe, torch.zeros((2, 4, 600), dtype=torch.uint8, device="cuda"),
                                           torch.arange(4, device="cuda"))
    with pytest.raises(ValueError, match="kv_dim"):
        ma.kv_mla_linear_to_paged_fp8_rows(x[:, :384], pe, torch.zeros((2, 4, 528), dtype=torch.uint8, device="cuda"),
                                           torch.arange(4, device="cuda"))
    with pytest.raises(ValueError, match="out of bounds"):
        ma.kv_mla_linear_to_paged_fp8_rows(x, pe, torch.zeros((2, 4, 656), dtype=torch.uint8, device="cuda"),
                                           torch.tensor([0, 1, 2, 8], device="cuda"))


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", ("bfloat16", "float16"))
def test_every_input_under_fixed_group_amax(cuda_device, dt, fmt):
    """Every finite 16-bit input value, quantised under several group scales: each group of 128
    starts with its amax A, the other 127 values are all inputs with |x| <= A (exhaustive)."""
    allv = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(TORCH[dt]).float()
    allv = allv[torch.isfinite(allv)]
    groups = []
    # amax values put the group scale inside, at and outside the division-free range
    # [2^-60, 2^16] of the store (fp8.cuh fast_quot); inf keeps every finite input in the
    # group next to an infinite one
    for amax in (1.0, 3.0, 0.37, 448.0, 1.0e-3, 12345.0, 2.0**-20, 57344.0, 6.0e4, 2.0**-51, 2.0**-52, 2.0**-44,
                 3.0e7, 2.0**25, 2.0**32, float("inf")):
        a = torch.tensor(amax).to(TORCH[dt]).float()
        vals = allv[allv.abs() <= a]
        n = (vals.numel() + 126) // 127
        pad = torch.zeros(n * 127 - vals.numel())
        body = torch.cat([vals, pad]).reshape(n, 127)
        groups.append(torch.cat([a.expand(n, 1), body], dim=1))
    special = torch.zeros(128)
    special[:8] = torch.tensor([float("nan"), -float("inf"), float("inf"), -0.0, 5.0, -5.0, 1.0e-30, -1.0e-30])
    groups.append(special[None])
    g = torch.cat(groups)
    g = torch.cat([g, torch.zeros((-g.shape[0]) % 4, 128)])  # whole rows of 4 groups
    x = g.reshape(-1, 512).to(TORCH[dt])
    t = x.shape[0]
    pe = torch.zeros((t, 64), dtype=TORCH[dt])
    row = ma.mla_fp8_row_bytes()
    nb = (t + 63) // 64
    cache = torch.zeros((nb, 64, row), dtype=torch.uint8, device="cuda")
    slots = torch.arange(t)
    ma.kv_mla_linear_to_paged_fp8_rows(x.cuda(), pe.cuda(), cache, slots.cuda(), fp8_format=fmt)
    want = np.zeros((1, nb * 64, row), np.uint8)
    O.mla_fp8_rows_store(to_np(x)[None], to_np(pe)[None], want, slots.numpy(), in_dtype=dt, fp8_format=fmt)
    eq(cache.view(1, nb * 64, row), want, f"{t} rows, every input")
    okv, _ = ma.kv_paged_fp8_rows_to_mla_linear(cache, slots.cuda(), out_dtype=TORCH[dt], fp8_format=fmt)
    rk, _ = O.mla_fp8_rows_load(want, slots.numpy(), kv_dim=512, pe_dim=64, out_dtype=dt, fp8_format=fmt)
    eq(okv, rk[0], "decode")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", ("bfloat16", "float16"))
def test_division_free_quotient_selfcheck(cuda_device, dt, fmt):
    """The store divides by a group scale through one reciprocal per group and a
    Markstein correction per value; on the device it must agree with the IEEE fp32
    division for every 16-bit input and every scale significand, at the ends of the
    fast range and in between."""
    from musa_aiter import _native

    lib = _native.load()
    counts = torch.zeros(2, dtype=torch.int64, device="cuda")
    code = _native.dtype_code(TORCH[dt])
    f = _native.MAK_FP8_E4M3 if fmt == "e4m3" else _native.MAK_FP8_E5M2
    # the ends of the flush-to-zero encoder's threshold placement and of the fast range, and
    # exponents where 16-bit inputs near the flush threshold are subnormal, normal or absent
    for e in (-60, -41, -20, -12, -9, -1, 0, 5, 6, 8, 13, 14, 16):
        rc = lib.mak_fp8_quotient_selfcheck(code, f, e, counts.data_ptr(), _native.stream_ptr(counts.device))
        _native.check(rc, "mak_fp8_quotient_selfcheck")
    assert counts.tolist() == [0, 0], f"differing codes / quotients: {counts.tolist()}"


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", ("bfloat16", "float16"))
def test_load_every_code_byte(cuda_device, dt, fmt):
    """Rows holding all 256 code bytes in every lane position (also the codes the encoder
    never writes: exponent field 0 with a mantissa, the top codes) under finite scales of
    several magnitudes decode as the reference decoder does."""
    row = ma.mla_fp8_row_bytes()
    t = 512
    g = torch.Generator().manual_seed(11)
    codes = torch.stack([torch.roll(torch.arange(256, dtype=torch.int32), s)[torch.arange(512) % 256]
                         for s in range(t)]).to(torch.uint8)
    # includes both ends of the flush-to-zero decoder's scale range (E4M3 [2^-120, 2^8),
    # E5M2 [2^-112, 2^16)), values just outside them, negative and subnormal scales
    scale_pool = torch.tensor([1.0, 0.5, 3.0e-3, 1.7e5, 2.0**-60, 2.0**20, 0.0, 1.0e-40, 2.0**-120, 2.0**-121,
                               2.0**-112, 2.0**-113, 255.99998, 256.0, 65535.996, 65536.0, -1.0, -3.0e-3,
                               2.0**-126, 2.0**-149], dtype=torch.float32)
    scales = scale_pool[torch.randint(0, scale_pool.numel(), (t, 4), generator=g)]
    pe = torch.randn((t, 64), generator=g).to(TORCH[dt])
    rows = torch.cat([codes, scales.view(torch.uint8).reshape(t, 16), pe.view(torch.uint8).reshape(t, 128)], dim=1)
    cache = rows.reshape(8, 64, row).contiguous()
    slots = torch.randperm(t, generator=g)
    slots[5] = -1
    okv, ope = ma.kv_paged_fp8_rows_to_mla_linear(cache.cuda(), slots.cuda(), out_dtype=TORCH[dt], fp8_format=fmt)
    rk, rp = O.mla_fp8_rows_load(cache.numpy().reshape(1, t, row), slots.numpy(), kv_dim=512, pe_dim=64,
                                 out_dtype=dt, fp8_format=fmt)
    eq(okv, rk[0], "decoded latent")
    eq(ope, rp[0], "rope")
