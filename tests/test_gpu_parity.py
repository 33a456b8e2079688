"""GPU parity: the sm_100a kernels (through the public ``musa_aiter`` API, which
calls the C ABI) against the reference's own outputs (golden vectors) and
against the CPU oracle on larger seeded inputs.  Every comparison is
bit-exact (integer/byte work and the FP8 codec given the same scales)."""

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
def tile():
    return np.load(GOLDEN / "tile.npz")


@pytest.fixture(scope="module")
def fp8():
    return np.load(GOLDEN / "fp8.npz")


@pytest.fixture(scope="module")
def rows():
    return np.load(GOLDEN / "rows.npz")


def T(a, dt=None):
    return to_torch(a, dt)


def full(shape, value, dt):
    return torch.full(shape, value, dtype=TORCH_OF[dt], device="cuda")


def eq(a, b, what=""):
    assert same_bits(a, b), f"{what}: {first_diff(a, b)}"


# ---------------------------------------------------------------------------
# golden replay: tile family
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("dt", DTYPES)
def test_golden_tile(cuda_device, tile, dt):
    p = f"gather/{dt}"
    kc, vc, sl = T(tile[f"{p}/k_cache"], dt), T(tile[f"{p}/v_cache"], dt), T(tile[f"{p}/slots"])
    ok, ov = ma.kv_paged_to_linear(kc, vc, sl)
    eq(ok, tile[f"{p}/out_k"], "gather k")
    eq(ov, tile[f"{p}/out_v"], "gather v")
    pk = full(tuple(ok.shape), 3.0, dt)
    pv = full(tuple(ov.shape), -2.0, dt)
    ma.kv_paged_to_linear(kc, vc, sl, fill_skipped="preserve", out_k=pk, out_v=pv)
    eq(pk, tile[f"{p}/preserve_k"], "preserve k")
    eq(pv, tile[f"{p}/preserve_v"], "preserve v")

    q = f"scatter/{dt}"
    kd = torch.zeros_like(kc)
    vd = full(tuple(vc.shape), 1.5, dt)
    ma.kv_linear_to_paged(T(tile[f"{q}/k_lin"], dt), T(tile[f"{q}/v_lin"], dt), kd, vd, T(tile[f"{q}/slots"]))
    eq(kd, tile[f"{q}/k_cache"], "scatter k")
    eq(vd, tile[f"{q}/v_cache"], "scatter v")

    r = f"gather_ml/{dt}"
    kc3, vc3 = T(tile[f"{r}/k_cache"], dt), T(tile[f"{r}/v_cache"], dt)
    ok3, ov3 = ma.kv_paged_to_linear_multi_layer(kc3, vc3, T(tile[f"{r}/slots"]))
    eq(ok3, tile[f"{r}/out_k"], "ml gather k")
    eq(ov3, tile[f"{r}/out_v"], "ml gather v")
    s = f"scatter_ml/{dt}"
    kd3, vd3 = torch.zeros_like(kc3), torch.zeros_like(vc3)
    ma.kv_linear_to_paged_multi_layer(T(tile[f"{s}/k_lin"], dt), T(tile[f"{s}/v_lin"], dt), kd3, vd3, T(tile[f"{s}/slots"]))
    eq(kd3, tile[f"{s}/k_cache"], "ml scatter k")
    eq(vd3, tile[f"{s}/v_cache"], "ml scatter v")

    eq(ma.kv_paged_to_merged_linear(kc, vc, sl), tile[f"merged/{dt}/gather"], "merged gather")
    eq(ma.kv_paged_to_merged_linear_multi_layer(kc3, vc3, sl), tile[f"merged/{dt}/gather_ml"], "merged ml gather")
    kd, vd = torch.zeros_like(kc), torch.zeros_like(vc)
    ma.kv_merged_linear_to_paged(T(tile[f"merged/{dt}/scatter_in"], dt), kd, vd, T(tile[f"scatter/{dt}/slots"]))
    eq(kd, tile[f"merged/{dt}/scatter_k"], "merged scatter k")
    eq(vd, tile[f"merged/{dt}/scatter_v"], "merged scatter v")


# ---------------------------------------------------------------------------
# golden replay: FP8 codec
# ---------------------------------------------------------------------------


def _enc(fp8, key, fmt, dt):
    kc = torch.zeros(fp8[f"{key}/k_cache"].shape, dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    ks = torch.from_numpy(fp8[f"{key}/k_scale"]).cuda()
    vs = torch.from_numpy(fp8[f"{key}/v_scale"]).cuda()
    ma.kv_linear_to_paged_fp8(T(fp8[f"{key}/k_lin"], dt), T(fp8[f"{key}/v_lin"], dt), kc, vc, T(fp8[f"{key}/slots"]), ks, vs,
                              fp8_format=fmt)
    eq(kc, fp8[f"{key}/k_cache"], f"{key} k")
    eq(vc, fp8[f"{key}/v_cache"], f"{key} v")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
def test_golden_fp8_encode_exhaustive(cuda_device, fp8, fmt):
    for i in range(2):
        _enc(fp8, f"enc_bf16/{fmt}/{i}", fmt, "bfloat16")
    _enc(fp8, f"enc_f16/{fmt}/0", fmt, "float16")
    _enc(fp8, f"enc_f32/{fmt}/0", fmt, "float32")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", DTYPES)
def test_golden_fp8_decode_all_codes(cuda_device, fp8, fmt, dt):
    kc, vc, sl = T(fp8["dec/k_cache"]), T(fp8["dec/v_cache"]), T(fp8["dec/slots"])
    for j in range(2):
        p = f"dec/{fmt}/{dt}/{j}"
        ks = torch.from_numpy(fp8[f"{p}/k_scale"]).cuda()
        vs = torch.from_numpy(fp8[f"{p}/v_scale"]).cuda()
        ok, ov = ma.kv_paged_fp8_to_linear(kc, vc, sl, ks, vs, out_dtype=TORCH_OF[dt], fp8_format=fmt)
        eq(ok, fp8[f"{p}/out_k"], p + " k")
        eq(ov, fp8[f"{p}/out_v"], p + " v")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", DTYPES)
def test_golden_fp8_multi_layer(cuda_device, fp8, fmt, dt):
    p = f"ml/{fmt}/{dt}"
    sl = T(fp8["ml/slots"])
    ks = torch.from_numpy(fp8[f"{p}/k_scale"]).cuda()
    vs = torch.from_numpy(fp8[f"{p}/v_scale"]).cuda()
    kc = torch.zeros(fp8[f"{p}/k_cache"].shape, dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    ma.kv_linear_to_paged_fp8_multi_layer(T(fp8[f"{p}/k_lin"], dt), T(fp8[f"{p}/v_lin"], dt), kc, vc, sl, ks, vs, fp8_format=fmt)
    eq(kc, fp8[f"{p}/k_cache"], p + " store k")
    eq(vc, fp8[f"{p}/v_cache"], p + " store v")
    ok, ov = ma.kv_paged_fp8_to_linear_multi_layer(kc, vc, sl, ks, vs, out_dtype=TORCH_OF[dt], fp8_format=fmt)
    eq(ok, fp8[f"{p}/out_k"], p + " load k")
    eq(ov, fp8[f"{p}/out_v"], p + " load v")


# ---------------------------------------------------------------------------
# golden replay: row family (LMCache / SGLang MP / MLA)
# ---------------------------------------------------------------------------


@pytest.mark.parametrize("dt", DTYPES)
def test_golden_lmcache(cuda_device, rows, dt):
    gs, ss = T(rows["gslots"]), T(rows["sslots"])
    nl, nb, bs, nh, hs = 3, 4, 4, 2, 8
    p = f"six_d/{dt}"
    buf = full(rows[f"{p}/gather"].shape, 13.0, dt)
    assert ma.lmcache_paged_to_kv_buffer(T(rows[f"{p}/paged"], dt), buf, gs) is True
    eq(buf, rows[f"{p}/gather"], "6-D gather")
    dst = full(rows[f"{p}/scatter_dst"].shape, 0.25, dt)
    assert ma.lmcache_kv_buffer_to_paged(T(rows[f"{p}/scatter_src"], dt), dst, ss) is True
    eq(dst, rows[f"{p}/scatter_dst"], "6-D scatter")

    p = f"list/{dt}"
    caches = list(T(rows[f"{p}/caches"], dt).unbind(0))
    mem = full(rows[f"{p}/gather"].shape, 9.0, dt)
    assert ma.lmcache_kv_paged_to_buffer(caches, mem, gs, bs, nh, hs) is True
    eq(mem, rows[f"{p}/gather"], "list gather")
    dcaches = [torch.zeros_like(c).contiguous() for c in caches]
    assert ma.lmcache_kv_buffer_to_paged(T(rows[f"{p}/scatter_src"], dt), dcaches, ss, 2, bs, nh, hs) is True
    eq(torch.stack(dcaches), rows[f"{p}/scatter_dst"], "list scatter")

    p = f"two_x_nl/{dt}"
    two_t = T(rows[f"{p}/caches"], dt)
    two = [[two_t[kv, layer].contiguous() for layer in range(nl)] for kv in range(2)]
    mem = full(rows[f"{p}/gather"].shape, 4.0, dt)
    assert ma.lmcache_kv_paged_to_buffer(two, mem, gs, bs, nh, hs) is True
    eq(mem, rows[f"{p}/gather"], "two_x_nl gather")
    dtwo = [[full((nb, bs, nh, hs), -1.0, dt) for _ in range(nl)] for _ in range(2)]
    assert ma.lmcache_kv_buffer_to_paged_two_x_nl(T(rows[f"{p}/scatter_src"], dt), dtwo, ss, 1, bs, nh, hs) is True
    eq(torch.stack([torch.stack(x) for x in dtwo]), rows[f"{p}/scatter_dst"], "two_x_nl scatter")


@pytest.mark.parametrize("dt", DTYPES)
def test_golden_mla(cuda_device, rows, dt):
    gs, ss = T(rows["gslots"]), T(rows["sslots"])
    p = f"mla/{dt}"
    buf = full(rows[f"{p}/gather"].shape, 5.0, dt)
    assert ma.lmcache_paged_to_kv_buffer_mla(T(rows[f"{p}/paged"], dt), buf, gs) is True
    eq(buf, rows[f"{p}/gather"], "mla gather")
    dst = full(rows[f"{p}/scatter_dst"].shape, 0.0, dt)
    assert ma.lmcache_kv_buffer_to_paged_mla(T(rows[f"{p}/scatter_src"], dt), dst, ss) is True
    eq(dst, rows[f"{p}/scatter_dst"], "mla scatter")

    p = f"mla_list/{dt}"
    caches = [c.contiguous() for c in T(rows[f"{p}/caches"], dt).unbind(0)]
    mem = full(rows[f"{p}/gather"].shape, 7.0, dt)
    assert ma.lmcache_mla_paged_to_buffer(caches, mem, gs, 4, 12) is True
    eq(mem, rows[f"{p}/gather"], "mla list gather")
    dl = [torch.zeros_like(c) for c in caches]
    assert ma.lmcache_mla_buffer_to_paged(T(rows[f"{p}/scatter_src"], dt), dl, ss, 1, 4, 12) is True
    eq(torch.stack(dl), rows[f"{p}/scatter_dst"], "mla list scatter")

    p = f"mla_flat/{dt}"
    kvc, pec = T(rows[f"{p}/kv_cache"], dt), T(rows[f"{p}/pe_cache"], dt)
    okv, ope = ma.kv_paged_to_mla_linear(kvc[0], pec[0], gs)
    eq(okv, rows[f"{p}/gather_kv"], "mla flat kv")
    eq(ope, rows[f"{p}/gather_pe"], "mla flat pe")
    okv3, ope3 = ma.kv_paged_to_mla_linear_multi_layer(kvc, pec, gs)
    eq(okv3, rows[f"{p}/gather_ml_kv"], "mla flat ml kv")
    eq(ope3, rows[f"{p}/gather_ml_pe"], "mla flat ml pe")
    dkv, dpe = torch.zeros_like(kvc), torch.zeros_like(pec)
    assert ma.kv_mla_linear_to_paged_multi_layer(T(rows[f"{p}/scatter_kv_in"], dt), T(rows[f"{p}/scatter_pe_in"], dt),
                                                 dkv, dpe, ss) is True
    eq(dkv, rows[f"{p}/scatter_kv"], "mla flat scatter kv")
    eq(dpe, rows[f"{p}/scatter_pe"], "mla flat scatter pe")


# ---------------------------------------------------------------------------
# larger seeded cases against the oracle
# ---------------------------------------------------------------------------


def block_table_slots(lens, nb, bs, gen) -> torch.Tensor:
    """Per-sequence block tables drawn from one permutation (distinct blocks), as in the bench configs."""
    perm = torch.randperm(nb, generator=gen)
    slots, used = [], 0
    for n in lens:
        nblk = (n + bs - 1) // bs
        bt = perm[used: used + nblk]
        used += nblk
        pos = torch.arange(n)
        slots.append(bt[pos // bs] * bs + pos % bs)
    return torch.cat(slots).to(torch.int64)


@pytest.mark.parametrize("dt", ("float16", "bfloat16"))
def test_config1_tile_round_trip_vs_oracle(cuda_device, dt):
    """Config 1 shapes ([256,16,8,128] caches permuted to [NB,NH,HD,BS]), sequences {100,513,1024,2047}."""
    g = torch.Generator().manual_seed(1)
    nb, bs, nh, hd = 256, 16, 8, 128
    slots = block_table_slots([100, 513, 1024, 2047], nb, bs, g)
    kc = torch.randn((nb, nh, hd, bs), generator=g).to(TORCH_OF[dt])
    vc = torch.randn((nb, nh, hd, bs), generator=g).to(TORCH_OF[dt])
    ok, ov = ma.kv_paged_to_linear(kc.cuda(), vc.cuda(), slots.cuda())
    rk, rv = O.kv_paged_to_linear(to_np(kc), to_np(vc), slots.numpy())
    eq(ok, rk, "cfg1 gather k")
    eq(ov, rv, "cfg1 gather v")
    kd = torch.zeros_like(kc).cuda()
    vd = torch.zeros_like(vc).cuda()
    ma.kv_linear_to_paged(ok, ov, kd, vd, slots.cuda())
    touched = slots.numpy()
    b, o = touched // bs, touched % bs
    assert same_bits(to_np(kd)[b, :, :, o], to_np(kc)[b, :, :, o])
    assert same_bits(to_np(vd)[b, :, :, o], to_np(vc)[b, :, :, o])


@pytest.mark.parametrize("dt", DTYPES)
def test_random_slots_tile_multi_layer_vs_oracle(cuda_device, dt):
    """Random slots with negatives and duplicates, odd head_dim and block_size (element paths)."""
    g = torch.Generator().manual_seed(7)
    for (nl, nb, nh, hd, bs, t) in [(3, 40, 3, 24, 16, 300), (2, 17, 2, 13, 5, 101), (4, 64, 8, 128, 16, 1000)]:
        kc = torch.randn((nl, nb, nh, hd, bs), generator=g).to(TORCH_OF[dt])
        vc = torch.randn((nl, nb, nh, hd, bs), generator=g).to(TORCH_OF[dt])
        slots = torch.randint(-2, nb * bs, (t,), generator=g)
        ok, ov = ma.kv_paged_to_linear_multi_layer(kc.cuda(), vc.cuda(), slots.cuda())
        rk, rv = O.kv_paged_to_linear_multi_layer(to_np(kc), to_np(vc), slots.numpy())
        eq(ok, rk, f"gather {nl,nb,nh,hd,bs}")
        eq(ov, rv, f"gather {nl,nb,nh,hd,bs}")
        kl = torch.randn((nl, t, nh, hd), generator=g).to(TORCH_OF[dt])
        vl = torch.randn((nl, t, nh, hd), generator=g).to(TORCH_OF[dt])
        kd, vd = kc.clone().cuda(), vc.clone().cuda()
        ma.kv_linear_to_paged_multi_layer(kl.cuda(), vl.cuda(), kd, vd, slots.to(torch.int32).cuda())
        rkc, rvc = to_np(kc), to_np(vc)
        O.kv_linear_to_paged_multi_layer(to_np(kl), to_np(vl), rkc, rvc, slots.numpy())
        eq(kd, rkc, "scatter k")
        eq(vd, rvc, "scatter v")


@pytest.mark.parametrize("fmt", (None, "e4m3", "e5m2"))
def test_decode_batch_head_split_vs_oracle(cuda_device, fmt):
    """Decode-sized batches of random slots: the single-token launch splits each window's heads
    over several warp items (num_heads 1..16, head_dim 64..256, splits of 1, 2 and up to 16 warps
    per window), with negative and duplicate slots; gathers, scatters, FP8 stores and loads."""
    g = torch.Generator().manual_seed(11)
    for (nl, nb, nh, hd, bs, t) in [(2, 256, 8, 128, 16, 40), (1, 64, 6, 96, 16, 17), (3, 128, 16, 64, 16, 9),
                                    (1, 64, 1, 256, 16, 33), (2, 96, 2, 128, 8, 64), (1, 300, 4, 128, 16, 200)]:
        slots = torch.randperm(nb * bs, generator=g)[:t]
        slots[::7] = -1
        slots[5::11] = slots[3]
        if fmt is None:
            kc = torch.randn((nl, nb, nh, hd, bs), generator=g).to(torch.bfloat16)
            vc = torch.randn((nl, nb, nh, hd, bs), generator=g).to(torch.bfloat16)
            ok, ov = ma.kv_paged_to_linear_multi_layer(kc.cuda(), vc.cuda(), slots.cuda())
            rk, rv = O.kv_paged_to_linear_multi_layer(to_np(kc), to_np(vc), slots.numpy())
            eq(ok, rk, f"gather {nl, nb, nh, hd, bs, t}")
            eq(ov, rv, f"gather {nl, nb, nh, hd, bs, t}")
            kl = torch.randn((nl, t, nh, hd), generator=g).to(torch.bfloat16)
            vl = torch.randn((nl, t, nh, hd), generator=g).to(torch.bfloat16)
            kd, vd = kc.clone().cuda(), vc.clone().cuda()
            ma.kv_linear_to_paged_multi_layer(kl.cuda(), vl.cuda(), kd, vd, slots.cuda())
            rkc, rvc = to_np(kc), to_np(vc)
            O.kv_linear_to_paged_multi_layer(to_np(kl), to_np(vl), rkc, rvc, slots.numpy())
            eq(kd, rkc, f"scatter k {nl, nb, nh, hd, bs, t}")
            eq(vd, rvc, f"scatter v {nl, nb, nh, hd, bs, t}")
            continue
        kl = (torch.randn((nl, t, nh, hd), generator=g) * 2.0).to(torch.bfloat16)
        vl = (torch.randn((nl, t, nh, hd), generator=g) * 2.0).to(torch.bfloat16)
        fmax = 448.0 if fmt == "e4m3" else 57344.0
        ks = kl.float().abs().amax(dim=(1, 3)) / fmax
        vs = vl.float().abs().amax() / fmax
        kc = torch.randint(0, 256, (nl, nb, nh, hd, bs), generator=g, dtype=torch.uint8)
        vc = torch.randint(0, 256, (nl, nb, nh, hd, bs), generator=g, dtype=torch.uint8)
        kd, vd = kc.cuda(), vc.cuda()
        ma.kv_linear_to_paged_fp8_multi_layer(kl.cuda(), vl.cuda(), kd, vd, slots.cuda(), ks.cuda(), vs.cuda(), fp8_format=fmt)
        rkc, rvc = kc.numpy().copy(), vc.numpy().copy()
        O.kv_linear_to_paged_fp8_multi_layer(to_np(kl), to_np(vl), rkc, rvc, slots.numpy(), ks.numpy(), vs.numpy(),
                                             fp8_format=fmt)
        eq(kd, rkc, f"fp8 store k {nl, nb, nh, hd, bs, t}")
        eq(vd, rvc, f"fp8 store v {nl, nb, nh, hd, bs, t}")
        ok, ov = ma.kv_paged_fp8_to_linear_multi_layer(kd, vd, slots.cuda(), ks.cuda(), vs.cuda(), out_dtype=torch.bfloat16,
                                                       fp8_format=fmt)
        rk, rv = O.kv_paged_fp8_to_linear_multi_layer(rkc, rvc, slots.numpy(), ks.numpy(), vs.numpy(), out_dtype="bfloat16",
                                                      fp8_format=fmt)
        eq(ok, rk, f"fp8 load k {nl, nb, nh, hd, bs, t}")
        eq(ov, rv, f"fp8 load v {nl, nb, nh, hd, bs, t}")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
def test_config3_fp8_random_slots_vs_oracle(cuda_device, fmt):
    """Config 3 style: randn*2 bf16, random unique slots, per-layer-head (E4M3) / scalar (E5M2) scales."""
    g = torch.Generator().manual_seed(3)
    nl, nb, nh, hd, bs, t = 4, 512, 8, 128, 16, 256
    kl = (torch.randn((nl, t, nh, hd), generator=g) * 2.0).to(torch.bfloat16)
    vl = (torch.randn((nl, t, nh, hd), generator=g) * 2.0).to(torch.bfloat16)
    slots = torch.randperm(nb * bs, generator=g)[:t]
    if fmt == "e4m3":
        ks = kl.float().abs().amax(dim=(1, 3)) / 448.0  # [L, NH]
        vs = vl.float().abs().amax(dim=(1, 3)) / 448.0
    else:
        ks = kl.float().abs().amax() / 57344.0
        vs = vl.float().abs().amax() / 57344.0
    kc = torch.zeros((nl, nb, nh, hd, bs), dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    ma.kv_linear_to_paged_fp8_multi_layer(kl.cuda(), vl.cuda(), kc, vc, slots.cuda(), ks.cuda(), vs.cuda(), fp8_format=fmt)
    rkc = np.zeros(kc.shape, np.uint8)
    rvc = np.zeros(vc.shape, np.uint8)
    O.kv_linear_to_paged_fp8_multi_layer(to_np(kl), to_np(vl), rkc, rvc, slots.numpy(), ks.numpy(), vs.numpy(), fp8_format=fmt)
    eq(kc, rkc, "fp8 store k")
    eq(vc, rvc, "fp8 store v")
    ok, ov = ma.kv_paged_fp8_to_linear_multi_layer(kc, vc, slots.cuda(), ks.cuda(), vs.cuda(), out_dtype=torch.bfloat16, fp8_format=fmt)
    rk, rv = O.kv_paged_fp8_to_linear_multi_layer(rkc, rvc, slots.numpy(), ks.numpy(), vs.numpy(), out_dtype="bfloat16", fp8_format=fmt)
    eq(ok, rk, "fp8 load k")
    eq(ov, rv, "fp8 load v")


def test_fp8_block_table_slots_packed_path(cuda_device):
    """Block-table slots (full 16-token runs) exercise the 16-byte FP8 vector path."""
    g = torch.Generator().manual_seed(5)
    nb, nh, hd, bs = 128, 4, 64, 16
    slots = block_table_slots([37, 160, 301], nb, bs, g)
    t = slots.numel()
    kl = torch.randn((t, nh, hd), generator=g).to(torch.float16)
    vl = torch.randn((t, nh, hd), generator=g).to(torch.float16)
    ks = torch.rand(nh, generator=g) * 0.01 + 0.002
    kc = torch.zeros((nb, nh, hd, bs), dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    ma.kv_linear_to_paged_fp8(kl.cuda(), vl.cuda(), kc, vc, slots.cuda(), ks.cuda(), 0.004)
    rkc, rvc = np.zeros(kc.shape, np.uint8), np.zeros(vc.shape, np.uint8)
    O.kv_linear_to_paged_fp8(kl.numpy(), vl.numpy(), rkc, rvc, slots.numpy(), ks.numpy(), np.float32(0.004), lin_dtype="float16")
    eq(kc, rkc, "fp8 packed store k")
    eq(vc, rvc, "fp8 packed store v")
    ok, ov = ma.kv_paged_fp8_to_linear(kc, vc, slots.cuda(), ks.cuda(), 0.004, out_dtype=torch.float32)
    rk, rv = O.kv_paged_fp8_to_linear(rkc, rvc, slots.numpy(), ks.numpy(), np.float32(0.004), out_dtype="float32")
    eq(ok, rk, "fp8 packed load k")
    eq(ov, rv, "fp8 packed load v")


def test_lmcache_list_config2_subset_vs_oracle(cuda_device):
    """Config 2 geometry (8 heads x 128, BS 16) on a reduced cache: list gather/scatter, one launch."""
    g = torch.Generator().manual_seed(2)
    nl, nb, bs, nh, hs = 4, 2048, 16, 8, 128
    lens = torch.randint(256, 4097, (6,), generator=g).tolist()
    slots = block_table_slots(lens, nb, bs, g)
    t = slots.numel()
    caches = [torch.randn((2, nb, bs, nh, hs), generator=g).to(torch.bfloat16) for _ in range(nl)]
    mem = torch.empty((2, nl, t, nh * hs), dtype=torch.bfloat16, device="cuda")
    dcaches = [c.cuda() for c in caches]
    assert ma.lmcache_kv_paged_to_buffer(dcaches, mem, slots.cuda(), bs, nh, hs) is True
    ref = np.zeros((2, nl, t, nh * hs), np.uint16)
    O.lmcache_list_paged_to_buffer([to_np(c) for c in caches], ref, slots.numpy())
    eq(mem, ref, "list gather")
    fresh = [torch.zeros_like(c) for c in dcaches]
    assert ma.lmcache_kv_buffer_to_paged(mem, fresh, slots.cuda(), 0, bs, nh, hs) is True
    for c_src, c_dst in zip(dcaches, fresh):
        flat_s = c_src.view(2, nb * bs, nh * hs)[:, slots.cuda()]
        flat_d = c_dst.view(2, nb * bs, nh * hs)[:, slots.cuda()]
        assert torch.equal(flat_s.view(torch.int16), flat_d.view(torch.int16))


def test_current_stream_is_used(cuda_device):
    """Kernels run on the caller's current stream (op_tests/test_phase5_musa.py:608-639 checks the same)."""
    nb, bs, nh, hs, nl = 64, 16, 2, 64, 2
    caches = [torch.randn((2, nb, bs, nh, hs), device="cuda", dtype=torch.float16) for _ in range(nl)]
    slots = torch.arange(200, device="cuda")
    mem = torch.empty((2, nl, 200, nh * hs), device="cuda", dtype=torch.float16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ma.lmcache_kv_paged_to_buffer(caches, mem, slots, bs, nh, hs)
        ev = torch.cuda.Event()
        ev.record(s)
    ev.synchronize()
    expect = torch.stack([torch.stack([c[kv].reshape(-1, nh * hs)[:200] for c in caches]) for kv in range(2)])
    assert torch.equal(mem, expect)


def test_empty_and_out_of_range(cuda_device):
    kc = torch.randn((4, 2, 8, 4), device="cuda")
    vc = torch.randn((4, 2, 8, 4), device="cuda")
    ok, ov = ma.kv_paged_to_linear(kc, vc, torch.empty(0, dtype=torch.int64, device="cuda"))
    assert ok.shape == (0, 2, 8)
    with pytest.raises(ValueError, match="out of bounds"):
        ma.kv_paged_to_linear(kc, vc, torch.tensor([0, 16], device="cuda"))
    with pytest.raises(ValueError, match="out of bounds"):
        ma.kv_linear_to_paged(torch.zeros((1, 2, 8), device="cuda"), torch.zeros((1, 2, 8), device="cuda"), kc, vc,
                              torch.tensor([99], device="cuda"))
    all_neg = torch.full((5,), -1, device="cuda")
    ok, _ = ma.kv_paged_to_linear(kc, vc, all_neg)
    assert torch.count_nonzero(ok) == 0


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", ("bfloat16", "float16"))
def test_fp8_block_table_store_bounded_and_fallback_chunks(cuda_device, dt, fmt):
    """Full 16-token chunks whose values stay below fp8_max * scale take the division-free
    encoder, the others the per-element one; both must equal the reference rule: amax-derived
    per-head scales, plus chunks holding -0, values at and below the flush threshold, values
    beyond the scaled range, inf and nan."""
    g = torch.Generator().manual_seed(17)
    nb, nh, hd, bs = 64, 2, 128, 16
    slots = block_table_slots([160, 96, 33], nb, bs, g)
    t = slots.numel()
    fmax = 448.0 if fmt == "e4m3" else 57344.0
    flush = 2.0**-6 if fmt == "e4m3" else 2.0**-14
    kl = torch.randn((t, nh, hd), generator=g) * 3.0
    ks = kl.abs().amax(dim=(0, 2)) / fmax  # [NH]
    kl[5, 0, :8] = torch.tensor([-0.0, 0.0, flush * ks[0] * 0.999, -flush * ks[0] * 0.999, flush * ks[0],
                                 -flush * ks[0] * 1.001, ks[0] * fmax * 0.9999, -ks[0] * fmax])
    kl[40, 1, 16:20] = torch.tensor([ks[1] * fmax * 4.0, -ks[1] * fmax * 1.2, 1.0e-30, -1.0e-30])
    kl[70, 0, 64] = float("inf")
    kl[71, 1, 100] = float("nan")
    kl[100, 0, 3] = -float("inf")
    kl = kl.to(TORCH_OF[dt])
    vl = (torch.randn((t, nh, hd), generator=g) * 0.5).to(TORCH_OF[dt])
    vs = torch.tensor(0.5 / fmax)
    kc = torch.zeros((nb, nh, hd, bs), dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    ma.kv_linear_to_paged_fp8(kl.cuda(), vl.cuda(), kc, vc, slots.cuda(), ks.cuda(), float(vs), fp8_format=fmt)
    rkc, rvc = np.zeros(kc.shape, np.uint8), np.zeros(vc.shape, np.uint8)
    O.kv_linear_to_paged_fp8(to_np(kl), to_np(vl), rkc, rvc, slots.numpy(), ks.numpy(), np.float32(vs), lin_dtype=dt,
                             fp8_format=fmt)
    eq(kc, rkc, "fp8 block-table store k")
    eq(vc, rvc, "fp8 block-table store v")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", ("bfloat16", "float16", "float32"))
def test_fp8_block_table_load_scales_inside_and_outside_fast_range(cuda_device, dt, fmt):
    """Full-chunk FP8 loads decode through a flush-to-zero multiply when the scale lies in
    [2^(bias-127), 2^(bias+1)) and field by field otherwise; every code byte under per-head scales
    at, inside and outside both ends of that range must decode as the reference does."""
    g = torch.Generator().manual_seed(23)
    nb, nh, hd, bs = 32, 8, 64, 16
    slots = block_table_slots([160, 96], nb, bs, g)
    kc = torch.randint(0, 256, (nb, nh, hd, bs), generator=g, dtype=torch.int32).to(torch.uint8)
    vc = torch.randint(0, 256, (nb, nh, hd, bs), generator=g, dtype=torch.int32).to(torch.uint8)
    hi = 2.0**8 if fmt == "e4m3" else 2.0**16
    lo = 2.0**-120 if fmt == "e4m3" else 2.0**-112
    ks = torch.tensor([1.0, hi, hi * 0.999999, lo, lo * 0.5, 3.0e-3, 2.0**-126, 1.0e-30], dtype=torch.float32)
    vs = torch.tensor(0.0371, dtype=torch.float32)
    ok, ov = ma.kv_paged_fp8_to_linear(kc.cuda(), vc.cuda(), slots.cuda(), ks.cuda(), float(vs), out_dtype=TORCH_OF[dt],
                                       fp8_format=fmt)
    rk, rv = O.kv_paged_fp8_to_linear(kc.numpy(), vc.numpy(), slots.numpy(), ks.numpy(), np.float32(vs), out_dtype=dt,
                                      fp8_format=fmt)
    eq(ok, rk, "fp8 block-table load k")
    eq(ov, rv, "fp8 block-table load v")


def _mixed_run_slots(n_target, nb, bs, gen, stretch=1) -> torch.Tensor:
    """Unique slots in runs of every kind the tile launches split between them: whole blocks,
    runs of 1-15 slots from a random in-block offset, lone random slots (stretches of up to
    ``stretch`` of them in a row, each in a block of its own) and negatives."""
    perm = torch.randperm(nb, generator=gen).tolist()
    kinds = torch.randint(0, 4, (n_target,), generator=gen).tolist()
    lens = torch.randint(1, bs, (n_target,), generator=gen).tolist()
    offs = torch.randint(0, bs, (n_target,), generator=gen).tolist()
    reps = torch.randint(1, stretch + 1, (n_target,), generator=gen).tolist()
    out, n, i, nxt = [], 0, 0, 0
    while n < n_target:
        k = kinds[i]
        if k == 0:
            piece = [perm[nxt] * bs + o for o in range(bs)]
            nxt += 1
        elif k == 1:
            o0 = min(offs[i], bs - lens[i])
            piece = [perm[nxt] * bs + o0 + o for o in range(lens[i])]
            nxt += 1
        elif k == 2:
            piece = [perm[nxt + j] * bs + (offs[i] + 5 * j) % bs for j in range(reps[i])]
            nxt += reps[i]
        else:
            piece = [-1] * (1 + offs[i] % 3)
        out.extend(piece)
        n += len(piece)
        i += 1
    return torch.tensor(out[:n_target], dtype=torch.int64)


@pytest.mark.parametrize("stretch", (1, 24))
@pytest.mark.parametrize("stale_bits", (0, 1))
@pytest.mark.parametrize("fp8", (False, True))
def test_tile_segment_map_skips_only_clean_windows(cuda_device, monkeypatch, fp8, stale_bits, stretch):
    """The run launch moves the single tokens of the windows that hold at most four of them and
    records, per window, whether it left single tokens to the single-token launch, which skips the
    other windows and tokens: results equal the unmapped launches' (where the run launch leaves
    every single token) and the oracle's for calls whose window sizes differ between the two
    launches (8 to 32 tokens), with lone slots scattered (stretch 1) or in stretches of up to 24
    (windows with many single tokens next to windows with few), also when the map already holds
    this call's epoch (entry = epoch << 2 | bit) marked clean everywhere (stale_bits 0) or marked
    everywhere (stale_bits 1) -- the run launch rewrites every entry before the single-token
    launch reads it."""
    from musa_aiter import _native

    g = torch.Generator().manual_seed(11 + stretch)
    nb, nh, hd, bs = 32768 if stretch == 1 else 131072, 1, 16, 16
    ks, vs = torch.tensor(0.013), torch.tensor(0.021)
    for t in (600, 40000, 170000):
        slots = _mixed_run_slots(t, nb, bs, g, stretch)
        if fp8:
            kc = torch.randint(0, 256, (nb, nh, hd, bs), generator=g, dtype=torch.uint8)
            vc = torch.randint(0, 256, (nb, nh, hd, bs), generator=g, dtype=torch.uint8)
            kc[(kc & 0x7F) == 0x7F] = 0  # e4m3 nan codes decode to nan: keep the comparison bitwise
            vc[(vc & 0x7F) == 0x7F] = 0
            load = lambda: ma.kv_paged_fp8_to_linear(kc.cuda(), vc.cuda(), slots.cuda(), ks.cuda(), vs.cuda())  # noqa: E731
            rk, rv = O.kv_paged_fp8_to_linear(kc.numpy(), vc.numpy(), slots.numpy(), ks.numpy(), vs.numpy())
        else:
            kc = torch.randn((nb, nh, hd, bs), generator=g).to(torch.bfloat16)
            vc = torch.randn((nb, nh, hd, bs), generator=g).to(torch.bfloat16)
            load = lambda: ma.kv_paged_to_linear(kc.cuda(), vc.cuda(), slots.cuda())  # noqa: E731
            rk, rv = O.kv_paged_to_linear(to_np(kc), to_np(vc), slots.numpy())
        kl = (torch.randn((t, nh, hd), generator=g) * 3.0).to(torch.bfloat16)
        vl = (torch.randn((t, nh, hd), generator=g) * 3.0).to(torch.bfloat16)

        def store():
            kd = torch.zeros((nb, nh, hd, bs), dtype=torch.uint8 if fp8 else torch.bfloat16, device="cuda")
            vd = torch.zeros_like(kd)
            if fp8:
                ma.kv_linear_to_paged_fp8(kl.cuda(), vl.cuda(), kd, vd, slots.cuda(), ks.cuda(), vs.cuda())
            else:
                ma.kv_linear_to_paged(kl.cuda(), vl.cuda(), kd, vd, slots.cuda())
            return kd, vd

        # this stream's map, pre-set to "clean" for the epoch the next call takes
        dev = torch.device("cuda", torch.cuda.current_device())
        _native.seg_map(dev, _native.stream_ptr(dev), t)
        ent = _native._SEGMAPS[(dev.index, _native.stream_ptr(dev))]
        ent[0].fill_((ent[3] << 2) | stale_bits)
        mk, mv = load()
        ent[0].fill_((ent[3] << 2) | stale_bits)
        sk, sv = store()
        eq(mk, rk, f"mapped load k t={t}")
        eq(mv, rv, f"mapped load v t={t}")
        with monkeypatch.context() as m:
            m.setattr(_native, "seg_map", lambda *a: (None, 0, 0))
            uk, uv = load()
            usk, usv = store()
        assert torch.equal(mk.view(torch.int16), uk.view(torch.int16)) and torch.equal(mv.view(torch.int16), uv.view(torch.int16))
        assert torch.equal(sk.view(torch.uint8), usk.view(torch.uint8)) and torch.equal(sv.view(torch.uint8), usv.view(torch.uint8))
        if fp8:
            rkc, rvc = np.zeros(sk.shape, np.uint8), np.zeros(sv.shape, np.uint8)
            O.kv_linear_to_paged_fp8(to_np(kl), to_np(vl), rkc, rvc, slots.numpy(), ks.numpy(), vs.numpy())
        else:
            rkc, rvc = np.zeros(sk.shape, to_np(kl).dtype), np.zeros(sv.shape, to_np(vl).dtype)
            O.kv_linear_to_paged(to_np(kl), to_np(vl), rkc, rvc, slots.numpy())
        eq(sk, rkc, f"mapped store k t={t}")
        eq(sv, rvc, f"mapped store v t={t}")


@pytest.mark.parametrize("fp8", (False, True))
def test_tile_owned_scatter_duplicates_vs_workspace_and_oracle(cuda_device, monkeypatch, fp8):
    """Tile scatters resolve duplicate slots through the stream's owner table: block tables that
    share blocks (runs written several times, later tokens win), lone duplicates and negatives give
    the oracle's cache and the workspace path's, also after a row scatter used the same table."""
    from musa_aiter import _native

    g = torch.Generator().manual_seed(21)
    nl, nb, nh, hd, bs = 2, 96, 4, 64, 16
    tables = [torch.randperm(nb, generator=g)[:6] for _ in range(5)]  # sequences share blocks
    slots = torch.cat([(bt[:, None] * bs + torch.arange(bs)[None, :]).flatten()[: 70 + 3 * i] for i, bt in enumerate(tables)])
    extra = torch.randint(-3, nb * bs, (200,), generator=g)
    slots = torch.cat([slots, extra, slots[:40]])  # lone duplicates, negatives, a repeated run
    t = slots.numel()
    kl = (torch.randn((nl, t, nh, hd), generator=g) * 2.0).to(torch.bfloat16)
    vl = (torch.randn((nl, t, nh, hd), generator=g) * 2.0).to(torch.bfloat16)
    ks, vs = torch.rand(nh, generator=g) * 0.01 + 0.003, torch.tensor(0.02)
    dt = torch.uint8 if fp8 else torch.bfloat16

    def store():
        kc = torch.zeros((nl, nb, nh, hd, bs), dtype=dt, device="cuda")
        vc = torch.zeros_like(kc)
        if fp8:
            ma.kv_linear_to_paged_fp8_multi_layer(kl.cuda(), vl.cuda(), kc, vc, slots.cuda(), ks.cuda(), vs.cuda())
        else:
            ma.kv_linear_to_paged_multi_layer(kl.cuda(), vl.cuda(), kc, vc, slots.cuda())
        return kc, vc

    # a row scatter on the same stream first leaves its own marks in the owner table
    rows_dst = torch.zeros((4 * nb * bs, 8), dtype=torch.uint8, device="cuda")
    ma.kv_copy_paged_rows(torch.randint(0, 256, (64, 8), generator=g, dtype=torch.uint8).cuda(), rows_dst,
                          torch.arange(64, device="cuda"), torch.arange(64, device="cuda") * 3)
    ok_k, ok_v = store()
    with monkeypatch.context() as m:
        m.setattr(_native, "owned_scatter", lambda *a: None)
        ws_k, ws_v = store()
    assert torch.equal(ok_k.view(torch.uint8), ws_k.view(torch.uint8))
    assert torch.equal(ok_v.view(torch.uint8), ws_v.view(torch.uint8))
    if fp8:
        rk, rv = np.zeros(ok_k.shape, np.uint8), np.zeros(ok_v.shape, np.uint8)
        O.kv_linear_to_paged_fp8_multi_layer(to_np(kl), to_np(vl), rk, rv, slots.numpy(), ks.numpy(), vs.numpy())
    else:
        rk, rv = np.zeros(ok_k.shape, to_np(kl).dtype), np.zeros(ok_v.shape, to_np(vl).dtype)
        O.kv_linear_to_paged_multi_layer(to_np(kl), to_np(vl), rk, rv, slots.numpy())
    eq(ok_k, rk, "owned scatter k")
    eq(ok_v, rv, "owned scatter v")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
def test_fp8_small_calls_take_every_token_vs_oracle(cuda_device, fmt):
    """FP8 calls of at most 512 tokens skip the run launch: one kernel moves every token, the
    tokens of block-table runs element by element, last writer winning on duplicate slots, and a
    gather writes zero rows for the tokens without a slot.  Stores and loads at 40, 300 and 512
    tokens (and 513, the first size that takes the run launch again) equal the oracle's bytes,
    with multi-layer per-head scales."""
    g = torch.Generator().manual_seed(31 if fmt == "e4m3" else 32)
    nl, nb, nh, hd, bs = 2, 256, 2, 128, 16
    for t in (40, 300, 512, 513):
        slots = _mixed_run_slots(t, nb, bs, g, stretch=3)
        slots[t // 3] = slots[t // 2] if slots[t // 2] >= 0 else slots[t // 3]  # a duplicate slot
        kl = (torch.randn((nl, t, nh, hd), generator=g) * 3.0).to(torch.bfloat16)
        vl = (torch.randn((nl, t, nh, hd), generator=g) * 3.0).to(torch.bfloat16)
        ks = torch.rand((nl, nh), generator=g) * 0.02 + 0.005
        vs = torch.rand((nl, nh), generator=g) * 0.02 + 0.005
        k8 = torch.randint(0, 120, (nl, nb, nh, hd, bs), generator=g, dtype=torch.uint8)
        v8 = torch.randint(0, 120, (nl, nb, nh, hd, bs), generator=g, dtype=torch.uint8)
        dk, dv = k8.cuda(), v8.cuda()
        ma.kv_linear_to_paged_fp8_multi_layer(kl.cuda(), vl.cuda(), dk, dv, slots.cuda(), ks.cuda(), vs.cuda(), fp8_format=fmt)
        rk, rv = k8.numpy().copy(), v8.numpy().copy()
        O.kv_linear_to_paged_fp8_multi_layer(to_np(kl), to_np(vl), rk, rv, slots.numpy(), ks.numpy(), vs.numpy(), fp8_format=fmt)
        eq(dk, rk, f"store k t={t}")
        eq(dv, rv, f"store v t={t}")
        ok, ov = ma.kv_paged_fp8_to_linear_multi_layer(dk, dv, slots.cuda(), ks.cuda(), vs.cuda(), out_dtype=torch.bfloat16,
                                                       fp8_format=fmt)
        qk, qv = O.kv_paged_fp8_to_linear_multi_layer(rk, rv, slots.numpy(), ks.numpy(), vs.numpy(), out_dtype="bfloat16",
                                                       fp8_format=fmt)
        eq(ok, qk, f"load k t={t}")
        eq(ov, qv, f"load v t={t}")


@pytest.mark.parametrize("dt", ("bfloat16", "float16"))
def test_small_tile_calls_take_every_token_vs_oracle(cuda_device, dt):
    """16-bit tile calls of at most 512 tokens skip the run launch as well: one kernel moves every
    token, the tokens of block-table runs element by element, the last writer winning on a
    duplicate slot, and a gather zero-fills the tokens without a slot.  Scatters and gathers at
    40, 300, 512 and 513 tokens equal the oracle's bytes."""
    g = torch.Generator().manual_seed(41 if dt == "bfloat16" else 42)
    nl, nb, nh, hd, bs = 2, 256, 2, 64, 16
    for t in (40, 300, 512, 513):
        slots = _mixed_run_slots(t, nb, bs, g, stretch=3)
        slots[t // 3] = slots[t // 2] if slots[t // 2] >= 0 else slots[t // 3]  # a duplicate slot
        kl = torch.randn((nl, t, nh, hd), generator=g).to(TORCH_OF[dt])
        vl = torch.randn((nl, t, nh, hd), generator=g).to(TORCH_OF[dt])
        kc = torch.randn((nl, nb, nh, hd, bs), generator=g).to(TORCH_OF[dt])
        vc = torch.randn((nl, nb, nh, hd, bs), generator=g).to(TORCH_OF[dt])
        dk, dv = kc.cuda(), vc.cuda()
        ma.kv_linear_to_paged_multi_layer(kl.cuda(), vl.cuda(), dk, dv, slots.cuda())
        rk, rv = to_np(kc).copy(), to_np(vc).copy()
        O.kv_linear_to_paged_multi_layer(to_np(kl), to_np(vl), rk, rv, slots.numpy())
        eq(dk, rk, f"scatter k t={t}")
        eq(dv, rv, f"scatter v t={t}")
        ok, ov = ma.kv_paged_to_linear_multi_layer(dk, dv, slots.cuda())
        qk, qv = O.kv_paged_to_linear_multi_layer(rk, rv, slots.numpy())
        eq(ok, qk, f"gather k t={t}")
        eq(ov, qv, f"gather v t={t}")
