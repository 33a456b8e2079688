"""Pin the CPU oracle to the reference: replay the golden vectors (recorded by
running the reference itself, see tests/golden/make_golden.py) through
``oracle.kv_oracle`` and require bit-identical results."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import kv_oracle as O

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


def same_bits(a: np.ndarray, b: np.ndarray) -> bool:
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    return a.shape == b.shape and a.dtype.itemsize == b.dtype.itemsize and a.tobytes() == b.tobytes()


@pytest.mark.parametrize("dt", DTYPES)
def test_tile_gather_scatter(tile, dt):
    p = f"gather/{dt}"
    ok, ov = O.kv_paged_to_linear(tile[f"{p}/k_cache"], tile[f"{p}/v_cache"], tile[f"{p}/slots"])
    assert same_bits(ok, tile[f"{p}/out_k"]) and same_bits(ov, tile[f"{p}/out_v"])
    pk = np.full_like(ok, 0)
    pv = np.full_like(ov, 0)
    pk[...] = O.from_f32(np.full(pk.shape, 3.0, np.float32), dt)
    pv[...] = O.from_f32(np.full(pv.shape, -2.0, np.float32), dt)
    O.kv_paged_to_linear(tile[f"{p}/k_cache"], tile[f"{p}/v_cache"], tile[f"{p}/slots"], fill_skipped="preserve", out_k=pk, out_v=pv)
    assert same_bits(pk, tile[f"{p}/preserve_k"]) and same_bits(pv, tile[f"{p}/preserve_v"])

    q = f"scatter/{dt}"
    kd = np.zeros_like(tile[f"{p}/k_cache"])
    vd = np.zeros_like(tile[f"{p}/v_cache"])
    vd[...] = O.from_f32(np.full(vd.shape, 1.5, np.float32), dt)
    O.kv_linear_to_paged(tile[f"{q}/k_lin"], tile[f"{q}/v_lin"], kd, vd, tile[f"{q}/slots"])
    assert same_bits(kd, tile[f"{q}/k_cache"]) and same_bits(vd, tile[f"{q}/v_cache"])


@pytest.mark.parametrize("dt", DTYPES)
def test_tile_multi_layer_and_merged(tile, dt):
    r = f"gather_ml/{dt}"
    ok, ov = O.kv_paged_to_linear_multi_layer(tile[f"{r}/k_cache"], tile[f"{r}/v_cache"], tile[f"{r}/slots"])
    assert same_bits(ok, tile[f"{r}/out_k"]) and same_bits(ov, tile[f"{r}/out_v"])
    merged_ml = np.stack([ok, ov], axis=2)
    assert same_bits(merged_ml, tile[f"merged/{dt}/gather_ml"])
    g = f"gather/{dt}"
    k1, v1 = O.kv_paged_to_linear(tile[f"{g}/k_cache"], tile[f"{g}/v_cache"], tile[f"{g}/slots"])
    assert same_bits(np.stack([k1, v1], axis=1), tile[f"merged/{dt}/gather"])

    s = f"scatter_ml/{dt}"
    kd = np.zeros_like(tile[f"{r}/k_cache"])
    vd = np.zeros_like(tile[f"{r}/v_cache"])
    O.kv_linear_to_paged_multi_layer(tile[f"{s}/k_lin"], tile[f"{s}/v_lin"], kd, vd, tile[f"{s}/slots"])
    assert same_bits(kd, tile[f"{s}/k_cache"]) and same_bits(vd, tile[f"{s}/v_cache"])

    m_in = tile[f"merged/{dt}/scatter_in"]
    kd = np.zeros_like(tile[f"{g}/k_cache"])
    vd = np.zeros_like(tile[f"{g}/v_cache"])
    O.kv_linear_to_paged(m_in[:, 0], m_in[:, 1], kd, vd, tile[f"scatter/{dt}/slots"])
    assert same_bits(kd, tile[f"merged/{dt}/scatter_k"]) and same_bits(vd, tile[f"merged/{dt}/scatter_v"])


def _enc_case(fp8, key, fmt, lin_dtype):
    kc = np.zeros_like(fp8[f"{key}/k_cache"])
    vc = np.zeros_like(fp8[f"{key}/v_cache"])
    O.kv_linear_to_paged_fp8(
        fp8[f"{key}/k_lin"], fp8[f"{key}/v_lin"], kc, vc, fp8[f"{key}/slots"],
        fp8[f"{key}/k_scale"], fp8[f"{key}/v_scale"], fp8_format=fmt, lin_dtype=lin_dtype,
    )
    assert same_bits(kc, fp8[f"{key}/k_cache"]), key
    assert same_bits(vc, fp8[f"{key}/v_cache"]), key


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
def test_fp8_encode_exhaustive(fp8, fmt):
    for i in range(2):
        _enc_case(fp8, f"enc_bf16/{fmt}/{i}", fmt, "bfloat16")
    _enc_case(fp8, f"enc_f16/{fmt}/0", fmt, "float16")
    _enc_case(fp8, f"enc_f32/{fmt}/0", fmt, "float32")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", DTYPES)
def test_fp8_decode_all_codes(fp8, fmt, dt):
    for j in range(2):
        p = f"dec/{fmt}/{dt}/{j}"
        ok, ov = O.kv_paged_fp8_to_linear(
            fp8["dec/k_cache"], fp8["dec/v_cache"], fp8["dec/slots"], fp8[f"{p}/k_scale"], fp8[f"{p}/v_scale"],
            out_dtype=dt, fp8_format=fmt,
        )
        assert same_bits(ok, fp8[f"{p}/out_k"]) and same_bits(ov, fp8[f"{p}/out_v"]), p


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", DTYPES)
def test_fp8_multi_layer(fp8, fmt, dt):
    p = f"ml/{fmt}/{dt}"
    kc = np.zeros_like(fp8[f"{p}/k_cache"])
    vc = np.zeros_like(fp8[f"{p}/v_cache"])
    O.kv_linear_to_paged_fp8_multi_layer(
        fp8[f"{p}/k_lin"], fp8[f"{p}/v_lin"], kc, vc, fp8["ml/slots"], fp8[f"{p}/k_scale"], fp8[f"{p}/v_scale"],
        fp8_format=fmt, lin_dtype=dt,
    )
    assert same_bits(kc, fp8[f"{p}/k_cache"]) and same_bits(vc, fp8[f"{p}/v_cache"])
    ok, ov = O.kv_paged_fp8_to_linear_multi_layer(
        fp8[f"{p}/k_cache"], fp8[f"{p}/v_cache"], fp8["ml/slots"], fp8[f"{p}/k_scale"], fp8[f"{p}/v_scale"],
        out_dtype=dt, fp8_format=fmt,
    )
    assert same_bits(ok, fp8[f"{p}/out_k"]) and same_bits(ov, fp8[f"{p}/out_v"])


@pytest.mark.parametrize("dt", DTYPES)
def test_lmcache_rows(rows, dt):
    gs, ss = rows["gslots"], rows["sslots"]
    # 6-D
    p = f"six_d/{dt}"
    paged = rows[f"{p}/paged"]
    buf = np.zeros_like(rows[f"{p}/gather"])
    O.lmcache_paged_to_kv_buffer(paged, buf, gs)
    assert same_bits(buf, rows[f"{p}/gather"])
    dst = np.empty_like(rows[f"{p}/scatter_dst"])
    dst[...] = O.from_f32(np.full(dst.shape, 0.25, np.float32), dt)
    O.lmcache_kv_buffer_to_paged(rows[f"{p}/scatter_src"], dst, ss)
    assert same_bits(dst, rows[f"{p}/scatter_dst"])
    # list
    p = f"list/{dt}"
    caches = list(rows[f"{p}/caches"])
    mem = np.empty_like(rows[f"{p}/gather"])
    mem[...] = O.from_f32(np.full(mem.shape, 9.0, np.float32), dt)
    O.lmcache_list_paged_to_buffer(caches, mem, gs)
    assert same_bits(mem, rows[f"{p}/gather"])
    dcaches = [np.zeros_like(c) for c in caches]
    O.lmcache_list_buffer_to_paged(rows[f"{p}/scatter_src"], dcaches, ss, skip_prefix=2)
    assert same_bits(np.stack(dcaches), rows[f"{p}/scatter_dst"])
    # two_x_nl
    p = f"two_x_nl/{dt}"
    two = [list(x) for x in rows[f"{p}/caches"]]
    mem = np.zeros_like(rows[f"{p}/gather"])
    O.lmcache_two_x_nl_paged_to_buffer(two, mem, gs)
    assert same_bits(mem, rows[f"{p}/gather"])
    dtwo = [[np.empty_like(c) for c in x] for x in two]
    for x in dtwo:
        for c in x:
            c[...] = O.from_f32(np.full(c.shape, -1.0, np.float32), dt)
    O.lmcache_two_x_nl_buffer_to_paged(rows[f"{p}/scatter_src"], dtwo, ss, skip_prefix=1)
    assert same_bits(np.stack([np.stack(x) for x in dtwo]), rows[f"{p}/scatter_dst"])


@pytest.mark.parametrize("dt", DTYPES)
def test_mla_rows(rows, dt):
    gs, ss = rows["gslots"], rows["sslots"]
    p = f"mla/{dt}"
    buf = np.zeros_like(rows[f"{p}/gather"])
    O.lmcache_paged_to_kv_buffer_mla(rows[f"{p}/paged"], buf, gs)
    assert same_bits(buf, rows[f"{p}/gather"])
    dst = np.zeros_like(rows[f"{p}/scatter_dst"])
    O.lmcache_kv_buffer_to_paged_mla(rows[f"{p}/scatter_src"], dst, ss)
    assert same_bits(dst, rows[f"{p}/scatter_dst"])
    p = f"mla_list/{dt}"
    caches = list(rows[f"{p}/caches"])
    mem = np.zeros_like(rows[f"{p}/gather"])
    O.lmcache_mla_paged_to_buffer(caches, mem, gs)
    assert same_bits(mem, rows[f"{p}/gather"])
    dl = [np.zeros_like(c) for c in caches]
    O.lmcache_mla_buffer_to_paged(rows[f"{p}/scatter_src"], dl, ss, skip_prefix=1)
    assert same_bits(np.stack(dl), rows[f"{p}/scatter_dst"])
    p = f"mla_flat/{dt}"
    kvc, pec = rows[f"{p}/kv_cache"], rows[f"{p}/pe_cache"]
    okv, ope = O.kv_paged_to_mla_linear(kvc[0], pec[0], gs)
    assert same_bits(okv, rows[f"{p}/gather_kv"]) and same_bits(ope, rows[f"{p}/gather_pe"])
    okv3 = np.stack([O.kv_paged_to_mla_linear(kvc[i], pec[i], gs)[0] for i in range(kvc.shape[0])])
    ope3 = np.stack([O.kv_paged_to_mla_linear(kvc[i], pec[i], gs)[1] for i in range(kvc.shape[0])])
    assert same_bits(okv3, rows[f"{p}/gather_ml_kv"]) and same_bits(ope3, rows[f"{p}/gather_ml_pe"])
    dkv = np.zeros_like(kvc)
    dpe = np.zeros_like(pec)
    for i in range(kvc.shape[0]):
        O.kv_mla_linear_to_paged(rows[f"{p}/scatter_kv_in"][i], rows[f"{p}/scatter_pe_in"][i], dkv[i], dpe[i], ss)
    assert same_bits(dkv, rows[f"{p}/scatter_kv"]) and same_bits(dpe, rows[f"{p}/scatter_pe"])


def test_last_writer_mask_matches_sequential_loop():
    rng = np.random.default_rng(3)
    slots = rng.integers(-3, 20, size=500)
    keep = O.last_writer_mask(slots)
    seen = {}
    for t, s in enumerate(slots):
        if s >= 0:
            seen[int(s)] = t
    expected = np.zeros_like(keep)
    expected[list(seen.values())] = True
    assert np.array_equal(keep, expected)


@pytest.fixture(scope="module")
def misc():
    return np.load(GOLDEN / "misc.npz")


@pytest.mark.parametrize("dt", DTYPES)
def test_flash_triton_blocks(misc, dt):
    p = f"flash/{dt}"
    bt, lens = misc["flash/block_tables"], misc["flash/seq_lens"]
    ok, ov = O.kv_load_and_reshape_flash(misc[f"{p}/k_cache"], misc[f"{p}/v_cache"], bt, lens, max_seq_len=15)
    assert same_bits(ok, misc[f"{p}/out_k"]) and same_bits(ov, misc[f"{p}/out_v"])
    kd, vd = misc[f"{p}/k_cache"].copy(), misc[f"{p}/v_cache"].copy()
    O.kv_reshape_and_cache_back_flash(misc[f"{p}/dense_k"], misc[f"{p}/dense_v"], kd, vd, bt, lens)
    assert same_bits(kd, misc[f"{p}/back_k"]) and same_bits(vd, misc[f"{p}/back_v"])
    q = f"triton/{dt}"
    tk, tv = O.kv_triton_indexed_to_dense(misc[f"{q}/pool_k"], misc[f"{q}/pool_v"], misc["triton/indptr"], misc[f"{q}/indices"], 9)
    assert same_bits(tk, misc[f"{q}/out_k"]) and same_bits(tv, misc[f"{q}/out_v"])
    r = f"blocks/{dt}"
    dk = np.zeros_like(misc[f"{r}/dst_k"])
    dv = np.zeros_like(misc[f"{r}/dst_v"])
    n = O.kv_copy_paged_blocks(misc[f"{r}/src_k"], misc[f"{r}/src_v"], dk, dv, misc["blocks/pairs"])
    assert n == int(misc[f"{r}/count"]) and same_bits(dk, misc[f"{r}/dst_k"]) and same_bits(dv, misc[f"{r}/dst_v"])
    dk1 = np.zeros_like(misc[f"{r}/dst1_k"])
    dv1 = np.zeros_like(misc[f"{r}/dst1_v"])
    n1 = O.kv_copy_paged_blocks(misc[f"{r}/src_k"][0], misc[f"{r}/src_v"][0], dk1, dv1, misc["blocks/pairs"])
    assert n1 == int(misc[f"{r}/count1"]) and same_bits(dk1, misc[f"{r}/dst1_k"]) and same_bits(dv1, misc[f"{r}/dst1_v"])


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
def test_fp8_flash(misc, fmt):
    ok, ov = O.kv_load_and_dequantize_fp8_flash(misc["fp8flash/k8"], misc["fp8flash/v8"], misc["fp8flash/bt"],
                                                misc["fp8flash/lens"], np.float32(0.03), np.array([0.5, 0.25], np.float32),
                                                out_dtype="bfloat16", fp8_format=fmt)
    assert same_bits(ok, misc[f"fp8flash/{fmt}/out_k"]) and same_bits(ov, misc[f"fp8flash/{fmt}/out_v"])


def test_rows_and_hicache(misc):
    for width in (1, 24, 1729):
        d = misc[f"rows/{width}/dst"].copy()
        O.kv_copy_paged_rows(misc[f"rows/{width}/src"], d, misc["rows/si"], misc["rows/di"])
        assert same_bits(d, misc[f"rows/{width}/out"]), width
    lf_k, lf_v, pf_k, pf_v = misc["hicache/lf_k"], misc["hicache/lf_v"], misc["hicache/pf_k"], misc["hicache/pf_v"]
    si, di = misc["hicache/si"], misc["hicache/di"]
    cases = {
        "per_layer": (lf_k, lf_v, "layer_first", "layer_first", 1, 1, lf_k.shape),
        "per_layer_pf_lf": (pf_k, pf_v, "page_first", "layer_first", 2, 1, lf_k.shape),
        "all_layer": (lf_k, lf_v, "layer_first", "layer_first", 0, 3, lf_k.shape),
        "all_layer_lf_pf": (lf_k, lf_v, "layer_first", "page_first", 0, 3, pf_k.shape),
        "mla_per_layer": (lf_k, None, "layer_first", "layer_first", 0, 1, lf_k.shape),
        "mla_pf_lf": (pf_k, None, "page_first", "layer_first", 1, 1, lf_k.shape),
        "mla_all": (lf_k, None, "layer_first", "layer_first", 0, 3, lf_k.shape),
        "mla_all_lf_pf": (lf_k, None, "layer_first", "page_first", 0, 3, pf_k.shape),
    }
    for key, (sk, sv, sl, dl, start, num, dshape) in cases.items():
        dk = np.zeros(dshape, np.float16)
        dv = np.zeros(dshape, np.float16) if sv is not None else None
        O.hicache_transfer(sk, dk, sv, dv, si, di, sl, dl, start, num)
        assert same_bits(dk, misc[f"hicache/out/{key}/0"]), key
        if sv is not None:
            assert same_bits(dv, misc[f"hicache/out/{key}/1"]), key
    src = list(misc["hicache/direct/src"])
    dst = [np.zeros((20, 2, 8), np.uint16) for _ in range(2)]
    O.hicache_direct(src, dst, misc["hicache/direct/si"], misc["hicache/direct/di"], 4)
    assert same_bits(np.stack(dst), misc["hicache/direct/out"])


def test_cachegen(misc):
    for name, dt in (("f32_256", "float32"), ("bf16_256", "bfloat16"), ("f16_16", "float16"), ("f32_2", "float32"), ("const", "float32")):
        p = f"cachegen/{name}"
        x = O.to_f32(misc[f"{p}/x"], dt)
        bins = misc[f"{p}/codebook"].shape[0]
        enc, cb, cdf = O.kv_cachegen_encode(x, bins)
        assert same_bits(enc, misc[f"{p}/enc"]), name
        assert same_bits(cb, misc[f"{p}/codebook"]), name
        assert same_bits(cdf, misc[f"{p}/cdf"]), name
        if f"{p}/dec" in misc:
            assert same_bits(O.from_f32(O.kv_cachegen_decode(enc, cb), dt), misc[f"{p}/dec"]), name


@pytest.mark.parametrize("bins", (2, 17, 256))
def test_cachegen_magic_number_rounding_matches_rint_clamp(bins):
    """The encode kernel forms a code as clamp(q, 0, bins - 1) + 1.5 * 2^23 in fp32 and keeps the
    low mantissa bits (no rint / float-to-int conversion); the oracle rounds half to even and
    clamps.  Same codes for every quotient the kernel can meet: uniform values over and beyond the
    range, every half-integer and its fp32 neighbours, signed zero, infinities and NaN (which
    fmaxf, like numpy's fmax, drops to 0)."""
    rng = np.random.default_rng(bins)
    top = np.float32(bins - 1)
    halves = np.arange(-4, bins + 4, dtype=np.float32)[:, None] + np.float32(0.5)
    q = np.concatenate([
        rng.uniform(-3, bins + 3, 200_000).astype(np.float32),
        halves.ravel(),
        np.nextafter(halves, np.float32(-np.inf)).ravel(),
        np.nextafter(halves, np.float32(np.inf)).ravel(),
        np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 3e38, -3e38, 1e-45], dtype=np.float32),
    ])
    with np.errstate(invalid="ignore"):
        want = np.fmin(np.fmax(np.rint(q), np.float32(0)), top).astype(np.uint32)
        clamped = np.fmin(np.fmax(q, np.float32(0)), top).astype(np.float32)
        got = (clamped + np.float32(12582912.0)).astype(np.float32).view(np.uint32) - np.uint32(0x4B400000)
    assert np.array_equal(got, want)


# ---- MLA FP8 rows: the reference's element codec under per-128 group scales ----


@pytest.fixture(scope="module")
def mla_fp8():
    return np.load(GOLDEN / "mla_fp8.npz")


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
@pytest.mark.parametrize("dt", ("bfloat16", "float16"))
def test_mla_fp8_rows_codec(mla_fp8, dt, fmt):
    p = f"{dt}/{fmt}"
    x = mla_fp8[f"{p}/x"]
    x32 = O.to_f32(x, dt)
    scales = O.mla_fp8_group_scales(x32, fmt)
    assert scales.tobytes() == mla_fp8[f"{p}/scale"].tobytes()
    pe = np.zeros((x.shape[0], 64), dtype=x.dtype)
    rows = O.mla_fp8_encode_rows(x, pe, dt, fmt)
    assert rows.shape == (x.shape[0], O.mla_fp8_row_bytes(512, 64))
    assert np.array_equal(rows[:, :512], mla_fp8[f"{p}/codes"])
    cache = rows[None]
    kv, _ = O.mla_fp8_rows_load(cache, np.arange(x.shape[0]), kv_dim=512, pe_dim=64, out_dtype=dt, fp8_format=fmt)
    assert kv[0].tobytes() == mla_fp8[f"{p}/dec"].tobytes()


# ---- `cache` family: RoPE (per-operation rounding) and the KV-cache write -------


@pytest.fixture(scope="module")
def cache_g():
    return np.load(GOLDEN / "cache.npz")


CACHE_DT = ("float32", "float16", "bfloat16")


@pytest.mark.parametrize("inter", (0, 1))
@pytest.mark.parametrize("cn", CACHE_DT)
@pytest.mark.parametrize("xn", CACHE_DT)
def test_apply_rope_dtype_pairs(cache_g, xn, cn, inter):
    p = f"rope/{xn}/{cn}/{inter}"
    out = O.apply_rope(cache_g[f"{p}/x"], cache_g[f"{p}/cos"], cache_g[f"{p}/sin"], x_dtype=xn, cos_dtype=cn,
                       sin_dtype=cn, interleaved=bool(inter))
    assert out.tobytes() == cache_g[f"{p}/out"].tobytes()


def test_apply_rope_mixed_and_growing_broadcast(cache_g):
    out = O.apply_rope(cache_g["rope_mixed/x"], cache_g["rope_mixed/cos"], cache_g["rope_mixed/sin"],
                       x_dtype="bfloat16", cos_dtype="float16", sin_dtype="float32")
    assert out.shape == cache_g["rope_mixed/out"].shape
    assert out.tobytes() == cache_g["rope_mixed/out"].tobytes()


@pytest.mark.parametrize("cn", CACHE_DT)
def test_rope_key_cache_and_copy(cache_g, cn):
    p = f"rope_cache/{cn}"
    kc = cache_g[f"{p}/cache_in"].copy()
    O.apply_rope_to_key_cache(kc, cache_g[f"{p}/slots"], cache_g[f"{p}/positions"], cache_g[f"{p}/cos"],
                              cache_g[f"{p}/sin"], cache_dtype=cn, cos_dtype=cn, sin_dtype=cn)
    assert kc.tobytes() == cache_g[f"{p}/cache_out"].tobytes()
    kc = cache_g[f"{p}/cache_in"].copy()
    O.apply_rope_to_key_cache(kc, cache_g[f"{p}/slots"], cache_g[f"{p}/positions"], cache_g[f"{p}/cos"][4],
                              cache_g[f"{p}/sin"][4], cache_dtype=cn, cos_dtype=cn, sin_dtype=cn, interleaved=True)
    assert kc.tobytes() == cache_g[f"{p}/cache_out_1d_inter"].tobytes()
    q = f"copy/{cn}"
    kcc = np.zeros_like(cache_g[f"{q}/kc"])
    vcc = np.zeros_like(cache_g[f"{q}/vc"])
    O.copy_to_kv_cache(cache_g[f"{q}/k"], cache_g[f"{q}/v"], kcc, vcc, cache_g[f"{q}/slots"])
    assert kcc.tobytes() == cache_g[f"{q}/kc"].tobytes() and vcc.tobytes() == cache_g[f"{q}/vc"].tobytes()


@pytest.fixture(scope="module")
def merged_fp8():
    return np.load(GOLDEN / "merged_fp8.npz")


def _merged_fp8_keys(g):
    """(block size, format, input dtype, scale form) of every case in merged_fp8.npz."""
    return sorted({tuple(k.split("/")[:4]) for k in g.files if k.count("/") == 4})


def test_merged_fp8_store_and_load(merged_fp8):
    g = merged_fp8
    cases = _merged_fp8_keys(g)
    assert len(cases) == 2 * 2 * 2 * 5, cases  # bs x format x dtype x (2 single + 3 multi-layer scale forms)
    for bs, fmt, dt, form in cases:
        p = f"{bs}/{fmt}/{dt}/{form}"
        slots, gslots = g[f"{bs}/slots"], g[f"{bs}/gslots"]
        kc = np.zeros_like(g[f"{p}/k_cache"])
        vc = np.zeros_like(g[f"{p}/v_cache"])
        ks, vs = g[f"{p}/k_scale"], g[f"{p}/v_scale"]
        if form.startswith("ml_"):
            O.kv_merged_linear_to_paged_fp8_multi_layer(g[f"{p}/merged"], kc, vc, slots, ks, vs, fp8_format=fmt, lin_dtype=dt)
            out = O.kv_paged_fp8_to_merged_linear_multi_layer(kc, vc, gslots, ks, vs, out_dtype=dt, fp8_format=fmt)
        else:
            O.kv_merged_linear_to_paged_fp8(g[f"{p}/merged"], kc, vc, slots, ks, vs, fp8_format=fmt, lin_dtype=dt)
            out = O.kv_paged_fp8_to_merged_linear(kc, vc, gslots, ks, vs, out_dtype=dt, fp8_format=fmt)
        assert same_bits(kc, g[f"{p}/k_cache"]) and same_bits(vc, g[f"{p}/v_cache"]), p
        assert same_bits(out, g[f"{p}/gather"]), p


def test_multi_pool_rows():
    g = np.load(GOLDEN / "pools.npz")
    idx = g["indices"]
    for direction in ("H2D", "D2H"):
        n = len({k.split("/")[1] for k in g.files if k.startswith(direction)})
        pools = [(list(g[f"{direction}/{p}/src"]), [d.copy() for d in g[f"{direction}/{p}/dst_in"]]) for p in range(n)]
        O.kv_copy_paged_rows_multi_pool(pools, idx)
        for p, (_, dsts) in enumerate(pools):
            assert same_bits(np.stack(dsts), g[f"{direction}/{p}/dst_out"]), (direction, p)
