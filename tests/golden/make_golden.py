"""Generate golden vectors for the kvcache oracle by running the reference itself.

Usage (in a container that holds the reference source tree)::

    MUSA_AITER_REF=/path/to/musa-aiter python tests/golden/make_golden.py

The script imports the reference ``musa_aiter`` package (pure PyTorch on CPU),
feeds it seeded inputs and stores inputs + outputs in ``tests/golden/*.npz``.
``tests/test_oracle_golden.py`` replays every case through ``oracle.kv_oracle``
and requires bit-identical results.  bfloat16 tensors are stored as uint16 bit
patterns, FP8 caches as raw uint8.

Families:
- tile.npz    kv_paged_to_linear / kv_linear_to_paged (+ multi-layer, merged)
- fp8.npz     exhaustive FP8 encode (all 65536 bf16 and fp16 inputs), edge fp32
              inputs, all 256 codes decoded, multi-layer scale forms
- rows.npz    LMCache 6-D / list / SGLang MP two_x_nl / MLA buffers, MLA flat caches
- misc.npz    Flash dense load / cache-back / FP8 dequant, Triton-indexed dense gather,
              block copies, DSV4 byte rows, HiCache transfers, CacheGen codec
- mla_fp8.npz MLA latent rows encoded / decoded by the reference's FP8 element codec
              (``_fp8_quantize_to_uint8`` / ``_fp8_dequantize_from_uint8``) with per-128
              group scales amax/fp8_max (the group rule is this build's choice)

- cache.npz   apply_rope (dtype pairs, interleaved, broadcast shapes), apply_rope_to_key_cache
              (1-D and 2-D tables, repeated slots), copy_to_kv_cache
- merged_fp8.npz  FP8 merged store / load, single and multi-layer, e4m3 / e5m2, scalar /
              [NH] / [L, NH] scales, block_size 16 and 4, negative and duplicate slots
- pools.npz   DSV4 multi-pool page-row copy, both directions, four pools of different widths

``python tests/golden/make_golden.py mla_fp8`` regenerates one family only.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np

sys.dont_write_bytecode = True
REF = os.environ.get("MUSA_AITER_REF")
if not REF:
    raise SystemExit("set MUSA_AITER_REF to the reference musa-aiter source tree")
if REF not in sys.path:
    sys.path.insert(0, REF)

import torch  # noqa: E402

import musa_aiter as ref  # noqa: E402  (the reference package, not this repo's)

assert str(Path(ref.__file__).resolve()).startswith(str(Path(REF).resolve())), ref.__file__

OUT = Path(__file__).resolve().parent


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
        return t.view(torch.uint8).numpy()
    return t.numpy()


class Store:
    def __init__(self) -> None:
        self.d: dict[str, np.ndarray] = {}

    def put(self, key: str, value) -> None:
        assert key not in self.d, key
        if isinstance(value, torch.Tensor):
            value = to_np(value)
        self.d[key] = np.asarray(value)

    def save(self, name: str) -> None:
        np.savez_compressed(OUT / name, **self.d)
        print(f"wrote {name}: {len(self.d)} arrays")


def gen(seed: int) -> torch.Generator:
    g = torch.Generator()
    g.manual_seed(seed)
    return g


def randn(shape, dtype, g):
    return torch.randn(shape, generator=g, dtype=torch.float32).to(dtype)


DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


# ---------------------------------------------------------------------------
def make_tile() -> None:
    st = Store()
    nb, nh, hd, bs = 5, 2, 8, 4
    for dname, dt in DTYPES.items():
        g = gen(10)
        kc = randn((nb, nh, hd, bs), dt, g)
        vc = randn((nb, nh, hd, bs), dt, g)
        slots = torch.tensor([0, 5, 19, -1, 7, 3, -4, 12, 13, 14, 15, 16], dtype=torch.int64)
        p = f"gather/{dname}"
        st.put(f"{p}/k_cache", kc)
        st.put(f"{p}/v_cache", vc)
        st.put(f"{p}/slots", slots)
        ok, ov = ref.kv_paged_to_linear(kc, vc, slots)
        st.put(f"{p}/out_k", ok)
        st.put(f"{p}/out_v", ov)
        # preserve mode into prefilled buffers
        pk = torch.full((slots.numel(), nh, hd), 3.0, dtype=dt)
        pv = torch.full((slots.numel(), nh, hd), -2.0, dtype=dt)
        ref.kv_paged_to_linear(kc, vc, slots, fill_skipped="preserve", out_k=pk, out_v=pv)
        st.put(f"{p}/preserve_k", pk)
        st.put(f"{p}/preserve_v", pv)
        # scatter with duplicate slots (last writer wins) and negative slots
        sslots = torch.tensor([3, 9, -1, 3, 17, 0, 9, 19, -2, 3], dtype=torch.int32)
        kl = randn((sslots.numel(), nh, hd), dt, g)
        vl = randn((sslots.numel(), nh, hd), dt, g)
        kd = torch.zeros_like(kc)
        vd = torch.full_like(vc, 1.5)
        ref.kv_linear_to_paged(kl, vl, kd, vd, sslots)
        q = f"scatter/{dname}"
        st.put(f"{q}/k_lin", kl)
        st.put(f"{q}/v_lin", vl)
        st.put(f"{q}/slots", sslots)
        st.put(f"{q}/k_cache", kd)
        st.put(f"{q}/v_cache", vd)
        # multi-layer gather + scatter
        nl = 3
        kc3 = randn((nl, nb, nh, hd, bs), dt, g)
        vc3 = randn((nl, nb, nh, hd, bs), dt, g)
        ok3, ov3 = ref.kv_paged_to_linear_multi_layer(kc3, vc3, slots)
        r = f"gather_ml/{dname}"
        st.put(f"{r}/k_cache", kc3)
        st.put(f"{r}/v_cache", vc3)
        st.put(f"{r}/slots", slots)
        st.put(f"{r}/out_k", ok3)
        st.put(f"{r}/out_v", ov3)
        kl3 = randn((nl, sslots.numel(), nh, hd), dt, g)
        vl3 = randn((nl, sslots.numel(), nh, hd), dt, g)
        kd3 = torch.zeros_like(kc3)
        vd3 = torch.zeros_like(vc3)
        ref.kv_linear_to_paged_multi_layer(kl3, vl3, kd3, vd3, sslots)
        r = f"scatter_ml/{dname}"
        st.put(f"{r}/k_lin", kl3)
        st.put(f"{r}/v_lin", vl3)
        st.put(f"{r}/slots", sslots)
        st.put(f"{r}/k_cache", kd3)
        st.put(f"{r}/v_cache", vd3)
        # merged layouts
        merged = ref.kv_paged_to_merged_linear(kc, vc, slots)
        st.put(f"merged/{dname}/gather", merged)
        merged_ml = ref.kv_paged_to_merged_linear_multi_layer(kc3, vc3, slots)
        st.put(f"merged/{dname}/gather_ml", merged_ml)
        ml_in = randn((sslots.numel(), 2, nh, hd), dt, g)
        kd = torch.zeros_like(kc)
        vd = torch.zeros_like(vc)
        ref.kv_merged_linear_to_paged(ml_in, kd, vd, sslots)
        st.put(f"merged/{dname}/scatter_in", ml_in)
        st.put(f"merged/{dname}/scatter_k", kd)
        st.put(f"merged/{dname}/scatter_v", vd)
    st.save("tile.npz")


# ---------------------------------------------------------------------------
def _fp8_store(st: Store, key: str, k_lin, v_lin, nb, bs, k_scale, v_scale, fmt, slots=None):
    t, nh, hd = k_lin.shape
    kc = torch.zeros((nb, nh, hd, bs), dtype=torch.uint8)
    vc = torch.zeros((nb, nh, hd, bs), dtype=torch.uint8)
    if slots is None:
        slots = torch.arange(t, dtype=torch.int64)
    ref.kv_linear_to_paged_fp8(k_lin, v_lin, kc, vc, slots, k_scale, v_scale, fp8_format=fmt)
    st.put(f"{key}/k_lin", k_lin)
    st.put(f"{key}/v_lin", v_lin)
    st.put(f"{key}/slots", slots)
    st.put(f"{key}/k_scale", torch.as_tensor(k_scale, dtype=torch.float32))
    st.put(f"{key}/v_scale", torch.as_tensor(v_scale, dtype=torch.float32))
    st.put(f"{key}/k_cache", kc)
    st.put(f"{key}/v_cache", vc)


def make_fp8() -> None:
    st = Store()
    all16 = torch.arange(65536, dtype=torch.int32).to(torch.int16)
    bf = all16.view(torch.bfloat16).reshape(512, 4, 32)
    hf = all16.view(torch.float16).reshape(512, 4, 32)
    scale_sets = [
        (1.0, [0.5, 1.0, 3.75, 0.0123]),
        (0.0371, [448.0 / 7.0, 2.0**-10, 1e-3, 117.0]),
    ]
    for fmt in ("e4m3", "e5m2"):
        for i, (ks, vs) in enumerate(scale_sets):
            _fp8_store(st, f"enc_bf16/{fmt}/{i}", bf, bf.flip(0), 32, 16, ks, vs, fmt)
        _fp8_store(st, f"enc_f16/{fmt}/0", hf, hf.flip(0), 32, 16, scale_sets[1][0], scale_sets[0][1], fmt)
    # fp32 edge values: specials, ties around the top codes and the min-normal boundaries
    specials = [0.0, -0.0, float("inf"), float("-inf"), float("nan"), 448.0, 464.0, 464.0001, 479.9, 480.0, 480.1,
                1e30, -1e30, 57344.0, 61439.996, 61440.0, 61440.004, 65536.0, 114688.0, 114687.9, 2e5,
                2.0**-6, 2.0**-6 * 0.99999994, 2.0**-7, 2.0**-14, 2.0**-14 * 0.99999994, 2.0**-15, 2.0**-9 * 1.5,
                0.3125, 0.34375, 1.0625, 1.125, 1.1875, 15.5, 240.0, 248.0, 256.0, 3.0e-5]
    g = gen(20)
    mags = torch.exp2(torch.rand(4096 - 2 * len(specials), generator=g) * 60.0 - 30.0)
    signs = torch.where(torch.rand(mags.numel(), generator=g) < 0.5, -1.0, 1.0)
    vals = torch.cat([torch.tensor(specials), -torch.tensor(specials), mags * signs]).to(torch.float32)
    x32 = vals.reshape(32, 4, 32)
    for fmt in ("e4m3", "e5m2"):
        _fp8_store(st, f"enc_f32/{fmt}/0", x32, x32 * 3.0, 2, 16, 1.0, [1.0, 0.5, 2.0, 1.0 / 3.0], fmt)
    # decode every code: cache holds codes 0..255 at slots 0..255 for [NB=16, NH=1, HD=16, BS=16]
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8)
    nb, nh, hd, bs = 4, 2, 8, 16
    cache = codes.repeat(4).reshape(nb, nh, hd, bs).contiguous()
    slots = torch.tensor([0, 1, 2, 3, -1, 17, 18, 33, 60, 63, 47, -3], dtype=torch.int64)
    for fmt in ("e4m3", "e5m2"):
        for oname, odt in DTYPES.items():
            for j, (ks, vs) in enumerate([(1.0, [0.25, 3.0]), (0.0371, 1.7)]):
                ok, ov = ref.kv_paged_fp8_to_linear(cache, cache.flip(0).contiguous(), slots, ks, vs, out_dtype=odt, fp8_format=fmt)
                p = f"dec/{fmt}/{oname}/{j}"
                st.put(f"{p}/k_scale", torch.as_tensor(ks, dtype=torch.float32))
                st.put(f"{p}/v_scale", torch.as_tensor(vs, dtype=torch.float32))
                st.put(f"{p}/out_k", ok)
                st.put(f"{p}/out_v", ov)
    st.put("dec/k_cache", cache)
    st.put("dec/v_cache", cache.flip(0).contiguous())
    st.put("dec/slots", slots)
    # multi-layer: [L, NH] scales, duplicates and negative slots, bf16 and fp16 input
    nl, nb, nh, hd, bs = 3, 4, 2, 16, 16
    sl = torch.tensor([5, 6, 7, -1, 5, 40, 63, 0, 1, 2, 3, 4, 8, 9, 10, 11, 12, 13, 14, 15], dtype=torch.int64)
    for fmt in ("e4m3", "e5m2"):
        for lname, ldt in (("bfloat16", torch.bfloat16), ("float16", torch.float16), ("float32", torch.float32)):
            g = gen(30)
            kl = (randn((nl, sl.numel(), nh, hd), torch.float32, g) * 2.0).to(ldt)
            vl = (randn((nl, sl.numel(), nh, hd), torch.float32, g) * 2.0).to(ldt)
            ks = torch.rand((nl, nh), generator=g) * 0.02 + 0.001
            vs = 0.0173
            kc = torch.zeros((nl, nb, nh, hd, bs), dtype=torch.uint8)
            vc = torch.zeros((nl, nb, nh, hd, bs), dtype=torch.uint8)
            ref.kv_linear_to_paged_fp8_multi_layer(kl, vl, kc, vc, sl, ks, vs, fp8_format=fmt)
            p = f"ml/{fmt}/{lname}"
            st.put(f"{p}/k_lin", kl)
            st.put(f"{p}/v_lin", vl)
            st.put(f"{p}/k_scale", ks)
            st.put(f"{p}/v_scale", torch.tensor(vs, dtype=torch.float32))
            st.put(f"{p}/k_cache", kc)
            st.put(f"{p}/v_cache", vc)
            ok, ov = ref.kv_paged_fp8_to_linear_multi_layer(kc, vc, sl, ks, vs, out_dtype=ldt, fp8_format=fmt)
            st.put(f"{p}/out_k", ok)
            st.put(f"{p}/out_v", ov)
    st.put("ml/slots", sl)
    st.save("fp8.npz")


# ---------------------------------------------------------------------------
def make_rows() -> None:
    st = Store()
    nl, nb, bs, nh, hs = 3, 4, 4, 2, 8
    h = nh * hs
    gslots = torch.tensor([0, 3, 5, -1, 15, 7, 8, 9, 10, -2], dtype=torch.int64)
    sslots = torch.tensor([2, 14, -1, 2, 6, 0, 14, 11], dtype=torch.int64)
    for dname, dt in DTYPES.items():
        g = gen(40)
        # 6-D legacy layout
        paged = randn((nl, 2, nb, bs, nh, hs), dt, g)
        buf = torch.empty(2, nl, gslots.numel(), h, dtype=dt)
        ref.lmcache_paged_to_kv_buffer(paged, buf, gslots)
        p = f"six_d/{dname}"
        st.put(f"{p}/paged", paged)
        st.put(f"{p}/gather", buf)
        src = randn((2, nl, sslots.numel(), h), dt, g)
        dst = torch.full((nl, 2, nb, bs, nh, hs), 0.25, dtype=dt)
        ref.lmcache_kv_buffer_to_paged(src, dst, sslots)
        st.put(f"{p}/scatter_src", src)
        st.put(f"{p}/scatter_dst", dst)
        # list layout [2, NB, BS, NH, HS] per layer, memory with extra tail tokens
        caches = [randn((2, nb, bs, nh, hs), dt, g) for _ in range(nl)]
        mem = torch.full((2, nl, gslots.numel() + 3, h), 9.0, dtype=dt)
        ref.lmcache_kv_paged_to_buffer(caches, mem, gslots, bs, nh, hs)
        p = f"list/{dname}"
        st.put(f"{p}/caches", torch.stack(caches))
        st.put(f"{p}/gather", mem)
        msrc = randn((2, nl, sslots.numel() + 2, h), dt, g)
        dcaches = [torch.zeros((2, nb, bs, nh, hs), dtype=dt) for _ in range(nl)]
        ref.lmcache_kv_buffer_to_paged(msrc, dcaches, sslots, 2, bs, nh, hs)
        st.put(f"{p}/scatter_src", msrc)
        st.put(f"{p}/scatter_dst", torch.stack(dcaches))
        # SGLang MP 2 x NL x [NB, BS, NH, HS]
        two = [[randn((nb, bs, nh, hs), dt, g) for _ in range(nl)] for _ in range(2)]
        mem2 = torch.full((2, nl, gslots.numel(), h), 4.0, dtype=dt)
        ref.lmcache_kv_paged_to_buffer_two_x_nl(two, mem2, gslots, bs, nh, hs)
        p = f"two_x_nl/{dname}"
        st.put(f"{p}/caches", torch.stack([torch.stack(x) for x in two]))
        st.put(f"{p}/gather", mem2)
        msrc2 = randn((2, nl, sslots.numel() + 1, h), dt, g)
        dtwo = [[torch.full((nb, bs, nh, hs), -1.0, dtype=dt) for _ in range(nl)] for _ in range(2)]
        ref.lmcache_kv_buffer_to_paged_two_x_nl(msrc2, dtwo, sslots, 1, bs, nh, hs)
        st.put(f"{p}/scatter_src", msrc2)
        st.put(f"{p}/scatter_dst", torch.stack([torch.stack(x) for x in dtwo]))
        # MLA buffer [NL, T, HS] <-> [NL, NB, BS, HS]
        hsm = 12
        mpaged = randn((nl, nb, bs, hsm), dt, g)
        mbuf = torch.full((nl, gslots.numel(), hsm), 5.0, dtype=dt)
        ref.lmcache_paged_to_kv_buffer_mla(mpaged, mbuf, gslots)
        p = f"mla/{dname}"
        st.put(f"{p}/paged", mpaged)
        st.put(f"{p}/gather", mbuf)
        msrc3 = randn((nl, sslots.numel(), hsm), dt, g)
        mdst = torch.zeros((nl, nb, bs, hsm), dtype=dt)
        ref.lmcache_kv_buffer_to_paged_mla(msrc3, mdst, sslots)
        st.put(f"{p}/scatter_src", msrc3)
        st.put(f"{p}/scatter_dst", mdst)
        # MLA list [1, NL, T, HS] <-> list of [NB, BS, HS]
        mlist = [randn((nb, bs, hsm), dt, g) for _ in range(nl)]
        mmem = torch.full((1, nl, gslots.numel() + 2, hsm), 7.0, dtype=dt)
        ref.lmcache_mla_paged_to_buffer(mlist, mmem, gslots, bs, hsm)
        p = f"mla_list/{dname}"
        st.put(f"{p}/caches", torch.stack(mlist))
        st.put(f"{p}/gather", mmem)
        msrc4 = randn((1, nl, sslots.numel() + 1, hsm), dt, g)
        mldst = [torch.zeros((nb, bs, hsm), dtype=dt) for _ in range(nl)]
        ref.lmcache_mla_buffer_to_paged(msrc4, mldst, sslots, 1, bs, hsm)
        st.put(f"{p}/scatter_src", msrc4)
        st.put(f"{p}/scatter_dst", torch.stack(mldst))
        # MLA flat asymmetric caches (kv_dim 12, pe_dim 4), single and multi layer
        kvc = randn((nl, nb, bs, 12), dt, g)
        pec = randn((nl, nb, bs, 4), dt, g)
        okv, ope = ref.kv_paged_to_mla_linear(kvc[0], pec[0], gslots)
        p = f"mla_flat/{dname}"
        st.put(f"{p}/kv_cache", kvc)
        st.put(f"{p}/pe_cache", pec)
        st.put(f"{p}/gather_kv", okv)
        st.put(f"{p}/gather_pe", ope)
        okv3, ope3 = ref.kv_paged_to_mla_linear_multi_layer(kvc, pec, gslots)
        st.put(f"{p}/gather_ml_kv", okv3)
        st.put(f"{p}/gather_ml_pe", ope3)
        lkv = randn((nl, sslots.numel(), 12), dt, g)
        lpe = randn((nl, sslots.numel(), 4), dt, g)
        dkv = torch.zeros_like(kvc)
        dpe = torch.zeros_like(pec)
        ref.kv_mla_linear_to_paged_multi_layer(lkv, lpe, dkv, dpe, sslots)
        st.put(f"{p}/scatter_kv_in", lkv)
        st.put(f"{p}/scatter_pe_in", lpe)
        st.put(f"{p}/scatter_kv", dkv)
        st.put(f"{p}/scatter_pe", dpe)
    st.put("gslots", gslots)
    st.put("sslots", sslots)
    st.save("rows.npz")


def make_misc() -> None:
    st = Store()
    nb, nh, hd, bs = 12, 2, 8, 4
    for dname, dt in DTYPES.items():
        g = gen(50)
        kc = randn((nb, nh, hd, bs), dt, g)
        vc = randn((nb, nh, hd, bs), dt, g)
        bt = torch.tensor([[3, 7, 1, 0], [5, 2, 11, 9], [8, 4, 0, 0]], dtype=torch.int32)
        lens = torch.tensor([10, 13, 4], dtype=torch.int64)
        ok, ov = ref.kv_load_and_reshape_flash(kc, vc, bt, lens, max_seq_len=15)
        p = f"flash/{dname}"
        st.put(f"{p}/k_cache", kc)
        st.put(f"{p}/v_cache", vc)
        st.put(f"{p}/out_k", ok)
        st.put(f"{p}/out_v", ov)
        dk = randn((3, 15, nh, hd), dt, g)
        dv = randn((3, 15, nh, hd), dt, g)
        kd, vd = kc.clone(), vc.clone()
        ref.kv_reshape_and_cache_back_flash(dk, dv, kd, vd, bt, lens)
        st.put(f"{p}/dense_k", dk)
        st.put(f"{p}/dense_v", dv)
        st.put(f"{p}/back_k", kd)
        st.put(f"{p}/back_v", vd)
        # triton-indexed dense gather from a token pool
        pool_k = randn((40, nh, hd), dt, g)
        pool_v = randn((40, nh, hd), dt, g)
        indptr = torch.tensor([0, 5, 5, 17, 20], dtype=torch.int64)
        indices = torch.randperm(40, generator=g)[:20].to(torch.int32)
        tk, tv = ref.ops.kv_transfer.kv_triton_indexed_to_dense(pool_k, pool_v, indptr, indices, max_seq_len=9)
        q = f"triton/{dname}"
        st.put(f"{q}/pool_k", pool_k)
        st.put(f"{q}/pool_v", pool_v)
        st.put(f"{q}/indices", indices)
        st.put(f"{q}/out_k", tk)
        st.put(f"{q}/out_v", tv)
        # block copies, single and multi layer, with a duplicate destination and skipped pairs
        pairs = torch.tensor([[1, 4], [6, 0], [-1, 3], [2, 4], [9, -1], [11, 7]], dtype=torch.int64)
        src3 = randn((3, nb, nh, hd, bs), dt, g)
        srcv3 = randn((3, nb, nh, hd, bs), dt, g)
        dst3 = torch.zeros((3, 8, nh, hd, bs), dtype=dt)
        dstv3 = torch.zeros((3, 8, nh, hd, bs), dtype=dt)
        n3 = ref.kv_copy_paged_blocks(src3, srcv3, dst3, dstv3, pairs)
        r = f"blocks/{dname}"
        st.put(f"{r}/src_k", src3)
        st.put(f"{r}/src_v", srcv3)
        st.put(f"{r}/dst_k", dst3)
        st.put(f"{r}/dst_v", dstv3)
        st.put(f"{r}/count", torch.tensor(n3))
        d1k = torch.zeros((8, nh, hd, bs), dtype=dt)
        d1v = torch.zeros((8, nh, hd, bs), dtype=dt)
        n1 = ref.kv_copy_paged_blocks(src3[0], srcv3[0], d1k, d1v, pairs)
        st.put(f"{r}/dst1_k", d1k)
        st.put(f"{r}/dst1_v", d1v)
        st.put(f"{r}/count1", torch.tensor(n1))
    st.put("flash/block_tables", torch.tensor([[3, 7, 1, 0], [5, 2, 11, 9], [8, 4, 0, 0]], dtype=torch.int32))
    st.put("flash/seq_lens", torch.tensor([10, 13, 4], dtype=torch.int64))
    st.put("triton/indptr", torch.tensor([0, 5, 5, 17, 20], dtype=torch.int64))
    st.put("blocks/pairs", torch.tensor([[1, 4], [6, 0], [-1, 3], [2, 4], [9, -1], [11, 7]], dtype=torch.int64))
    # FP8 flash dequant
    g = gen(51)
    k8 = torch.randint(0, 256, (nb, nh, hd, 16), generator=g, dtype=torch.int32).to(torch.uint8)
    v8 = torch.randint(0, 256, (nb, nh, hd, 16), generator=g, dtype=torch.int32).to(torch.uint8)
    bt8 = torch.tensor([[3, 7], [5, 2], [8, 0]], dtype=torch.int64)
    lens8 = torch.tensor([20, 32, 5], dtype=torch.int64)
    for fmt in ("e4m3", "e5m2"):
        ok, ov = ref.kv_load_and_dequantize_fp8_flash(k8, v8, bt8, lens8, 0.03, [0.5, 0.25], out_dtype=torch.bfloat16, fp8_format=fmt)
        st.put(f"fp8flash/{fmt}/out_k", ok)
        st.put(f"fp8flash/{fmt}/out_v", ov)
    st.put("fp8flash/k8", k8)
    st.put("fp8flash/v8", v8)
    st.put("fp8flash/bt", bt8)
    st.put("fp8flash/lens", lens8)
    # DSV4 byte rows with odd widths and a duplicate destination
    for width in (1, 24, 1729):
        src = torch.randint(0, 256, (30, width), generator=g, dtype=torch.int32).to(torch.uint8)
        dst = torch.randint(0, 256, (25, width), generator=g, dtype=torch.int32).to(torch.uint8)
        si = torch.tensor([0, 5, 29, 7, 7, 13, 2], dtype=torch.int64)
        di = torch.tensor([3, 24, 0, 3, 11, 17, 8], dtype=torch.int32)
        d2 = dst.clone()
        ref.kv_copy_paged_rows(src, d2, si, di)
        st.put(f"rows/{width}/src", src)
        st.put(f"rows/{width}/dst", dst)
        st.put(f"rows/{width}/out", d2)
    st.put("rows/si", torch.tensor([0, 5, 29, 7, 7, 13, 2], dtype=torch.int64))
    st.put("rows/di", torch.tensor([3, 24, 0, 3, 11, 17, 8], dtype=torch.int32))
    # HiCache: layer-first / page-first, K+V and MLA, per-layer and all-layer
    L, P, item = 3, 10, 16
    hsrc_k = randn((L, P, item), torch.float16, g)
    hsrc_v = randn((L, P, item), torch.float16, g)
    hpf_k = randn((P, L, item), torch.float16, g)
    hpf_v = randn((P, L, item), torch.float16, g)
    si = torch.tensor([4, -1, 9, 0, 4], dtype=torch.int64)
    di = torch.tensor([1, 2, 7, 5, 3], dtype=torch.int64)
    st.put("hicache/lf_k", hsrc_k)
    st.put("hicache/lf_v", hsrc_v)
    st.put("hicache/pf_k", hpf_k)
    st.put("hicache/pf_v", hpf_v)
    st.put("hicache/si", si)
    st.put("hicache/di", di)
    outs = {}
    dk, dv = torch.zeros_like(hsrc_k), torch.zeros_like(hsrc_v)
    ref.hicache_transfer_kv_per_layer(hsrc_k, dk, hsrc_v, dv, si, di, layer_id=1)
    outs["per_layer"] = (dk, dv)
    dk, dv = torch.zeros_like(hsrc_k), torch.zeros_like(hsrc_v)
    ref.hicache_transfer_kv_per_layer_pf_lf(hpf_k, dk, hpf_v, dv, si, di, layer_id=2)
    outs["per_layer_pf_lf"] = (dk, dv)
    dk, dv = torch.zeros_like(hsrc_k), torch.zeros_like(hsrc_v)
    ref.hicache_transfer_kv_all_layer(hsrc_k, dk, hsrc_v, dv, si, di)
    outs["all_layer"] = (dk, dv)
    dk, dv = torch.zeros_like(hpf_k), torch.zeros_like(hpf_v)
    ref.hicache_transfer_kv_all_layer_lf_pf(hsrc_k, dk, hsrc_v, dv, si, di)
    outs["all_layer_lf_pf"] = (dk, dv)
    dm = torch.zeros_like(hsrc_k)
    ref.hicache_transfer_kv_per_layer_mla(hsrc_k, dm, si, di, layer_id=0)
    outs["mla_per_layer"] = (dm,)
    dm = torch.zeros_like(hsrc_k)
    ref.hicache_transfer_kv_per_layer_mla_pf_lf(hpf_k, dm, si, di, layer_id=1)
    outs["mla_pf_lf"] = (dm,)
    dm = torch.zeros_like(hsrc_k)
    ref.hicache_transfer_kv_all_layer_mla(hsrc_k, dm, si, di)
    outs["mla_all"] = (dm,)
    dm = torch.zeros_like(hpf_k)
    ref.hicache_transfer_kv_all_layer_mla_lf_pf(hsrc_k, dm, si, di)
    outs["mla_all_lf_pf"] = (dm,)
    for key, ts in outs.items():
        for j, t in enumerate(ts):
            st.put(f"hicache/out/{key}/{j}", t)
    # direct page ranges (page 4): note only each page's first index is used
    tok_src = [randn((24, 2, 8), torch.bfloat16, g) for _ in range(2)]
    tok_dst = [torch.zeros((20, 2, 8), dtype=torch.bfloat16) for _ in range(2)]
    dsi = torch.tensor([8, 9, 10, 11, 0, 1, 2, 3, 16, 99, 5, 5], dtype=torch.int64)
    ddi = torch.tensor([4, 5, 6, 7, 12, 13, 14, 15, 0, 0, 0, 0], dtype=torch.int64)
    ref.hicache_transfer_kv_direct(tok_src, tok_dst, dsi, ddi, 4)
    st.put("hicache/direct/src", torch.stack(tok_src))
    st.put("hicache/direct/out", torch.stack(tok_dst))
    st.put("hicache/direct/si", dsi)
    st.put("hicache/direct/di", ddi)
    # CacheGen codec
    for cname, (shape, cdt, bins) in {
        "f32_256": ((33, 7), torch.float32, 256),
        "bf16_256": ((5, 16, 9), torch.bfloat16, 256),
        "f16_16": ((64, 3), torch.float16, 16),
        "f32_2": ((17,), torch.float32, 2),
    }.items():
        x = (torch.randn(shape, generator=g) * 3.0 + 0.5).to(cdt)
        enc, cb, cdf = ref.kv_cachegen_encode(x, num_bins=bins)
        dec = ref.kv_cachegen_decode(enc, cb, dtype=cdt)
        p = f"cachegen/{cname}"
        st.put(f"{p}/x", x)
        st.put(f"{p}/enc", enc)
        st.put(f"{p}/codebook", cb)
        st.put(f"{p}/cdf", cdf)
        st.put(f"{p}/dec", dec)
    const = torch.full((4, 4), 2.5, dtype=torch.float32)
    enc, cb, cdf = ref.kv_cachegen_encode(const, num_bins=8)
    st.put("cachegen/const/x", const)
    st.put("cachegen/const/enc", enc)
    st.put("cachegen/const/codebook", cb)
    st.put("cachegen/const/cdf", cdf)
    st.save("misc.npz")


def make_mla_fp8() -> None:
    """Per-group FP8 rows: values, group scales (amax over the finite |x| of the group, / fp8_max
    in fp32), the reference's element encoder on x / scale, and its decoder times the stored scale."""
    from musa_aiter.ops import kv_transfer as rk  # the reference module

    st = Store()
    g = gen(40)
    t, kvd = 24, 512
    x = randn((t, kvd), torch.float32, g) * torch.exp2(torch.randint(-12, 12, (t, 1), generator=g).float())
    x[1, :128] = 0.0                                   # all-zero group -> scale 0
    x[2, 5] = float("nan")                             # NaN ignored by the group amax
    x[3, 130] = float("inf")                           # non-finite values do not enter the amax
    x[4, 300:428] = -0.0
    x[5, 0] = 1e-30                                    # tiny values beside a large one
    x[5, 1] = 3.0e4
    for dname, dt in (("bfloat16", torch.bfloat16), ("float16", torch.float16)):
        xd = x.to(dt)
        for fmt, fmax in (("e4m3", 448.0), ("e5m2", 57344.0)):
            ax = xd.float().abs()
            a = torch.where(torch.isfinite(ax), ax, torch.zeros_like(ax)).reshape(t, kvd // 128, 128).amax(-1)
            scale = (a / torch.tensor(fmax, dtype=torch.float32)).to(torch.float32)
            per = scale.repeat_interleave(128, dim=1)
            codes = rk._fp8_quantize_to_uint8(xd, per, fmt)
            dec = rk._fp8_dequantize_from_uint8(codes, per, fmt, dt)
            p = f"{dname}/{fmt}"
            st.put(f"{p}/x", xd)
            st.put(f"{p}/scale", scale)
            st.put(f"{p}/codes", codes)
            st.put(f"{p}/dec", dec)
    st.save("mla_fp8.npz")


def make_cache() -> None:
    st = Store()
    g = gen(50)
    names = list(DTYPES)
    for xn in names:
        for cn in names:
            for inter in (False, True):
                x = (randn((3, 5, 4, 16), torch.float32, g) * 3.0).to(DTYPES[xn])
                ang = torch.rand((5, 1, 8), generator=g) * 6.0
                cos, sin = torch.cos(ang).to(DTYPES[cn]), torch.sin(ang).to(DTYPES[cn])
                out = ref.apply_rope(x, cos, sin, interleaved=inter)
                p = f"rope/{xn}/{cn}/{int(inter)}"
                st.put(f"{p}/x", x)
                st.put(f"{p}/cos", cos)
                st.put(f"{p}/sin", sin)
                st.put(f"{p}/out", out)
    # mixed cos / sin dtypes and a broadcast that grows the output
    x = (randn((4, 2, 8), torch.float32, g) * 2.0).to(torch.bfloat16)
    cos = torch.cos(torch.rand((3, 1, 1, 4), generator=g) * 6.0).to(torch.float16)
    sin = torch.sin(torch.rand((1, 4), generator=g) * 6.0).to(torch.float32)
    st.put("rope_mixed/x", x)
    st.put("rope_mixed/cos", cos)
    st.put("rope_mixed/sin", sin)
    st.put("rope_mixed/out", ref.apply_rope(x, cos, sin))
    for cn in names:
        dt = DTYPES[cn]
        kc = (randn((4, 2, 8, 4), torch.float32, g) * 2.0).to(dt)
        slots = torch.tensor([0, 6, -1, 13, 6, 15, 2], dtype=torch.int64)
        positions = torch.tensor([0, 3, 1, 7, 2, 5, 9], dtype=torch.int64)
        ang = torch.rand((10, 4), generator=g) * 6.0
        cos2, sin2 = torch.cos(ang).to(dt), torch.sin(ang).to(dt)
        p = f"rope_cache/{cn}"
        st.put(f"{p}/cache_in", kc)
        st.put(f"{p}/slots", slots)
        st.put(f"{p}/positions", positions)
        st.put(f"{p}/cos", cos2)
        st.put(f"{p}/sin", sin2)
        out2 = ref.apply_rope_to_key_cache(kc.clone(), slots, positions, cos2, sin2)
        st.put(f"{p}/cache_out", out2)
        out1 = ref.apply_rope_to_key_cache(kc.clone(), slots, positions, cos2[4], sin2[4], interleaved=True)
        st.put(f"{p}/cache_out_1d_inter", out1)
        k = randn((6, 2, 8), torch.float32, g).to(dt)
        v = randn((6, 2, 8), torch.float32, g).to(dt)
        kcc, vcc = torch.zeros((4, 2, 8, 4), dtype=dt), torch.zeros((4, 2, 8, 4), dtype=dt)
        cslots = torch.tensor([0, 5, -1, 5, 15, 9], dtype=torch.int64)
        ref.copy_to_kv_cache(k, v, kcc, vcc, cslots)
        st.put(f"copy/{cn}/k", k)
        st.put(f"copy/{cn}/v", v)
        st.put(f"copy/{cn}/slots", cslots)
        st.put(f"copy/{cn}/kc", kcc)
        st.put(f"copy/{cn}/vc", vcc)
    st.save("cache.npz")


def make_merged_fp8() -> None:
    """FP8 merged wrappers (reference ops/kv_transfer.py:3460-3553): a merged ``[T, 2, NH, HD]`` /
    ``[L, T, 2, NH, HD]`` buffer quantised into two uint8 tile caches and dequantised back, for
    both formats, scalar / ``[NH]`` / ``[L, NH]`` scales, negative and duplicate slots."""
    st = Store()
    nb, nh, hd = 6, 2, 16
    sl = torch.tensor([5, 6, 7, -1, 5, 40, 63, 0, 1, 2, 3, 4, 8, 9, 10, 11, 12, 13, 14, 15, 95, 16, 17, -7, 63],
                      dtype=torch.int64)
    gsl = torch.tensor([63, 5, -1, 6, 7, 40, 0, 1, 2, 3, 4, 8, 9, 10, 11, 12, 13, 14, 15, 95, 94, -3, 16], dtype=torch.int64)
    nl = 3
    for bs in (16, 4):
        t = int(sl.numel())
        ss = torch.where(sl < 0, sl, sl % (nb * bs))  # duplicates survive the fold (5, 63 twice)
        gs = torch.where(gsl < 0, gsl, gsl % (nb * bs))
        st.put(f"bs{bs}/slots", ss)
        st.put(f"bs{bs}/gslots", gs)
        for fmt in ("e4m3", "e5m2"):
            for lname, ldt in (("bfloat16", torch.bfloat16), ("float16", torch.float16)):
                g = gen(60 + bs)
                merged = (randn((t, 2, nh, hd), torch.float32, g) * 2.0).to(ldt)
                merged_ml = (randn((nl, t, 2, nh, hd), torch.float32, g) * 2.0).to(ldt)
                scale_forms = {
                    "scalar": (0.0123, 0.0177),
                    "head": (torch.rand((nh,), generator=g) * 0.02 + 0.001, torch.rand((nh,), generator=g) * 0.02 + 0.001),
                }
                for sname, (ks, vs) in scale_forms.items():
                    p = f"bs{bs}/{fmt}/{lname}/{sname}"
                    kc = torch.zeros((nb, nh, hd, bs), dtype=torch.uint8)
                    vc = torch.zeros((nb, nh, hd, bs), dtype=torch.uint8)
                    ref.kv_merged_linear_to_paged_fp8(merged, kc, vc, ss, ks, vs, fp8_format=fmt)
                    st.put(f"{p}/merged", merged)
                    st.put(f"{p}/k_scale", torch.as_tensor(ks, dtype=torch.float32))
                    st.put(f"{p}/v_scale", torch.as_tensor(vs, dtype=torch.float32))
                    st.put(f"{p}/k_cache", kc)
                    st.put(f"{p}/v_cache", vc)
                    out = ref.kv_paged_fp8_to_merged_linear(kc, vc, gs, ks, vs, out_dtype=ldt, fp8_format=fmt)
                    st.put(f"{p}/gather", out)
                ml_forms = dict(scale_forms)
                ml_forms["layer_head"] = (torch.rand((nl, nh), generator=g) * 0.02 + 0.001, 0.0149)
                for sname, (ks, vs) in ml_forms.items():
                    p = f"bs{bs}/{fmt}/{lname}/ml_{sname}"
                    kc = torch.zeros((nl, nb, nh, hd, bs), dtype=torch.uint8)
                    vc = torch.zeros((nl, nb, nh, hd, bs), dtype=torch.uint8)
                    ref.kv_merged_linear_to_paged_fp8_multi_layer(merged_ml, kc, vc, ss, ks, vs, fp8_format=fmt)
                    st.put(f"{p}/merged", merged_ml)
                    st.put(f"{p}/k_scale", torch.as_tensor(ks, dtype=torch.float32))
                    st.put(f"{p}/v_scale", torch.as_tensor(vs, dtype=torch.float32))
                    st.put(f"{p}/k_cache", kc)
                    st.put(f"{p}/v_cache", vc)
                    out = ref.kv_paged_fp8_to_merged_linear_multi_layer(kc, vc, gs, ks, vs, out_dtype=ldt, fp8_format=fmt)
                    st.put(f"{p}/gather", out)
    st.save("merged_fp8.npz")


def make_pools() -> None:
    """DSV4 multi-pool page-row copy (reference ops/kv_transfer.py:4619-4660): pools of different
    row widths and layer counts sharing one index vector, run on CPU tensors in both directions
    (the reference's copy is the same index_select / index_copy_ whatever the devices)."""
    from musa_aiter.ops.kv_transfer import PoolSpec as RefPoolSpec

    st = Store()
    g = gen(70)
    pages = 24
    idx = torch.tensor([3, 17, 0, 23, 8, 17, 22, 5], dtype=torch.int64)
    st.put("indices", idx)
    specs = [(2, 656), (1, 24), (3, 129), (1, 1)]  # (layers, item_bytes)
    for direction in ("H2D", "D2H"):
        pools = []
        for p, (nl, item) in enumerate(specs):
            srcs = [torch.randint(0, 256, (pages, item), generator=g, dtype=torch.int32).to(torch.uint8) for _ in range(nl)]
            dsts = [torch.randint(0, 256, (pages, item), generator=g, dtype=torch.int32).to(torch.uint8) for _ in range(nl)]
            st.put(f"{direction}/{p}/src", torch.stack(srcs))
            st.put(f"{direction}/{p}/dst_in", torch.stack(dsts))
            pools.append((srcs, dsts, item))
        ref.ops.kv_transfer.kv_copy_paged_rows_multi_pool(
            [RefPoolSpec(src_ptrs=s, dst_ptrs=d, item_bytes=i) for s, d, i in pools], idx, direction=direction)
        for p, (_, dsts, _) in enumerate(pools):
            st.put(f"{direction}/{p}/dst_out", torch.stack(dsts))
    st.save("pools.npz")


if __name__ == "__main__":
    torch.manual_seed(0)
    families = {"tile": make_tile, "fp8": make_fp8, "rows": make_rows, "misc": make_misc, "mla_fp8": make_mla_fp8,
                "cache": make_cache, "merged_fp8": make_merged_fp8, "pools": make_pools}
    for name in (sys.argv[1:] or list(families)):
        families[name]()
