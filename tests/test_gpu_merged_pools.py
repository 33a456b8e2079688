"""GPU parity for the FP8 merged entry points (reference ops/kv_transfer.py:3460-3553) and the
DSV4 multi-pool page-row copy (ops/kv_transfer.py:4619-4660): the public API (C ABI underneath)
against the reference's golden vectors and, on larger seeded inputs, the CPU oracle.  Every
comparison is bit for bit."""

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


@pytest.fixture(scope="module")
def merged_fp8():
    return np.load(GOLDEN / "merged_fp8.npz")


@pytest.fixture(scope="module")
def pools():
    return np.load(GOLDEN / "pools.npz")


def eq(a, b, what=""):
    assert same_bits(a, b), f"{what}: {first_diff(a, b)}"


def _scale(a: np.ndarray):
    """Golden scales as the caller would pass them: a Python float for scalars, a device tensor otherwise."""
    return float(a) if a.ndim == 0 else torch.from_numpy(a).cuda()


# ---------------------------------------------------------------------------
# a11: FP8 merged wrappers
# ---------------------------------------------------------------------------


def _cases(g):
    return sorted({tuple(k.split("/")[:4]) for k in g.files if k.count("/") == 4})


@pytest.mark.parametrize("fmt", ("e4m3", "e5m2"))
def test_golden_merged_fp8(cuda_device, merged_fp8, fmt):
    g = merged_fp8
    cases = [c for c in _cases(g) if c[1] == fmt]
    assert len(cases) == 20
    for bs, _, dt, form in cases:
        p = f"{bs}/{fmt}/{dt}/{form}"
        slots = torch.from_numpy(g[f"{bs}/slots"]).cuda()
        gslots = torch.from_numpy(g[f"{bs}/gslots"]).cuda()
        merged = to_torch(g[f"{p}/merged"], dt)
        kc = torch.zeros(g[f"{p}/k_cache"].shape, dtype=torch.uint8, device="cuda")
        vc = torch.zeros_like(kc)
        ks, vs = _scale(g[f"{p}/k_scale"]), _scale(g[f"{p}/v_scale"])
        if form.startswith("ml_"):
            assert ma.kv_merged_linear_to_paged_fp8_multi_layer(merged, kc, vc, slots, ks, vs, fp8_format=fmt) is None
            out = ma.kv_paged_fp8_to_merged_linear_multi_layer(kc, vc, gslots, ks, vs, out_dtype=TORCH_OF[dt], fp8_format=fmt)
        else:
            assert ma.kv_merged_linear_to_paged_fp8(merged, kc, vc, slots, ks, vs, fp8_format=fmt) is None
            out = ma.kv_paged_fp8_to_merged_linear(kc, vc, gslots, ks, vs, out_dtype=TORCH_OF[dt], fp8_format=fmt)
        eq(kc, g[f"{p}/k_cache"], f"{p} store k")
        eq(vc, g[f"{p}/v_cache"], f"{p} store v")
        eq(out, g[f"{p}/gather"], f"{p} gather")


def _block_runs(lens, nb, bs, gen):
    perm = torch.randperm(nb, generator=gen)
    out, used = [], 0
    for n in lens:
        k = (n + bs - 1) // bs
        bt = perm[used:used + k]
        used += k
        pos = torch.arange(n)
        out.append(bt[pos // bs] * bs + pos % bs)
    return torch.cat(out)


@pytest.mark.parametrize("fmt,scale_kind", (("e4m3", "layer_head"), ("e5m2", "scalar"), ("e4m3", "head")))
def test_merged_fp8_multi_layer_block_tables_vs_oracle(cuda_device, fmt, scale_kind):
    """Merged [L, T, 2, NH, HD] buffers at the Llama-3-8B head geometry with block-table slots
    (full 16-token runs, ragged sequence ends), negatives, duplicates and a repeated run; some
    chunks hold inf / nan / out-of-range values so both FP8 encoders of the run path are used;
    the gather writes into a caller-provided merged ``out`` (its 2*NH*HD token stride)."""
    g = torch.Generator().manual_seed(31)
    nl, nb, nh, hd, bs = 3, 384, 8, 128, 16
    slots = _block_runs([37, 160, 301, 16, 1, 700], nb, bs, g)
    slots = torch.cat([slots, torch.tensor([-1, -5]), slots[40:90], torch.randint(0, nb * bs, (64,), generator=g)])
    t = slots.numel()
    merged = (torch.randn((nl, t, 2, nh, hd), generator=g) * 2.0).to(torch.bfloat16)
    merged[1, 100, 0, 3, 7] = float("inf")
    merged[2, 333, 1, 0, 0] = float("nan")
    merged[0, 500:516, 1] *= 4000.0  # past the bounded encoder's range for e4m3 scales below
    if scale_kind == "layer_head":
        ks = merged[:, :, 0].float().abs().nan_to_num(0, 0, 0).amax(dim=(1, 3)) / 448.0
        vs = merged[:, :, 1].float().abs().nan_to_num(0, 0, 0).amax(dim=(1, 3)) / 448.0 / 64.0
        ks[0] = 0.003  # clamps: values reach past 448 * scale
    elif scale_kind == "head":
        ks = torch.rand(nh, generator=g) * 0.01 + 0.004
        vs = torch.rand(nh, generator=g) * 0.01 + 0.004
    else:
        ks = torch.tensor(merged.float().abs().nan_to_num(0, 0, 0).amax().item() / 57344.0)
        vs = torch.tensor(0.0007)
    kc = torch.zeros((nl, nb, nh, hd, bs), dtype=torch.uint8, device="cuda")
    vc = torch.zeros_like(kc)
    ma.kv_merged_linear_to_paged_fp8_multi_layer(merged.cuda(), kc, vc, slots.cuda(), ks.cuda(), vs.cuda(), fp8_format=fmt)
    rk, rv = np.zeros(kc.shape, np.uint8), np.zeros(vc.shape, np.uint8)
    O.kv_merged_linear_to_paged_fp8_multi_layer(to_np(merged), rk, rv, slots.numpy(), ks.numpy(), vs.numpy(), fp8_format=fmt)
    eq(kc, rk, "merged fp8 store k")
    eq(vc, rv, "merged fp8 store v")
    gsl = torch.cat([slots[:900], torch.tensor([-1, 3, 4, 5, -2])])
    out = torch.full((nl, gsl.numel(), 2, nh, hd), 7.0, dtype=torch.float16, device="cuda")
    got = ma.kv_paged_fp8_to_merged_linear_multi_layer(kc, vc, gsl.cuda(), ks.cuda(), vs.cuda(), out_dtype=torch.float16,
                                                       fp8_format=fmt, out=out)
    assert got.data_ptr() == out.data_ptr()
    want = O.kv_paged_fp8_to_merged_linear_multi_layer(rk, rv, gsl.numpy(), ks.numpy(), vs.numpy(), out_dtype="float16",
                                                       fp8_format=fmt)
    eq(out, want, "merged fp8 gather")


def test_merged_fp8_single_layer_random_slots_fp8_storage(cuda_device):
    """Single-layer merged store into torch.float8_e4m3fn storage (raw bytes either way) with
    random unique slots, then the merged gather; the bytes equal the oracle's."""
    g = torch.Generator().manual_seed(32)
    nb, nh, hd, bs, t = 256, 8, 128, 16, 1500
    slots = torch.randperm(nb * bs, generator=g)[:t]
    slots[::97] = -1
    merged = (torch.randn((t, 2, nh, hd), generator=g) * 2.0).to(torch.float16)
    ks = torch.rand(nh, generator=g) * 0.01 + 0.002
    kc = torch.zeros((nb, nh, hd, bs), dtype=torch.float8_e4m3fn, device="cuda")
    vc = torch.zeros_like(kc)
    ma.kv_merged_linear_to_paged_fp8(merged.cuda(), kc, vc, slots.cuda(), ks.cuda(), 0.0123)
    rk, rv = np.zeros(kc.shape, np.uint8), np.zeros(vc.shape, np.uint8)
    O.kv_merged_linear_to_paged_fp8(merged.numpy(), rk, rv, slots.numpy(), ks.numpy(), np.float32(0.0123), lin_dtype="float16")
    eq(kc.view(torch.uint8), rk, "merged fp8 (float8 storage) k")
    eq(vc.view(torch.uint8), rv, "merged fp8 (float8 storage) v")
    out = ma.kv_paged_fp8_to_merged_linear(kc, vc, slots.cuda(), ks.cuda(), 0.0123, out_dtype=torch.bfloat16)
    want = O.kv_paged_fp8_to_merged_linear(rk, rv, slots.numpy(), ks.numpy(), np.float32(0.0123), out_dtype="bfloat16")
    eq(out, want, "merged fp8 gather (float8 storage)")


# ---------------------------------------------------------------------------
# f2: DSV4 multi-pool page rows, host <-> device
# ---------------------------------------------------------------------------


def _host(a: np.ndarray, pinned: bool) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a).copy())
    return t.pin_memory() if pinned else t


@pytest.mark.parametrize("index_device", ("cpu", "cuda"))
def test_golden_multi_pool(cuda_device, pools, index_device):
    """Golden replay in both directions; pools 0 and 2 use pinned host tensors (addressed by the
    kernel in place), pools 1 and 3 pageable ones (staged through a pinned bounce buffer)."""
    idx = torch.from_numpy(pools["indices"]).to(index_device)
    for direction in ("H2D", "D2H"):
        n = len({k.split("/")[1] for k in pools.files if k.startswith(direction)})
        specs, outs = [], []
        for p in range(n):
            src, dst_in = pools[f"{direction}/{p}/src"], pools[f"{direction}/{p}/dst_in"]
            pinned = p % 2 == 0
            if direction == "H2D":
                srcs = [_host(s, pinned) for s in src]
                dsts = [torch.from_numpy(d.copy()).cuda() for d in dst_in]
            else:
                srcs = [torch.from_numpy(s.copy()).cuda() for s in src]
                dsts = [_host(d, pinned) for d in dst_in]
            specs.append(ma.PoolSpec(src_ptrs=srcs, dst_ptrs=dsts, item_bytes=int(src.shape[-1])))
            outs.append(dsts)
        assert ma.kv_copy_paged_rows_multi_pool(specs, idx, direction=direction) is None
        torch.cuda.synchronize()
        for p, dsts in enumerate(outs):
            eq(torch.stack([d.cpu() for d in dsts]), pools[f"{direction}/{p}/dst_out"], f"{direction} pool {p}")


@pytest.mark.parametrize("direction", ("H2D", "D2H"))
@pytest.mark.parametrize("pinned", (True, False))
def test_multi_pool_large_vs_oracle(cuda_device, direction, pinned):
    """DSV4-sized rows (656 B FP8 MLA rows, 1728 B, 8 B state) over 4096 pages, 1500 shared
    indices with repeats; back-to-back calls whose pageable bounce buffers are released while
    their copies are still queued; the bytes equal the oracle's."""
    g = torch.Generator().manual_seed(33)
    pages = 4096
    layout = [(3, 656), (2, 1728), (1, 8)]
    idx = torch.randint(0, pages, (1500,), generator=g)
    srcs_np = [[torch.randint(0, 256, (pages, w), generator=g, dtype=torch.uint8).numpy() for _ in range(nl)] for nl, w in layout]
    dsts_np = [[torch.randint(0, 256, (pages, w), generator=g, dtype=torch.uint8).numpy() for _ in range(nl)] for nl, w in layout]
    want = [[d.copy() for d in ds] for ds in dsts_np]
    O.kv_copy_paged_rows_multi_pool(list(zip(srcs_np, want)), idx.numpy())
    if direction == "H2D":
        srcs = [[_host(s, pinned) for s in ss] for ss in srcs_np]
        dsts = [[torch.from_numpy(d.copy()).cuda() for d in ds] for ds in dsts_np]
    else:
        srcs = [[torch.from_numpy(s.copy()).cuda() for s in ss] for ss in srcs_np]
        dsts = [[_host(d, pinned) for d in ds] for ds in dsts_np]
    specs = [ma.PoolSpec(src_ptrs=s, dst_ptrs=d, item_bytes=w) for s, d, (_, w) in zip(srcs, dsts, layout)]
    for _ in range(3):  # idempotent: the same rows land again
        ma.kv_copy_paged_rows_multi_pool(specs, idx.cuda(), direction=direction)
        # churn the pinned-memory cache so a released-too-early bounce block would be rewritten
        junk = [torch.full((1500, 1728), 0xA5, dtype=torch.uint8).pin_memory() for _ in range(4)]
        del junk
    torch.cuda.synchronize()
    for p, ds in enumerate(dsts):
        for l, d in enumerate(ds):
            eq(d.cpu(), want[p][l], f"{direction} pinned={pinned} pool {p} layer {l}")
