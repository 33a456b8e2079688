"""GPU parity for the `cache` family (apply_rope, apply_rope_to_key_cache, copy_to_kv_cache):
the reference's own outputs (golden vectors, every dtype pairing) and the CPU oracle on larger
seeded inputs.  Bit-exact: the kernels round after every operation as PyTorch does."""

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
DT = ("float32", "float16", "bfloat16")


def eq(got, want, what):
    assert same_bits(got, want), f"{what}: {first_diff(got, want)}"


@pytest.fixture(scope="module")
def g():
    return np.load(GOLDEN / "cache.npz")


@pytest.mark.parametrize("inter", (0, 1))
@pytest.mark.parametrize("cn", DT)
@pytest.mark.parametrize("xn", DT)
def test_golden_apply_rope(cuda_device, g, xn, cn, inter):
    p = f"rope/{xn}/{cn}/{inter}"
    out = ma.apply_rope(to_torch(g[f"{p}/x"], xn), to_torch(g[f"{p}/cos"], cn), to_torch(g[f"{p}/sin"], cn),
                        interleaved=bool(inter))
    eq(out, g[f"{p}/out"], p)


def test_golden_apply_rope_mixed(cuda_device, g):
    out = ma.apply_rope(to_torch(g["rope_mixed/x"], "bfloat16"), to_torch(g["rope_mixed/cos"], "float16"),
                        to_torch(g["rope_mixed/sin"], "float32"))
    eq(out, g["rope_mixed/out"], "mixed dtypes, growing broadcast")


@pytest.mark.parametrize("cn", DT)
def test_golden_key_cache_and_copy(cuda_device, g, cn):
    p = f"rope_cache/{cn}"
    kc = to_torch(g[f"{p}/cache_in"], cn)
    slots, pos = to_torch(g[f"{p}/slots"]), to_torch(g[f"{p}/positions"])
    out = ma.apply_rope_to_key_cache(kc, slots, pos, to_torch(g[f"{p}/cos"], cn), to_torch(g[f"{p}/sin"], cn))
    assert out.data_ptr() == kc.data_ptr()
    eq(kc, g[f"{p}/cache_out"], "rope key cache (repeated slot 6 rotated twice in token order)")
    kc = to_torch(g[f"{p}/cache_in"], cn)
    ma.apply_rope_to_key_cache(kc, slots, pos, to_torch(g[f"{p}/cos"][4], cn), to_torch(g[f"{p}/sin"][4], cn),
                               interleaved=True)
    eq(kc, g[f"{p}/cache_out_1d_inter"], "1-D table, interleaved")
    q = f"copy/{cn}"
    kcc = torch.zeros(g[f"{q}/kc"].shape, dtype=TORCH_OF[cn], device="cuda")
    vcc = torch.zeros_like(kcc)
    assert ma.copy_to_kv_cache(to_torch(g[f"{q}/k"], cn), to_torch(g[f"{q}/v"], cn), kcc, vcc,
                               to_torch(g[f"{q}/slots"])) is None
    eq(kcc, g[f"{q}/kc"], "copy k")
    eq(vcc, g[f"{q}/vc"], "copy v")


def test_random_rope_vs_oracle(cuda_device):
    gen = torch.Generator().manual_seed(3)
    x = (torch.randn((2, 33, 8, 128), generator=gen) * 4).to(torch.bfloat16)
    ang = torch.rand((33, 1, 64), generator=gen) * 100
    cos, sin = torch.cos(ang), torch.sin(ang)  # fp32 tables with a bf16 x: products in fp32
    for inter in (False, True):
        out = ma.apply_rope(x.cuda(), cos.cuda(), sin.cuda(), interleaved=inter)
        want = O.apply_rope(to_np(x), cos.numpy(), sin.numpy(), x_dtype="bfloat16", cos_dtype="float32",
                            sin_dtype="float32", interleaved=inter)
        eq(out, want, f"interleaved={inter}")
    # strided (non-contiguous) x
    xt = x.transpose(1, 2)
    out = ma.apply_rope(xt.cuda(), cos.transpose(0, 1).cuda(), sin.transpose(0, 1).cuda())
    want = O.apply_rope(to_np(xt), cos.transpose(0, 1).numpy(), sin.transpose(0, 1).numpy(), x_dtype="bfloat16",
                        cos_dtype="float32", sin_dtype="float32")
    eq(out, want, "strided x")


def test_random_key_cache_vs_oracle(cuda_device):
    gen = torch.Generator().manual_seed(4)
    nb, nh, hd, bs = 64, 8, 128, 16
    kc = (torch.randn((nb, nh, hd, bs), generator=gen) * 2).to(torch.float16)
    slots = torch.randint(-1, nb * bs, (300,), generator=gen)
    slots[10] = slots[200]
    pos = torch.randint(0, 4096, (300,), generator=gen)
    ang = torch.rand((4096, hd // 2), generator=gen) * 50
    cos, sin = torch.cos(ang).half(), torch.sin(ang).half()
    dk = kc.cuda()
    ma.apply_rope_to_key_cache(dk, slots.cuda(), pos.cuda(), cos.cuda(), sin.cuda())
    want = to_np(kc).copy()
    O.apply_rope_to_key_cache(want, slots.numpy(), pos.numpy(), cos.numpy(), sin.numpy(), cache_dtype="float16",
                              cos_dtype="float16", sin_dtype="float16")
    eq(dk, want, "key cache rope")


def _block_table_slots(gen, nb, bs, whole, ragged):
    """`whole` block-table blocks of `bs` tokens, a ragged run of `ragged` tokens, single tokens
    and negative slots between them (all slots distinct)."""
    blocks = torch.randperm(nb, generator=gen)[: whole + 2]
    runs = (blocks[:whole, None] * bs + torch.arange(bs)).flatten()
    tail = blocks[whole] * bs + torch.arange(ragged)
    singles = blocks[whole + 1] * bs + torch.tensor([0, 5, 3])
    return torch.cat([runs[: len(runs) // 2], torch.tensor([-1]), tail, singles, torch.tensor([-1, -7]),
                      runs[len(runs) // 2:]])


@pytest.mark.parametrize("whole", (40, 70))
@pytest.mark.parametrize("skip_validation", (False, True))
@pytest.mark.parametrize("inter", (False, True))
@pytest.mark.parametrize("hd", (128, 20))
@pytest.mark.parametrize("cn", DT)
def test_key_cache_block_tables_fp32_tables_vs_oracle(cuda_device, monkeypatch, cn, hd, inter, skip_validation,
                                                      whole):
    """fp32 cos / sin tables (every product in fp32) on block-table slots: lanes walk the tokens
    of a block together; head_dim 20 leaves a partial group of rotation pairs; 40 and 70 whole
    blocks give calls below and above 1024 tokens."""
    if skip_validation:
        monkeypatch.setenv("MUSA_AITER_SKIP_VALIDATION", "1")
    gen = torch.Generator().manual_seed(11 + hd + whole)
    nb, nh, bs = 96, 8, 16
    kc = (torch.randn((nb, nh, hd, bs), generator=gen) * 3).to(TORCH_OF[cn])
    slots = _block_table_slots(gen, nb, bs, whole, 7)
    pos = torch.randint(0, 2048, (slots.numel(),), generator=gen)
    ang = torch.rand((2048, hd // 2), generator=gen) * 80
    cos, sin = torch.cos(ang), torch.sin(ang)
    dk = kc.cuda()
    ma.apply_rope_to_key_cache(dk, slots.cuda(), pos.cuda(), cos.cuda(), sin.cuda(), interleaved=inter)
    want = to_np(kc).copy()
    O.apply_rope_to_key_cache(want, slots.numpy(), pos.numpy(), cos.numpy(), sin.numpy(), cache_dtype=cn,
                              cos_dtype="float32", sin_dtype="float32", interleaved=inter)
    eq(dk, want, f"{cn} cache, head_dim {hd}, interleaved={inter}")


@pytest.mark.parametrize("table", ("contiguous", "column view"))
@pytest.mark.parametrize("whole", (300, 1200))
def test_key_cache_large_block_tables_vs_oracle(cuda_device, whole, table):
    """Enough tokens for warp items of several heads (300 blocks) and of every head (1200), in a
    head-strided view of a wider cache, int32 slots and positions; fp32 tables read 16 bytes at a
    time when contiguous, element by element as a column view of a wider table."""
    gen = torch.Generator().manual_seed(whole)
    nb, nh, hd, bs = 1300, 8, 128, 16
    wide = (torch.randn((nb, nh + 2, hd, bs), generator=gen) * 3).to(torch.bfloat16)
    slots = _block_table_slots(gen, nb, bs, whole, 11).to(torch.int32)
    pos = torch.randint(0, 8192, (slots.numel(),), generator=gen).to(torch.int32)
    ang = torch.rand((8192, hd // 2), generator=gen) * 80
    cos, sin = torch.cos(ang), torch.sin(ang)
    if table == "contiguous":
        dcos, dsin = cos.cuda(), sin.cuda()
    else:
        dcos = torch.zeros((8192, hd // 2 + 3), device="cuda")[:, 1:hd // 2 + 1]
        dsin = torch.zeros((8192, hd // 2 + 3), device="cuda")[:, 2:hd // 2 + 2]
        dcos.copy_(cos)
        dsin.copy_(sin)
    dw = wide.cuda()
    ma.apply_rope_to_key_cache(dw[:, 1:nh + 1], slots.cuda(), pos.cuda(), dcos, dsin)
    want = to_np(wide).copy()
    view = want[:, 1:nh + 1]
    O.apply_rope_to_key_cache(view, slots.numpy(), pos.numpy(), cos.numpy(), sin.numpy(), cache_dtype="bfloat16",
                              cos_dtype="float32", sin_dtype="float32")
    eq(dw, want, f"{whole} whole blocks, heads 1..{nh} of {nh + 2}")


@pytest.mark.parametrize("whole", (6, 80))
def test_key_cache_negative_positions_skipped_without_validation(cuda_device, monkeypatch, whole):
    """With validation off nothing is read back, and a token whose position is negative (which
    the host check rejects) is skipped by the kernel instead of reading before the table (calls
    of 6 and 80 whole blocks)."""
    monkeypatch.setenv("MUSA_AITER_SKIP_VALIDATION", "1")
    gen = torch.Generator().manual_seed(21 + whole)
    nb, nh, hd, bs = 96, 4, 64, 16
    kc = (torch.randn((nb, nh, hd, bs), generator=gen) * 3).to(torch.bfloat16)
    slots = _block_table_slots(gen, nb, bs, whole, 5)
    pos = torch.randint(0, 512, (slots.numel(),), generator=gen)
    pos[::7] = -3
    ang = torch.rand((512, hd // 2), generator=gen) * 80
    cos, sin = torch.cos(ang), torch.sin(ang)
    dk = kc.cuda()
    ma.apply_rope_to_key_cache(dk, slots.cuda(), pos.cuda(), cos.cuda(), sin.cuda())
    keep = pos >= 0
    want = to_np(kc).copy()
    O.apply_rope_to_key_cache(want, slots[keep].numpy(), pos[keep].numpy(), cos.numpy(), sin.numpy(),
                              cache_dtype="bfloat16", cos_dtype="float32", sin_dtype="float32")
    eq(dk, want, "negative positions skipped")


def test_reference_errors(cuda_device):
    kc = torch.zeros(1, 1, 4, 2, device="cuda")
    with pytest.raises(ValueError, match="position exceeds cos/sin table"):
        ma.apply_rope_to_key_cache(kc, torch.tensor([0], device="cuda"), torch.tensor([2], device="cuda"),
                                   torch.ones(2, 2, device="cuda"), torch.zeros(2, 2, device="cuda"))
    with pytest.raises(ValueError, match="invalid block_id=1"):
        ma.apply_rope_to_key_cache(kc, torch.tensor([3], device="cuda"), torch.tensor([0], device="cuda"),
                                   torch.ones(2, 2, device="cuda"), torch.zeros(2, 2, device="cuda"))
    with pytest.raises(ValueError, match="head_dim must be even"):
        ma.apply_rope(torch.zeros(3, 5, device="cuda"), torch.ones(2, device="cuda"), torch.zeros(2, device="cuda"))
    k = torch.zeros(2, 1, 4, device="cuda")
    with pytest.raises(ValueError, match="invalid block_id"):
        ma.copy_to_kv_cache(k, k, torch.zeros(1, 1, 4, 2, device="cuda"), torch.zeros(1, 1, 4, 2, device="cuda"),
                            torch.tensor([0, 2], device="cuda"))
