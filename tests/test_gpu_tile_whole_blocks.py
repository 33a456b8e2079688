"""Tile-engine calls that mix whole cache blocks (block tables), partial last blocks, runs that
straddle a block boundary, lone slots, negatives and whole blocks written twice, over head
dims 16 to 256 and the merged K/V stride: gathers and scatters must equal the CPU oracle bit
for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import musa_aiter as ma
from oracle import kv_oracle as O

from ._util import first_diff, same_bits, to_np

pytestmark = pytest.mark.gpu


def eq(a, b, what=""):
    assert same_bits(a, b), f"{what}: {first_diff(a, b)}"


def _mixed_slots(nb, gen):
    """Whole blocks (block tables), a partial last block per sequence, a whole block shifted by
    one slot (never whole), lone slots, negatives, and whole blocks written twice (the later
    copy wins)."""
    perm = torch.randperm(nb, generator=gen)
    parts, used = [], 0
    for n in (16, 37, 160, 5, 301, 64):
        k = (n + 15) // 16
        bt = perm[used:used + k]
        used += k
        pos = torch.arange(n)
        parts.append(bt[pos // 16] * 16 + pos % 16)
    b = int(perm[used])
    parts.append(torch.arange(b * 16 + 1, b * 16 + 17))  # crosses into the next block: no whole block
    parts.append(torch.tensor([-1, int(perm[used + 2]) * 16 + 3, -5]))
    parts.append(parts[2][:32])  # a repeated pair of whole blocks
    return torch.cat(parts).to(torch.int64)


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float16))
@pytest.mark.parametrize("nh,hd", ((8, 128), (2, 64), (1, 256), (4, 16), (3, 48)))
def test_whole_blocks_gather_scatter_vs_oracle(cuda_device, dtype, nh, hd):
    g = torch.Generator().manual_seed(41 + hd)
    nl, nb = 3, 160
    slots = _mixed_slots(nb, g)
    t = slots.numel()
    kc = torch.randn((nl, nb, nh, hd, 16), generator=g).to(dtype)
    vc = torch.randn((nl, nb, nh, hd, 16), generator=g).to(dtype)
    ok, ov = ma.kv_paged_to_linear_multi_layer(kc.cuda(), vc.cuda(), slots.cuda())
    rk, rv = O.kv_paged_to_linear_multi_layer(to_np(kc), to_np(vc), slots.numpy())
    eq(ok, rk, "whole-block gather k")
    eq(ov, rv, "whole-block gather v")
    kl = torch.randn((nl, t, nh, hd), generator=g).to(dtype)
    vl = torch.randn((nl, t, nh, hd), generator=g).to(dtype)
    dk = torch.full((nl, nb, nh, hd, 16), 3.0, dtype=dtype, device="cuda")
    dv = torch.full_like(dk, -1.0)
    ma.kv_linear_to_paged_multi_layer(kl.cuda(), vl.cuda(), dk, dv, slots.cuda())
    wk, wv = to_np(torch.full((nl, nb, nh, hd, 16), 3.0, dtype=dtype)), to_np(torch.full((nl, nb, nh, hd, 16), -1.0, dtype=dtype))
    O.kv_linear_to_paged_multi_layer(to_np(kl), to_np(vl), wk, wv, slots.numpy())
    eq(dk, wk, "whole-block scatter k")
    eq(dv, wv, "whole-block scatter v")


def test_whole_blocks_merged_and_large_call_vs_oracle(cuda_device):
    """Merged [L, T, 2, NH, HD] buffers (2 * NH * HD token stride) and a call large enough for
    plane groups of 8 and many windows per warp; gathers then scatters back into fresh caches."""
    g = torch.Generator().manual_seed(43)
    nl, nb, nh, hd = 8, 2048, 8, 128
    lens = torch.randint(1, 700, (48,), generator=g).tolist()
    perm = torch.randperm(nb, generator=g)
    parts, used = [], 0
    for n in lens:
        k = (n + 15) // 16
        bt = perm[used:used + k]
        used += k
        pos = torch.arange(n)
        parts.append(bt[pos // 16] * 16 + pos % 16)
    slots = torch.cat(parts).to(torch.int64)
    kc = torch.randn((nl, nb, nh, hd, 16), generator=g).to(torch.bfloat16)
    vc = torch.randn((nl, nb, nh, hd, 16), generator=g).to(torch.bfloat16)
    merged = ma.kv_paged_to_merged_linear_multi_layer(kc.cuda(), vc.cuda(), slots.cuda())
    want = O.kv_paged_to_linear_multi_layer(to_np(kc), to_np(vc), slots.numpy())
    eq(merged[:, :, 0], want[0], "merged whole-block gather k")
    eq(merged[:, :, 1], want[1], "merged whole-block gather v")
    dk = torch.zeros_like(kc, device="cuda")
    dv = torch.zeros_like(vc, device="cuda")
    ma.kv_merged_linear_to_paged_multi_layer(merged, dk, dv, slots.cuda())
    wk, wv = np.zeros_like(to_np(kc)), np.zeros_like(to_np(vc))
    O.kv_linear_to_paged_multi_layer(want[0], want[1], wk, wv, slots.numpy())
    eq(dk, wk, "merged whole-block scatter k")
    eq(dv, wv, "merged whole-block scatter v")
