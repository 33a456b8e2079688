"""``lmcache_kv_strided_block_transfer`` checked against its page layout written out by hand.

The reference implements this transfer only as a MUSA kernel (csrc/kvcache/kv_transfer_float.mu:
3281-3405; its Python entry, ops/lmcache_kv_transfer.py:1294-1403, returns False without MUSA),
so no reference run can pin it.  This file pins each offset rule to the kernel source instead:
the expected pages and staging rows are built here, byte by byte, from the layout the kernel
states (kv_transfer_float.mu:3288-3296) and computes (:3336-3348), independently of the oracle:

* staging: ``[NL, staging_tokens, row_bytes]``; block ``p`` of the batch, token ``t`` is staging
  row ``offset_in_object + p * BS + t`` (:3330-3334);
* mode 0: the token's row sits at ``block * stride + t * row_bytes`` (:3337);
* mode 1: the row's first ``value_bytes`` sit at ``block * stride + t * value_bytes``, its last
  ``scale_bytes`` at ``block * stride + BS * value_bytes + t * scale_bytes`` (:3339-3347);
* bytes past ``BS * row_bytes`` in a block (the padding up to ``stride``) are never touched.

Every page byte carries a label of (layer, block, token, region, byte) so a wrong offset shows
up as a wrong label.  The CPU test checks the oracle; the GPU test checks the kernel.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import kv_oracle as O

NL, BS, NB = 3, 4, 7
SENTINEL = 0xEE


def _label(layer, blk, t, region, j):
    """Byte label; region 0 = value (or whole mode-0 row), 1 = scale."""
    return (layer * 101 + blk * 37 + t * 11 + region * 59 + j * 3 + 1) & 0xFF


def _case(mode):
    if mode == 0:
        row, vb, sb = 24, 0, 0
    else:
        row, vb, sb = 20, 12, 8
    stride = BS * row + 12  # 12 padding bytes per block
    block_ids = np.array([5, 0, 3, 6, 2], dtype=np.int64)
    idx_start, n_valid, offset = 1, 3, 2  # blocks 0, 3, 6 of the id list, staging rows from 2
    staging_tokens = offset + n_valid * BS + 3
    return row, vb, sb, stride, block_ids, idx_start, n_valid, offset, staging_tokens


def _hand_pages(mode, row, vb, sb, stride):
    """Every block of every layer filled by the layout rules; padding holds SENTINEL."""
    pages = np.full((NL, NB * stride), SENTINEL, np.uint8)
    for layer in range(NL):
        for blk in range(NB):
            base = blk * stride
            for t in range(BS):
                if mode == 0:
                    for j in range(row):
                        pages[layer, base + t * row + j] = _label(layer, blk, t, 0, j)
                else:
                    for j in range(vb):
                        pages[layer, base + t * vb + j] = _label(layer, blk, t, 0, j)
                    for j in range(sb):
                        pages[layer, base + BS * vb + t * sb + j] = _label(layer, blk, t, 1, j)
    return pages


def _hand_staging(mode, row, vb, sb, block_ids, idx_start, n_valid, offset, staging_tokens):
    """The staging rows the paged->staging direction must produce (others SENTINEL)."""
    st = np.full((NL, staging_tokens, row), SENTINEL, np.uint8)
    for layer in range(NL):
        for p in range(n_valid):
            blk = int(block_ids[idx_start + p])
            for t in range(BS):
                r = offset + p * BS + t
                if mode == 0:
                    st[layer, r] = [_label(layer, blk, t, 0, j) for j in range(row)]
                else:
                    st[layer, r, :vb] = [_label(layer, blk, t, 0, j) for j in range(vb)]
                    st[layer, r, vb:] = [_label(layer, blk, t, 1, j) for j in range(sb)]
    return st


def _expected_after_store(mode, row, vb, sb, stride, block_ids, idx_start, n_valid):
    """staging->paged onto SENTINEL pages: the touched blocks get their labelled rows, the
    padding and every untouched block keep SENTINEL."""
    full = _hand_pages(mode, row, vb, sb, stride)
    want = np.full_like(full, SENTINEL)
    for p in range(n_valid):
        blk = int(block_ids[idx_start + p])
        lo, hi = blk * stride, blk * stride + BS * row
        want[:, lo:hi] = full[:, lo:hi]
    return want


@pytest.mark.parametrize("mode", (0, 1))
def test_oracle_matches_kernel_source_layout(mode):
    row, vb, sb, stride, ids, i0, n, off, stt = _case(mode)
    pages = _hand_pages(mode, row, vb, sb, stride)
    staging = np.full((NL, stt, row), SENTINEL, np.uint8)
    O.strided_block_transfer(staging, list(pages), ids, 1, i0, n, off, BS, row, stride, mode, vb, sb)
    assert np.array_equal(staging, _hand_staging(mode, row, vb, sb, ids, i0, n, off, stt))
    back = np.full_like(pages, SENTINEL)
    O.strided_block_transfer(staging, list(back), ids, 0, i0, n, off, BS, row, stride, mode, vb, sb)
    assert np.array_equal(back, _expected_after_store(mode, row, vb, sb, stride, ids, i0, n))


@pytest.mark.gpu
@pytest.mark.parametrize("mode", (0, 1))
def test_kernel_matches_kernel_source_layout(cuda_device, mode):
    import musa_aiter as ma

    row, vb, sb, stride, ids, i0, n, off, stt = _case(mode)
    pages = [torch.from_numpy(p.copy()).cuda() for p in _hand_pages(mode, row, vb, sb, stride)]
    staging = torch.full((NL, stt, row), SENTINEL, dtype=torch.uint8, device="cuda")
    dids = torch.from_numpy(ids).cuda()
    assert ma.lmcache_kv_strided_block_transfer(staging, [p.data_ptr() for p in pages], dids, 1, NL, i0, n, off, stt, BS,
                                                row, stride, mode, vb, sb) is True
    got = staging.cpu().numpy()
    want = _hand_staging(mode, row, vb, sb, ids, i0, n, off, stt)
    assert np.array_equal(got, want), np.argwhere(got != want)[:5]
    blank = [torch.full((NB * stride,), SENTINEL, dtype=torch.uint8, device="cuda") for _ in range(NL)]
    assert ma.lmcache_kv_strided_block_transfer(staging, [p.data_ptr() for p in blank], dids, 0, NL, i0, n, off, stt, BS,
                                                row, stride, mode, vb, sb) is True
    got = torch.stack(blank).cpu().numpy()
    want = _expected_after_store(mode, row, vb, sb, stride, ids, i0, n)
    assert np.array_equal(got, want), np.argwhere(got != want)[:5]
