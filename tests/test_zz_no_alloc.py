"""The allocation-free row scatter (``mak_rows_scatter_static``) against the
regular one (``mak_rows_scatter`` with a caller workspace), through the C ABI.

``mak_rows_scatter_static`` serves callers that cannot call cudaMalloc (an
engine that reserved its HBM up front and scatters inside its step loop, or a
foreign-language caller holding only raw pointers from another framework's
allocator); its duplicate-slot scratch is a static device array inside the
library.  Two calls in a row must both match the regular entry point bit for
bit (the second call must not see the first call's scratch contents), also at
exactly the slot limit; a warmed-up call must leave the device's free memory
unchanged; and a call above the slot limit must be refused without touching
anything.

This file is named so pytest collects it last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_SLOTS = 65536  # MAK_STATIC_SCATTER_MAX_SLOTS in include/mak_kvcache.h
MAK_E_UNSUPPORTED = -2


def _planes(tensors, rows_per_block):
    from musa_aiter import _native

    t0 = tensors[0]
    e = t0.element_size()
    if rows_per_block > 1:  # paged [NB, BS, H]
        return _native.rows_desc([t.data_ptr() for t in tensors], rows_per_block, t0.stride(0) * e, t0.stride(1) * e,
                                 t0.shape[0] * t0.shape[1])
    return _native.rows_desc([t.data_ptr() for t in tensors], 1, t0.stride(0) * e, 0, t0.shape[0])


def _scatter_both(lib, linear, paged_a, paged_b, slots, skip):
    """Scatter ``linear`` into ``paged_a`` with the static variant and into ``paged_b`` with the regular one."""
    from musa_aiter import _native

    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    row_bytes = linear[0].shape[1] * linear[0].element_size()
    ld, la = _planes(linear, 1)
    pa, pa_arr = _planes(paged_a, paged_a[0].shape[1])
    rc = lib.mak_rows_scatter_static(ctypes.byref(ld), ctypes.byref(pa), None, row_bytes, ctypes.c_void_p(slots.data_ptr()),
                                     _native.MAK_DT_I64, slots.numel(), skip, stream)
    assert rc == 0, lib.mak_last_error()
    nbytes = int(lib.mak_scatter_workspace_bytes(slots.numel()))
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    pb, pb_arr = _planes(paged_b, paged_b[0].shape[1])
    rc = lib.mak_rows_scatter(ctypes.byref(ld), ctypes.byref(pb), None, row_bytes, ctypes.c_void_p(slots.data_ptr()),
                              _native.MAK_DT_I64, slots.numel(), skip, ctypes.c_void_p(ws.data_ptr()), nbytes, stream)
    assert rc == 0, lib.mak_last_error()
    torch.cuda.synchronize()


def test_static_scratch_scatter_matches_workspace_scatter_twice(cuda_device):
    from musa_aiter import _native

    lib = _native.load()
    g = torch.Generator(device="cuda").manual_seed(11)
    planes, nb, bs, hidden, t_mem = 6, 256, 16, 256, 4000
    base = [torch.randn((nb, bs, hidden), device="cuda", generator=g).to(torch.bfloat16) for _ in range(planes)]
    paged_a = [b.clone() for b in base]
    paged_b = [b.clone() for b in base]

    # call 1: duplicates and negative slots, no prefix skip
    linear = [torch.randn((t_mem, hidden), device="cuda", generator=g).to(torch.bfloat16) for _ in range(planes)]
    slots = torch.randint(-2, nb * bs, (3000,), device="cuda", generator=g)
    slots[100:200] = slots[0:100]  # guaranteed duplicates: the later copies must win
    _scatter_both(lib, linear, paged_a, paged_b, slots, 0)
    for a, b in zip(paged_a, paged_b):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))

    # call 2: new data and slots (different duplicate pattern), prefix skip 5
    linear = [torch.randn((t_mem, hidden), device="cuda", generator=g).to(torch.bfloat16) for _ in range(planes)]
    slots = torch.randint(0, nb * bs // 4, (3900,), device="cuda", generator=g)
    _scatter_both(lib, linear, paged_a, paged_b, slots, 5)
    for a, b in zip(paged_a, paged_b):
        assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_static_scratch_scatter_rejects_oversized_calls(cuda_device):
    from musa_aiter import _native

    lib = _native.load()
    nb, bs, hidden = 8, 16, 64
    paged = [torch.zeros((nb, bs, hidden), device="cuda")]
    linear = [torch.ones((MAX_SLOTS + 1, hidden), device="cuda")]
    slots = torch.zeros(MAX_SLOTS + 1, dtype=torch.int64, device="cuda")
    ld, la = _planes(linear, 1)
    pd, pa = _planes(paged, bs)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.mak_rows_scatter_static(ctypes.byref(ld), ctypes.byref(pd), None, hidden * 4, ctypes.c_void_p(slots.data_ptr()),
                                     _native.MAK_DT_I64, slots.numel(), 0, stream)
    assert rc == MAK_E_UNSUPPORTED
    assert b"static scratch limit" in lib.mak_last_error()
    torch.cuda.synchronize()
    assert torch.count_nonzero(paged[0]) == 0


def test_static_scratch_scatter_at_the_slot_limit_allocates_nothing(cuda_device):
    """A call of exactly MAK_STATIC_SCATTER_MAX_SLOTS slots (the size at which the hash keys,
    hash values and resolved-slot vector fill the fixed array) matches the workspace scatter,
    twice; and once warmed up, a static call leaves the device's free memory unchanged."""
    from musa_aiter import _native

    lib = _native.load()
    g = torch.Generator(device="cuda").manual_seed(12)
    planes, nb, bs, hidden = 2, 8192, 16, 256
    base = [torch.randn((nb, bs, hidden), device="cuda", generator=g).to(torch.bfloat16) for _ in range(planes)]
    paged_a = [b.clone() for b in base]
    paged_b = [b.clone() for b in base]
    for call in range(2):
        linear = [torch.randn((MAX_SLOTS, hidden), device="cuda", generator=g).to(torch.bfloat16) for _ in range(planes)]
        slots = torch.randint(-1, nb * bs // (2 + call), (MAX_SLOTS,), device="cuda", generator=g)
        slots[-4096:] = slots[:4096]  # duplicates across the whole call: the late copies win
        _scatter_both(lib, linear, paged_a, paged_b, slots, 0)
        for a, b in zip(paged_a, paged_b):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16)), f"call {call}"

    # free device memory across a warmed-up static call (no workspace, no allocator)
    ld, la = _planes(linear, 1)
    pa, pa_arr = _planes(paged_a, bs)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    row_bytes = hidden * 2

    def static_call():
        rc = lib.mak_rows_scatter_static(ctypes.byref(ld), ctypes.byref(pa), None, row_bytes,
                                         ctypes.c_void_p(slots.data_ptr()), _native.MAK_DT_I64, slots.numel(), 0, stream)
        assert rc == 0, lib.mak_last_error()

    static_call()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        static_call()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
