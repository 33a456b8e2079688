"""The ``cache`` family on B200: RoPE and the decode-loop KV-cache write.

Same public ABI as the reference (musa_aiter/ops/cache.py): ``apply_rope``,
``apply_rope_to_key_cache`` and ``copy_to_kv_cache`` keep their names,
arguments, return values and error messages, and run as sm_100a kernels.

Arithmetic follows the reference bit for bit: ``x1 * cos - x2 * sin`` and
``x1 * sin + x2 * cos`` with PyTorch's type promotion per operation (each
product in the promoted type of its operands, the sum / difference in the
promoted type of the products, f16 / bf16 steps rounded after every
operation), then cast to ``x.dtype`` (csrc/rope.cu).  ``copy_to_kv_cache`` is
the tile-engine scatter of ``kv_linear_to_paged`` with the reference's
validation; repeated slots keep the reference's token order (last writer wins
for the copy; successive rotations for ``apply_rope_to_key_cache``).
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from .. import _native
from ..dispatch import emit_native
from ._common import kernel_slots, require_cuda, validation_enabled

__all__ = ["apply_rope", "apply_rope_to_key_cache", "copy_to_kv_cache"]

_FLOAT_CODES = {torch.float16: _native.MAK_DT_F16, torch.bfloat16: _native.MAK_DT_BF16, torch.float32: _native.MAK_DT_F32}


class RopeDenseDesc(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p), ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("out", ctypes.c_void_p),
        ("rows", ctypes.c_int64), ("half", ctypes.c_int64), ("sizes", ctypes.c_int64 * 6),
        ("x_strides", ctypes.c_int64 * 7), ("cos_strides", ctypes.c_int64 * 7), ("sin_strides", ctypes.c_int64 * 7),
        ("ndim", ctypes.c_int32), ("interleaved", ctypes.c_int32),
        ("x_dtype", ctypes.c_int32), ("cos_dtype", ctypes.c_int32), ("sin_dtype", ctypes.c_int32),
        ("prod1_dtype", ctypes.c_int32), ("prod2_dtype", ctypes.c_int32), ("sum_dtype", ctypes.c_int32),
        ("out_dtype", ctypes.c_int32), ("reserved", ctypes.c_int32),
    ]


class RopeCacheDesc(ctypes.Structure):
    _fields_ = [
        ("cache", ctypes.c_void_p), ("cos", ctypes.c_void_p), ("sin", ctypes.c_void_p), ("slots", ctypes.c_void_p),
        ("positions", ctypes.c_void_p), ("n_tokens", ctypes.c_int64), ("num_blocks", ctypes.c_int64),
        ("num_heads", ctypes.c_int64), ("head_dim", ctypes.c_int64), ("block_size", ctypes.c_int64),
        ("stride_block", ctypes.c_int64), ("stride_head", ctypes.c_int64), ("stride_dim", ctypes.c_int64),
        ("cos_stride_row", ctypes.c_int64), ("cos_stride_last", ctypes.c_int64),
        ("sin_stride_row", ctypes.c_int64), ("sin_stride_last", ctypes.c_int64),
        ("slot_dtype", ctypes.c_int32), ("pos_dtype", ctypes.c_int32), ("cache_dtype", ctypes.c_int32),
        ("cos_dtype", ctypes.c_int32), ("sin_dtype", ctypes.c_int32), ("prod1_dtype", ctypes.c_int32),
        ("prod2_dtype", ctypes.c_int32), ("sum_dtype", ctypes.c_int32), ("interleaved", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


def _code(dtype: torch.dtype, name: str) -> int:
    try:
        return _FLOAT_CODES[dtype]
    except KeyError:
        raise ValueError(f"{name}: the B200 backend supports float16, bfloat16 and float32 tensors, got {dtype}") from None


def _promotions(x_part: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> tuple[torch.dtype, torch.dtype, torch.dtype]:
    """Result types of x*cos, x*sin and of their sum (torch's rules, 0-dim operands included)."""
    r1 = torch.result_type(x_part, cos)
    r2 = torch.result_type(x_part, sin)
    return r1, r2, torch.promote_types(r1, r2)


def apply_rope(
    x: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    *,
    interleaved: bool = False,
) -> torch.Tensor:
    """Apply rotary positional embedding to a tensor (reference musa_aiter/ops/cache.py:9-42).

    x: [..., head_dim]; cos / sin broadcastable to x[..., :head_dim/2].  Returns a new tensor of
    x's dtype whose shape is the broadcast of x with cos / sin (on the head_dim axis: head_dim).
    """
    if x.shape[-1] % 2 != 0:
        raise ValueError("head_dim must be even for RoPE")
    name = "apply_rope"
    require_cuda(name, x, cos, sin)
    half = x.shape[-1] // 2
    x_part = x[..., :half]
    shape = torch.broadcast_shapes(x_part.shape, cos.shape, sin.shape)
    out_shape = tuple(shape[:-1]) + (2 * half,)
    out = torch.empty(out_shape, dtype=x.dtype, device=x.device)
    lead = len(shape) - 1
    if lead > 6:
        raise ValueError(f"{name}: at most 6 leading dimensions are supported, got {lead}")
    if out.numel() == 0:
        return out
    xe = x.expand(tuple(shape[:-1]) + (x.shape[-1],))
    ce = cos.expand(shape)
    se = sin.expand(shape)
    r1, r2, r3 = _promotions(x_part, cos, sin)
    d = RopeDenseDesc()
    d.x, d.cos, d.sin, d.out = xe.data_ptr(), ce.data_ptr(), se.data_ptr(), out.data_ptr()
    rows = 1
    for i, n in enumerate(shape[:-1]):
        d.sizes[i] = int(n)
        d.x_strides[i] = xe.stride(i)
        d.cos_strides[i] = ce.stride(i)
        d.sin_strides[i] = se.stride(i)
        rows *= int(n)
    d.x_strides[6] = xe.stride(-1)
    d.cos_strides[6] = ce.stride(-1)
    d.sin_strides[6] = se.stride(-1)
    d.rows, d.half, d.ndim, d.interleaved = rows, half, lead, int(bool(interleaved))
    d.x_dtype, d.cos_dtype, d.sin_dtype = _code(x.dtype, name), _code(cos.dtype, name), _code(sin.dtype, name)
    d.prod1_dtype, d.prod2_dtype, d.sum_dtype = _code(r1, name), _code(r2, name), _code(r3, name)
    d.out_dtype = _code(x.dtype, name)
    _native.check(_native.load().mak_rope_dense(ctypes.byref(d), _native.stream_ptr(x.device)), name)
    emit_native(name, x, "sm100a rope kernel (reference rounding per operation)")
    return out


def _occurrence_rounds(s: np.ndarray) -> list[np.ndarray] | None:
    """Token indices split into rounds of distinct slots, in token order; None when all distinct."""
    valid = np.nonzero(s >= 0)[0]
    if np.unique(s[valid]).size == valid.size:
        return None
    rank = np.zeros(s.size, dtype=np.int64)
    seen: dict[int, int] = {}
    for t in valid.tolist():
        k = int(s[t])
        rank[t] = seen.get(k, 0)
        seen[k] = rank[t] + 1
    return [valid[rank[valid] == r] for r in range(int(rank[valid].max()) + 1)]


def apply_rope_to_key_cache(
    key_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
    positions: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    *,
    interleaved: bool = False,
) -> torch.Tensor:
    """Rotate key_cache[block, :, :, offset] in place for each token (reference cache.py:45-102).

    With validation on (the default) slots and positions are read back once for the reference's
    checks, and repeated slots are rotated in successive launches in token order.  With
    ``MUSA_AITER_SKIP_VALIDATION=1`` nothing is read back and a call must not repeat a slot."""
    if key_cache.dim() != 4:
        raise ValueError("apply_rope_to_key_cache: key_cache must be [blocks, heads, head_dim, block_size]")
    if slot_mapping.dim() != 1 or positions.dim() != 1 or slot_mapping.numel() != positions.numel():
        raise ValueError("apply_rope_to_key_cache: slot_mapping and positions must be same-length vectors")
    if slot_mapping.dtype not in (torch.int16, torch.int32, torch.int64):
        raise ValueError("apply_rope_to_key_cache: slot_mapping must use an integer dtype")
    if positions.dtype not in (torch.int16, torch.int32, torch.int64):
        raise ValueError("apply_rope_to_key_cache: positions must use an integer dtype")
    if key_cache.shape[2] % 2 != 0:
        raise ValueError("apply_rope_to_key_cache: head_dim must be even for RoPE")
    if slot_mapping.device != key_cache.device or positions.device != key_cache.device:
        raise ValueError("apply_rope_to_key_cache: slot_mapping and positions must be on key_cache device")
    if cos.device != key_cache.device or sin.device != key_cache.device:
        raise ValueError("apply_rope_to_key_cache: cos/sin must be on key_cache device")
    if cos.shape != sin.shape or cos.dim() not in (1, 2):
        raise ValueError("apply_rope_to_key_cache: cos/sin must be [half_dim] or [max_positions, half_dim]")
    half = key_cache.shape[2] // 2
    if cos.shape[-1] != half:
        raise ValueError("apply_rope_to_key_cache: cos/sin last dim must equal head_dim / 2")
    name = "apply_rope_to_key_cache"
    require_cuda(name, key_cache, slot_mapping, positions, cos, sin)
    nb, nh, hd, bs = map(int, key_cache.shape)
    if key_cache.stride(3) != 1 and bs != 1:
        raise ValueError(f"{name}: the block_size axis must be contiguous")
    ks, kcode = kernel_slots(slot_mapping)
    ps, pcode = kernel_slots(positions)
    rounds = None
    if slot_mapping.numel() and validation_enabled():
        # The reference walks the tokens on the host and raises on the first bad one
        # (cache.py:86-99); one read-back of slots and positions gives the same checks
        # before any cache row changes, and the rounds for repeated slots.
        s_host = ks.detach().to("cpu", torch.int64).numpy()
        p_host = ps.detach().to("cpu", torch.int64).numpy()
        for t in np.nonzero(s_host >= 0)[0].tolist():
            block_id = int(s_host[t]) // bs
            if block_id >= nb:
                raise ValueError(f"apply_rope_to_key_cache: slot maps to invalid block_id={block_id}")
            position = int(p_host[t])
            if position < 0:
                raise ValueError("apply_rope_to_key_cache: positions must be non-negative")
            if cos.dim() == 2 and position >= cos.shape[0]:
                raise ValueError("apply_rope_to_key_cache: position exceeds cos/sin table")
        rounds = _occurrence_rounds(s_host)
    x_part = key_cache[0, :, :half, 0]
    r1, r2, r3 = _promotions(x_part, cos[0] if cos.dim() == 2 else cos, sin[0] if sin.dim() == 2 else sin)
    d = RopeCacheDesc()
    d.cache, d.cos, d.sin = key_cache.data_ptr(), cos.data_ptr(), sin.data_ptr()
    d.num_blocks, d.num_heads, d.head_dim, d.block_size = nb, nh, hd, bs
    d.stride_block, d.stride_head, d.stride_dim = key_cache.stride(0), key_cache.stride(1), key_cache.stride(2)
    d.cos_stride_row = cos.stride(0) if cos.dim() == 2 else 0
    d.cos_stride_last = cos.stride(-1)
    d.sin_stride_row = sin.stride(0) if sin.dim() == 2 else 0
    d.sin_stride_last = sin.stride(-1)
    d.slot_dtype, d.pos_dtype = kcode, pcode
    d.cache_dtype, d.cos_dtype, d.sin_dtype = _code(key_cache.dtype, name), _code(cos.dtype, name), _code(sin.dtype, name)
    d.prod1_dtype, d.prod2_dtype, d.sum_dtype = _code(r1, name), _code(r2, name), _code(r3, name)
    d.interleaved = int(bool(interleaved))
    lib = _native.load()
    stream = _native.stream_ptr(key_cache.device)
    if rounds is None:
        d.slots, d.positions, d.n_tokens = ks.data_ptr(), ps.data_ptr(), ks.numel()
        _native.check(lib.mak_rope_key_cache(ctypes.byref(d), stream), name)
    else:
        # Repeated slots: successive calls, each with distinct slots, in token order.
        for toks in rounds:
            idx = torch.from_numpy(toks).to(key_cache.device)
            rs, rp = ks[idx].contiguous(), ps[idx].contiguous()
            d.slots, d.positions, d.n_tokens = rs.data_ptr(), rp.data_ptr(), rs.numel()
            _native.check(lib.mak_rope_key_cache(ctypes.byref(d), stream), name)
    emit_native(name, key_cache, "sm100a in-place rope on selected cache slots")
    return key_cache


def copy_to_kv_cache(
    k: torch.Tensor,
    v: torch.Tensor,
    key_cache: torch.Tensor,
    value_cache: torch.Tensor,
    slot_mapping: torch.Tensor,
) -> None:
    """Reference KV-cache update (musa_aiter/ops/cache.py:105-144) on the tile engine.

    k/v [num_tokens, num_kv_heads, head_dim] -> caches [num_blocks, num_kv_heads, head_dim, block_size]
    at slot_mapping (negative slots skipped, last writer wins)."""
    if k.shape != v.shape:
        raise ValueError("k and v shapes must match")
    if key_cache.shape != value_cache.shape:
        raise ValueError("key_cache and value_cache shapes must match")
    if k.dim() != 3 or key_cache.dim() != 4:
        raise ValueError("k/v must be 3D and caches must be 4D")
    if slot_mapping.numel() != k.shape[0]:
        raise ValueError("slot_mapping length must equal number of tokens")
    if k.device != key_cache.device or v.device != value_cache.device or slot_mapping.device != k.device:
        raise ValueError("all tensors must be on same device")
    name = "copy_to_kv_cache"
    require_cuda(name, k, v, key_cache, value_cache, slot_mapping)
    nb, nh, hd, bs = map(int, key_cache.shape)
    if tuple(k.shape[1:]) != (nh, hd):
        raise ValueError(f"{name}: k/v [num_tokens, num_kv_heads, head_dim] must match the cache heads and head_dim")
    if k.dtype != key_cache.dtype or v.dtype != value_cache.dtype or k.dtype != v.dtype:
        raise ValueError(f"{name}: k/v and cache dtypes must match")
    ks, code = kernel_slots(slot_mapping)
    if ks.numel() == 0:
        return None
    if validation_enabled():
        max_slot = int(ks.max().item()) if ks.numel() else -1
        if max_slot >= 0 and max_slot // bs >= nb:
            raise ValueError(f"slot maps to invalid block_id={max_slot // bs}")
    kc = key_cache if key_cache.stride(3) == 1 or bs == 1 else None
    vc = value_cache if value_cache.stride(3) == 1 or bs == 1 else None
    if kc is None or vc is None:
        raise ValueError(f"{name}: the block_size axis of the caches must be contiguous")
    kl = k if k.stride(2) == 1 else k.contiguous()
    vl = v if v.stride(2) == 1 else v.contiguous()
    if vl.stride() != kl.stride():
        vl = vl.contiguous()
        kl = kl.contiguous()
    from .kv_transfer import _tile_scatter  # noqa: PLC0415 (kv_transfer does not import this module)

    # owner-table last-writer resolution and segment map, as the other tile scatters
    _tile_scatter(kl, vl, kc, vc, ks, layered=False, op=name)
    emit_native(name, k, "sm100a tile scatter (copy_to_kv_cache)")
    return None
