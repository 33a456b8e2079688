"""CPU oracle for the musa-aiter ``kvcache`` hot path — TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithms of the reference's PyTorch
implementation of the KV-cache movement and FP8 quantization path
(MooreThreads/musa-aiter v0.5.0).  It is the checker the CUDA kernels are
compared against: only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it.
The product path (``musa_aiter``) never imports or calls it.

Parity pinning: every function here is checked bit-for-bit against golden
vectors produced by running the reference itself (``tests/golden/make_golden.py``
imports the reference package and records inputs and outputs;
``tests/test_oracle_golden.py`` replays them).

Conventions:
- bfloat16 data is carried as ``uint16`` bit patterns (numpy has no bf16);
  float16 and float32 use numpy's own types.  Copies are bit copies.
- "slots" are ``block_id * block_size + offset``; negative slots are skipped.
- Scatters follow the reference's sequential token loop, so with duplicate
  slots the LAST token wins (musa_aiter/ops/kv_transfer.py:3092-3112).
"""

from __future__ import annotations

from concurrent.futures import ThreadPoolExecutor

import numpy as np

# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------


def last_writer_mask(slots: np.ndarray) -> np.ndarray:
    """True at index t when slots[t] >= 0 and no later index holds the same slot.

    Equivalent to the reference's in-order token loop with overwrite
    (musa_aiter/ops/kv_transfer.py:3104-3112, ops/lmcache_kv_transfer.py:90-96).
    """
    slots = np.asarray(slots, dtype=np.int64)
    keep = np.zeros(slots.shape[0], dtype=bool)
    valid = np.nonzero(slots >= 0)[0]
    if valid.size == 0:
        return keep
    rev = valid[::-1]
    _, first_in_rev = np.unique(slots[rev], return_index=True)
    keep[rev[first_in_rev]] = True
    return keep


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit pattern (torch's ``.to(bfloat16)``)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, np.uint16(0x7FC0), rounded)


def to_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return bf16_bits_to_f32(x)
    return np.asarray(x).astype(np.float32)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bfloat16":
        return f32_to_bf16_bits(x)
    if dtype == "float16":
        with np.errstate(over="ignore"):
            return np.asarray(x, dtype=np.float32).astype(np.float16)
    return np.asarray(x, dtype=np.float32)


# ---------------------------------------------------------------------------
# FP8 codec (musa_aiter/ops/kv_transfer.py:2094-2200)
# ---------------------------------------------------------------------------


def normalize_fp8_format(fp8_format: str) -> str:
    """musa_aiter/ops/kv_transfer.py:2094-2100."""
    n = fp8_format.lower().replace("-", "_")
    if n in ("fp8", "fp8_e4m3", "fp8_e4m3fn", "e4m3", "e4m3fn"):
        return "e4m3"
    if n in ("fp8_e5m2", "e5m2"):
        return "e5m2"
    raise ValueError(f"unsupported FP8 KV cache format: {fp8_format}")


def fp8_format_params(fp8_format: str) -> tuple[int, int, int, int]:
    """(exponent bits, mantissa bits, bias, max unbiased exponent): kv_transfer.py:2103-2107."""
    if normalize_fp8_format(fp8_format) == "e4m3":
        return 4, 3, 7, 8
    return 5, 2, 15, 16


def fp8_quantize_to_uint8(x_f32: np.ndarray, scale: np.ndarray | float, fp8_format: str) -> np.ndarray:
    """Restates ``_fp8_quantize_to_uint8`` (musa_aiter/ops/kv_transfer.py:2161-2183).

    ``floor(log2(safe))`` is taken exactly from ``frexp``; the reference's
    overflow branch (mantissa == 2^m -> exponent + 1) makes the result the same
    for any log2 that is off by one ulp around powers of two, and the
    exhaustive golden vectors pin it.
    """
    _, mb, bias, emax = fp8_format_params(fp8_format)
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        work = (np.asarray(x_f32, dtype=np.float32) / np.asarray(scale, dtype=np.float32)).astype(np.float32)
    sign = work < 0
    a = np.abs(work)
    a = np.where(np.isfinite(a), a, np.float32(0.0))
    max_value = np.float32((2.0 - 2.0 ** (-mb)) * (2.0**emax))
    min_normal = np.float32(2.0 ** (1 - bias))
    clipped = np.minimum(a, max_value)
    nonzero = clipped >= min_normal
    safe = np.where(nonzero, clipped, np.float32(1.0)).astype(np.float32)
    _, e2 = np.frexp(safe)
    exponent = (e2 - 1).astype(np.int32)
    exponent = np.clip(exponent, 1 - bias, emax)
    base = np.ldexp(np.float32(1.0), exponent).astype(np.float32)
    mant_f = ((safe / base - np.float32(1.0)) * np.float32(2**mb)).astype(np.float32)
    mantissa = np.round(mant_f).astype(np.int32)  # numpy rounds half to even, like torch.round
    overflow = mantissa == (1 << mb)
    exponent = np.minimum(np.where(overflow, exponent + 1, exponent), emax)
    mantissa = np.clip(np.where(overflow, 0, mantissa), 0, (1 << mb) - 1)
    exponent_field = np.where(nonzero, exponent + bias, 0)
    mantissa = np.where(nonzero, mantissa, 0)
    bits = (sign.astype(np.int32) << 7) | (exponent_field << mb) | mantissa
    return bits.astype(np.uint8)


def fp8_decode_f32(codes: np.ndarray, fp8_format: str) -> np.ndarray:
    """Value part of ``_fp8_dequantize_from_uint8`` (kv_transfer.py:2186-2200), before scaling."""
    _, mb, bias, _ = fp8_format_params(fp8_format)
    bits = np.asarray(codes).astype(np.int32)
    sign = (bits >> 7) & 1
    exponent_field = (bits >> mb) & ((1 << (7 - mb)) - 1)
    mantissa = bits & ((1 << mb) - 1)
    nonzero = exponent_field != 0
    value = (np.float32(1.0) + mantissa.astype(np.float32) / np.float32(2**mb)) * np.ldexp(
        np.float32(1.0), exponent_field - bias
    ).astype(np.float32)
    value = value.astype(np.float32)
    value = np.where(nonzero, value, np.float32(0.0))
    value = np.where(sign > 0, -value, value)
    return value.astype(np.float32)


def fp8_dequantize_from_uint8(codes: np.ndarray, scale, fp8_format: str, out_dtype: str) -> np.ndarray:
    """``(decode(code) * scale).to(out_dtype)`` in fp32 then RNE (kv_transfer.py:2186-2200)."""
    value = fp8_decode_f32(codes, fp8_format)
    return from_f32((value * np.asarray(scale, dtype=np.float32)).astype(np.float32), out_dtype)


def _scale_for_head(scale: np.ndarray, head_dim: int) -> np.ndarray:
    """kv_transfer.py:2124-2127: scalar stays scalar, [NH] -> [NH, HD] broadcast."""
    scale = np.asarray(scale, dtype=np.float32)
    if scale.ndim == 0:
        return scale
    return np.broadcast_to(scale.reshape(-1, 1), (scale.shape[-1], head_dim))


def _scale_for_layer_head(scale: np.ndarray, layer: int, head_dim: int) -> np.ndarray:
    """kv_transfer.py:2130-2135."""
    scale = np.asarray(scale, dtype=np.float32)
    if scale.ndim <= 1:
        return _scale_for_head(scale, head_dim)
    return np.broadcast_to(scale[layer].reshape(-1, 1), (scale.shape[-1], head_dim))


# ---------------------------------------------------------------------------
# tile caches [NB, NH, HD, BS] (musa_aiter/ops/kv_transfer.py:3047-3112)
# ---------------------------------------------------------------------------


def paged_to_linear(cache: np.ndarray, slots: np.ndarray, *, fill_skipped: str = "zeros", out: np.ndarray | None = None) -> np.ndarray:
    """One plane of ``_kv_paged_to_linear_compute`` (kv_transfer.py:3047-3089)."""
    nb, nh, hd, bs = cache.shape
    slots = np.asarray(slots, dtype=np.int64)
    valid = slots >= 0
    safe = np.where(valid, slots, 0)
    bid, off = safe // bs, safe % bs
    gathered = cache[bid, :, :, off]  # [T, NH, HD]
    if out is None:
        if fill_skipped == "preserve":
            raise ValueError("fill_skipped=preserve requires an out buffer")
        res = np.zeros_like(gathered)
        res[valid] = gathered[valid]
        return res
    if fill_skipped == "zeros":
        out[...] = 0
    out[valid] = gathered[valid]
    return out


def linear_to_paged(lin: np.ndarray, cache: np.ndarray, slots: np.ndarray) -> None:
    """One plane of ``_kv_linear_to_paged_scatter`` (kv_transfer.py:3092-3112), last writer wins."""
    bs = cache.shape[3]
    slots = np.asarray(slots, dtype=np.int64)
    keep = last_writer_mask(slots)
    t = np.nonzero(keep)[0]
    s = slots[t]
    cache[s // bs, :, :, s % bs] = lin[t]


def kv_paged_to_linear(k_cache, v_cache, slots, *, fill_skipped="zeros", out_k=None, out_v=None):
    """kv_transfer.py:3115-3206 (single layer)."""
    return (
        paged_to_linear(k_cache, slots, fill_skipped=fill_skipped, out=out_k),
        paged_to_linear(v_cache, slots, fill_skipped=fill_skipped, out=out_v),
    )


def kv_linear_to_paged(k_lin, v_lin, k_cache, v_cache, slots) -> None:
    """kv_transfer.py:3312-3379 (single layer)."""
    linear_to_paged(k_lin, k_cache, slots)
    linear_to_paged(v_lin, v_cache, slots)


def _map_layers(fn, n: int, threads: int):
    if threads <= 1 or n <= 1:
        return [fn(i) for i in range(n)]
    with ThreadPoolExecutor(max_workers=threads) as pool:
        return list(pool.map(fn, range(n)))


def kv_paged_to_linear_multi_layer(k_cache, v_cache, slots, *, fill_skipped="zeros", out_k=None, out_v=None, threads: int = 1):
    """kv_transfer.py:3209-3309: per-layer gather, stacked to [L, T, NH, HD]."""
    nl = k_cache.shape[0]
    t = np.asarray(slots).shape[0]
    if out_k is None:
        out_k = np.zeros((nl, t) + k_cache.shape[2:4], dtype=k_cache.dtype)
        out_v = np.zeros((nl, t) + v_cache.shape[2:4], dtype=v_cache.dtype)

    def one(i):
        paged_to_linear(k_cache[i], slots, fill_skipped=fill_skipped, out=out_k[i])
        paged_to_linear(v_cache[i], slots, fill_skipped=fill_skipped, out=out_v[i])

    _map_layers(one, nl, threads)
    return out_k, out_v


def kv_linear_to_paged_multi_layer(k_lin, v_lin, k_cache, v_cache, slots, *, threads: int = 1) -> None:
    """kv_transfer.py:3382-3457."""

    def one(i):
        linear_to_paged(k_lin[i], k_cache[i], slots)
        linear_to_paged(v_lin[i], v_cache[i], slots)

    _map_layers(one, k_cache.shape[0], threads)


# ---- FP8 tile caches (kv_transfer.py:2203-2398) -----------------------------


def kv_linear_to_paged_fp8(k_lin, v_lin, k_cache8, v_cache8, slots, k_scale, v_scale, *, fp8_format="e4m3", lin_dtype="bfloat16"):
    """kv_transfer.py:2203-2247: per-token quantize + scatter of raw bytes (last writer wins)."""
    hd = k_cache8.shape[2]
    bs = k_cache8.shape[3]
    slots = np.asarray(slots, dtype=np.int64)
    keep = last_writer_mask(slots)
    t = np.nonzero(keep)[0]
    s = slots[t]
    ks = _scale_for_head(k_scale, hd)
    vs = _scale_for_head(v_scale, hd)
    k_cache8[s // bs, :, :, s % bs] = fp8_quantize_to_uint8(to_f32(k_lin[t], lin_dtype), ks, fp8_format)
    v_cache8[s // bs, :, :, s % bs] = fp8_quantize_to_uint8(to_f32(v_lin[t], lin_dtype), vs, fp8_format)


def kv_paged_fp8_to_linear(k_cache8, v_cache8, slots, k_scale, v_scale, *, out_dtype="bfloat16", fp8_format="e4m3"):
    """kv_transfer.py:2250-2301: gather + dequantize, zeros for skipped slots."""
    nb, nh, hd, bs = k_cache8.shape
    slots = np.asarray(slots, dtype=np.int64)
    valid = slots >= 0
    safe = np.where(valid, slots, 0)
    outs = []
    for cache, scale in ((k_cache8, k_scale), (v_cache8, v_scale)):
        codes = cache[safe // bs, :, :, safe % bs]
        vals = fp8_dequantize_from_uint8(codes, _scale_for_head(scale, hd), fp8_format, out_dtype)
        vals[~valid] = 0
        outs.append(vals)
    return outs[0], outs[1]


def kv_linear_to_paged_fp8_multi_layer(k_lin, v_lin, k_cache8, v_cache8, slots, k_scale, v_scale, *, fp8_format="e4m3", lin_dtype="bfloat16", threads: int = 1):
    """kv_transfer.py:2304-2347 (scale scalar, [NH] or [L, NH])."""
    hd, bs = k_cache8.shape[3], k_cache8.shape[4]
    slots = np.asarray(slots, dtype=np.int64)
    keep = last_writer_mask(slots)
    t = np.nonzero(keep)[0]
    s = slots[t]

    def one(layer):
        ks = _scale_for_layer_head(k_scale, layer, hd)
        vs = _scale_for_layer_head(v_scale, layer, hd)
        k_cache8[layer, s // bs, :, :, s % bs] = fp8_quantize_to_uint8(to_f32(k_lin[layer, t], lin_dtype), ks, fp8_format)
        v_cache8[layer, s // bs, :, :, s % bs] = fp8_quantize_to_uint8(to_f32(v_lin[layer, t], lin_dtype), vs, fp8_format)

    _map_layers(one, k_cache8.shape[0], threads)


def kv_paged_fp8_to_linear_multi_layer(k_cache8, v_cache8, slots, k_scale, v_scale, *, out_dtype="bfloat16", fp8_format="e4m3", threads: int = 1):
    """kv_transfer.py:2350-2398."""
    nl, nb, nh, hd, bs = k_cache8.shape
    slots = np.asarray(slots, dtype=np.int64)
    valid = slots >= 0
    safe = np.where(valid, slots, 0)
    npdt = {"bfloat16": np.uint16, "float16": np.float16, "float32": np.float32}[out_dtype]
    out_k = np.zeros((nl, slots.shape[0], nh, hd), dtype=npdt)
    out_v = np.zeros_like(out_k)

    def one(layer):
        for cache, scale, out in ((k_cache8, k_scale, out_k), (v_cache8, v_scale, out_v)):
            codes = cache[layer, safe // bs, :, :, safe % bs]
            vals = fp8_dequantize_from_uint8(codes, _scale_for_layer_head(scale, layer, hd), fp8_format, out_dtype)
            vals[~valid] = 0
            out[layer] = vals

    _map_layers(one, nl, threads)
    return out_k, out_v


def kv_merged_linear_to_paged_fp8(merged, k_cache8, v_cache8, slots, k_scale, v_scale, *, fp8_format="e4m3",
                                  lin_dtype="bfloat16"):
    """kv_transfer.py:3489-3505: the K half ``merged[:, 0]`` and V half ``merged[:, 1]`` of a
    ``[T, 2, NH, HD]`` buffer go through the single-layer FP8 store."""
    kv_linear_to_paged_fp8(merged[:, 0], merged[:, 1], k_cache8, v_cache8, slots, k_scale, v_scale,
                           fp8_format=fp8_format, lin_dtype=lin_dtype)


def kv_paged_fp8_to_merged_linear(k_cache8, v_cache8, slots, k_scale, v_scale, *, out_dtype="bfloat16", fp8_format="e4m3"):
    """kv_transfer.py:3460-3486: FP8 gather + dequantize into ``[T, 2, NH, HD]`` (K at 0, V at 1)."""
    ok, ov = kv_paged_fp8_to_linear(k_cache8, v_cache8, slots, k_scale, v_scale, out_dtype=out_dtype, fp8_format=fp8_format)
    return np.stack([ok, ov], axis=1)


def kv_merged_linear_to_paged_fp8_multi_layer(merged, k_cache8, v_cache8, slots, k_scale, v_scale, *, fp8_format="e4m3",
                                              lin_dtype="bfloat16"):
    """kv_transfer.py:3537-3553: ``[L, T, 2, NH, HD]`` halves through the multi-layer FP8 store."""
    kv_linear_to_paged_fp8_multi_layer(merged[:, :, 0], merged[:, :, 1], k_cache8, v_cache8, slots, k_scale, v_scale,
                                       fp8_format=fp8_format, lin_dtype=lin_dtype)


def kv_paged_fp8_to_merged_linear_multi_layer(k_cache8, v_cache8, slots, k_scale, v_scale, *, out_dtype="bfloat16",
                                              fp8_format="e4m3"):
    """kv_transfer.py:3508-3534: multi-layer FP8 gather + dequantize into ``[L, T, 2, NH, HD]``."""
    ok, ov = kv_paged_fp8_to_linear_multi_layer(k_cache8, v_cache8, slots, k_scale, v_scale, out_dtype=out_dtype,
                                                fp8_format=fp8_format)
    return np.stack([ok, ov], axis=2)


# ---------------------------------------------------------------------------
# row caches (LMCache / SGLang MP / MLA flat): musa_aiter/ops/lmcache_kv_transfer.py
# ---------------------------------------------------------------------------


def rows_gather(plane_rows: np.ndarray, slots: np.ndarray, n_out: int | None = None) -> np.ndarray:
    """Gather rows of one plane ``[num_rows, W]`` at ``slots``; zeros for skipped slots and
    for tail rows beyond len(slots) (the reference zeroes the whole buffer first,
    ops/lmcache_kv_transfer.py:107-115, 258-269, 488-502)."""
    slots = np.asarray(slots, dtype=np.int64)
    t = slots.shape[0]
    n_out = t if n_out is None else n_out
    out = np.zeros((n_out,) + plane_rows.shape[1:], dtype=plane_rows.dtype)
    valid = np.nonzero(slots[: min(t, n_out)] >= 0)[0]
    out[valid] = plane_rows[slots[valid]]
    return out


def rows_scatter(buf_rows: np.ndarray, plane_rows: np.ndarray, slots: np.ndarray, skip_prefix: int = 0) -> None:
    """plane_rows[slots[t]] = buf_rows[skip_prefix + t], in token order (last writer wins)."""
    slots = np.asarray(slots, dtype=np.int64)
    keep = last_writer_mask(slots)
    t = np.nonzero(keep)[0]
    plane_rows[slots[t]] = buf_rows[skip_prefix + t]


def lmcache_paged_to_kv_buffer(paged: np.ndarray, kv_buffer: np.ndarray, slots: np.ndarray) -> None:
    """6-D ``[NL, 2, NB, BS, NH, HS]`` -> ``[2, NL, T, NH*HS]`` (lmcache_kv_transfer.py:101-115)."""
    nl, _, nb, bs, nh, hs = paged.shape
    for kv in range(2):
        for layer in range(nl):
            rows = paged[layer, kv].reshape(nb * bs, nh * hs)
            kv_buffer[kv, layer] = rows_gather(rows, slots, kv_buffer.shape[2])


def lmcache_kv_buffer_to_paged(kv_buffer: np.ndarray, paged: np.ndarray, slots: np.ndarray) -> None:
    """``[2, NL, T, H]`` -> 6-D cache (lmcache_kv_transfer.py:51-98, non-list branch)."""
    nl, _, nb, bs, nh, hs = paged.shape
    for kv in range(2):
        for layer in range(nl):
            rows = paged[layer, kv].reshape(nb * bs, nh * hs)
            rows_scatter(kv_buffer[kv, layer], rows, slots)


def lmcache_list_paged_to_buffer(kvcaches: list[np.ndarray], memory: np.ndarray, slots: np.ndarray, *, threads: int = 1) -> None:
    """List of ``[2, NB, BS, NH, HS]`` -> ``[2, NL, T, H]`` (lmcache_kv_transfer.py:473-490)."""

    def one(layer):
        cache = kvcaches[layer]
        nb, bs = cache.shape[1], cache.shape[2]
        for kv in range(2):
            memory[kv, layer] = rows_gather(cache[kv].reshape(nb * bs, -1), slots, memory.shape[2])

    _map_layers(one, len(kvcaches), threads)


def lmcache_list_buffer_to_paged(memory: np.ndarray, kvcaches: list[np.ndarray], slots: np.ndarray, skip_prefix: int = 0, *, threads: int = 1) -> None:
    """``[2, NL, T, H]`` -> list of ``[2, NB, BS, NH, HS]`` (lmcache_kv_transfer.py:451-470)."""

    def one(layer):
        cache = kvcaches[layer]
        nb, bs = cache.shape[1], cache.shape[2]
        for kv in range(2):
            rows_scatter(memory[kv, layer], cache[kv].reshape(nb * bs, -1), slots, skip_prefix)

    _map_layers(one, len(kvcaches), threads)


def lmcache_two_x_nl_paged_to_buffer(kvcaches: list[list[np.ndarray]], memory: np.ndarray, slots: np.ndarray) -> None:
    """SGLang MP ``2 x NL x [NB, BS, NH, HS]`` -> ``[2, NL, T, H]`` (lmcache_kv_transfer.py:229-269)."""
    for kv in range(2):
        for layer, cache in enumerate(kvcaches[kv]):
            nb, bs = cache.shape[0], cache.shape[1]
            memory[kv, layer] = rows_gather(cache.reshape(nb * bs, -1), slots, memory.shape[2])


def lmcache_two_x_nl_buffer_to_paged(memory: np.ndarray, kvcaches: list[list[np.ndarray]], slots: np.ndarray, skip_prefix: int = 0) -> None:
    """``[2, NL, T, H]`` -> SGLang MP caches (lmcache_kv_transfer.py:176-226)."""
    for kv in range(2):
        for layer, cache in enumerate(kvcaches[kv]):
            nb, bs = cache.shape[0], cache.shape[1]
            rows_scatter(memory[kv, layer], cache.reshape(nb * bs, -1), slots, skip_prefix)


def lmcache_paged_to_kv_buffer_mla(paged: np.ndarray, kv_buffer: np.ndarray, slots: np.ndarray) -> None:
    """``[NL, NB, BS, HS]`` -> ``[NL, T, HS]`` (lmcache_kv_transfer.py:135-151)."""
    nl, nb, bs, hs = paged.shape
    for layer in range(nl):
        kv_buffer[layer] = rows_gather(paged[layer].reshape(nb * bs, hs), slots, kv_buffer.shape[1])


def lmcache_kv_buffer_to_paged_mla(kv_buffer: np.ndarray, paged: np.ndarray, slots: np.ndarray) -> None:
    """``[NL, T, HS]`` -> ``[NL, NB, BS, HS]`` (lmcache_kv_transfer.py:118-132)."""
    nl, nb, bs, hs = paged.shape
    for layer in range(nl):
        rows_scatter(kv_buffer[layer], paged[layer].reshape(nb * bs, hs), slots)


def lmcache_mla_paged_to_buffer(kvcaches: list[np.ndarray], memory: np.ndarray, slots: np.ndarray) -> None:
    """List of ``[NB, BS, HS]`` -> ``[1, NL, T, HS]`` (lmcache_kv_transfer.py:488-502)."""
    for layer, cache in enumerate(kvcaches):
        nb, bs, hs = cache.shape
        memory[0, layer] = rows_gather(cache.reshape(nb * bs, hs), slots, memory.shape[2])


def lmcache_mla_buffer_to_paged(memory: np.ndarray, kvcaches: list[np.ndarray], slots: np.ndarray, skip_prefix: int = 0) -> None:
    """``[1, NL, T, HS]`` -> list of ``[NB, BS, HS]`` (lmcache_kv_transfer.py:473-485)."""
    for layer, cache in enumerate(kvcaches):
        nb, bs, hs = cache.shape
        rows_scatter(memory[0, layer], cache.reshape(nb * bs, hs), slots, skip_prefix)


# ---- MLA flat caches (musa_aiter/ops/kv_transfer.py:3786-4118) --------------


def kv_paged_to_mla_linear(kv_cache: np.ndarray, pe_cache: np.ndarray, slots: np.ndarray):
    """``[NB, BS, kv_dim]`` + ``[NB, BS, pe_dim]`` -> ``[T, kv_dim]`` + ``[T, pe_dim]`` (kv_transfer.py:3786-3815)."""
    nb, bs, _ = kv_cache.shape
    return (
        rows_gather(kv_cache.reshape(nb * bs, -1), slots),
        rows_gather(pe_cache.reshape(nb * bs, -1), slots),
    )


def kv_mla_linear_to_paged(kv_lin, pe_lin, kv_cache, pe_cache, slots) -> None:
    """kv_transfer.py:3818-3838 (last writer wins)."""
    nb, bs, _ = kv_cache.shape
    rows_scatter(kv_lin, kv_cache.reshape(nb * bs, -1), slots)
    rows_scatter(pe_lin, pe_cache.reshape(nb * bs, -1), slots)


# ---- MLA FP8 rows with per-group scales ----------------------------------------
# Row = [kv_dim FP8 codes][kv_dim/128 fp32 scales][pe_dim rope elements, 2 B each].
# Group scale = amax over the group's finite |x| (0 when none) / fp8_max in fp32,
# so every stored scale is finite; the element rule is the pinned ``fp8_quantize_to_uint8`` above
# (musa_aiter/ops/kv_transfer.py:2161-2183).  The grouping and byte layout are
# this build's documented choice (the reference only moves such rows as opaque
# bytes, kv_transfer.py:4411-4452, 4588-4616): parity for them is unpinned.

MLA_FP8_GROUP = 128


def mla_fp8_row_bytes(kv_dim: int, pe_dim: int) -> int:
    return kv_dim + (kv_dim // MLA_FP8_GROUP) * 4 + pe_dim * 2


def mla_fp8_group_scales(x_f32: np.ndarray, fp8_format: str) -> np.ndarray:
    """``[..., kv_dim]`` fp32 -> ``[..., kv_dim / 128]`` fp32 scales."""
    fmax = np.float32(448.0 if normalize_fp8_format(fp8_format) == "e4m3" else 57344.0)
    x = np.asarray(x_f32, dtype=np.float32)
    g = x.reshape(x.shape[:-1] + (x.shape[-1] // MLA_FP8_GROUP, MLA_FP8_GROUP))
    a = np.abs(g)
    a = np.where(np.isfinite(a), a, np.float32(0.0))
    amax = np.max(a, axis=-1, initial=np.float32(0.0)).astype(np.float32)
    return (amax / fmax).astype(np.float32)


def mla_fp8_encode_rows(kv: np.ndarray, pe: np.ndarray, in_dtype: str, fp8_format: str) -> np.ndarray:
    """Token rows ``[T, kv_dim]`` + ``[T, pe_dim]`` (in_dtype; bf16 as uint16 bits) -> ``[T, row]`` uint8."""
    x = to_f32(kv, in_dtype)
    t, kvd = x.shape
    scales = mla_fp8_group_scales(x, fp8_format)
    per_elem = np.repeat(scales, MLA_FP8_GROUP, axis=-1)
    codes = fp8_quantize_to_uint8(x, per_elem, fp8_format)
    pe = np.ascontiguousarray(pe)
    pe_bytes = pe.view(np.uint8).reshape(t, pe.shape[-1] * pe.itemsize)
    return np.concatenate([codes, np.ascontiguousarray(scales).view(np.uint8).reshape(t, -1), pe_bytes], axis=1)


def mla_fp8_rows_store(kv: np.ndarray, pe: np.ndarray, cache_rows: np.ndarray, slots: np.ndarray, *,
                       in_dtype: str, fp8_format: str = "e4m3") -> None:
    """``[L, T, kv_dim]`` + ``[L, T, pe_dim]`` -> ``cache_rows[L, NB*BS, row]`` at ``slots`` (last writer wins;
    negative / out-of-range slots skipped)."""
    slots = np.asarray(slots, dtype=np.int64)
    keep = last_writer_mask(slots) & (slots < cache_rows.shape[1])
    t = np.nonzero(keep)[0]
    for layer in range(kv.shape[0]):
        rows = mla_fp8_encode_rows(kv[layer], pe[layer], in_dtype, fp8_format)
        cache_rows[layer, slots[t]] = rows[t]


def mla_fp8_rows_load(cache_rows: np.ndarray, slots: np.ndarray, *, kv_dim: int, pe_dim: int, out_dtype: str,
                      fp8_format: str = "e4m3") -> tuple[np.ndarray, np.ndarray]:
    """``cache_rows[L, NB*BS, row]`` at ``slots`` -> (``[L, T, kv_dim]``, ``[L, T, pe_dim]``) in out_dtype
    (bf16 as uint16 bits); negative / out-of-range slots give zero rows."""
    slots = np.asarray(slots, dtype=np.int64)
    nl, nrows, _ = cache_rows.shape
    ok = (slots >= 0) & (slots < nrows)
    np_t = np.uint16 if out_dtype == "bfloat16" else np.float16
    kv = np.zeros((nl, slots.shape[0], kv_dim), dtype=np_t)
    pe = np.zeros((nl, slots.shape[0], pe_dim), dtype=np_t)
    idx = np.nonzero(ok)[0]
    g = kv_dim // MLA_FP8_GROUP
    for layer in range(nl):
        rows = cache_rows[layer, slots[idx]]
        codes = rows[:, :kv_dim]
        scales = np.ascontiguousarray(rows[:, kv_dim: kv_dim + 4 * g]).view(np.float32)
        per_elem = np.repeat(scales, MLA_FP8_GROUP, axis=-1)
        kv[layer, idx] = fp8_dequantize_from_uint8(codes, per_elem, fp8_format, out_dtype)
        pe[layer, idx] = np.ascontiguousarray(rows[:, kv_dim + 4 * g: kv_dim + 4 * g + 2 * pe_dim]).view(np_t)
    return kv, pe


# ---------------------------------------------------------------------------
# `cache` family: RoPE and the KV-cache write (musa_aiter/ops/cache.py)
# ---------------------------------------------------------------------------


def promote_float(a: str, b: str, *, b_is_0dim: bool = False) -> str:
    """torch's result type of a float tensor op between dtypes a and b (b a 0-dim tensor or not)."""
    if b_is_0dim or a == b:
        return a
    if "float32" in (a, b):
        return "float32"
    return "float32"  # float16 with bfloat16


def round_to(v: np.ndarray, dtype: str) -> np.ndarray:
    """fp32 values rounded to nearest-even in ``dtype`` and back to fp32."""
    v = np.asarray(v, dtype=np.float32)
    if dtype == "float16":
        with np.errstate(over="ignore"):
            return v.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        return bf16_bits_to_f32(f32_to_bf16_bits(v))
    return v


def _op(a, b, dtype, fn):
    with np.errstate(over="ignore", invalid="ignore"):
        return round_to(fn(round_to(a, dtype), round_to(b, dtype)).astype(np.float32), dtype)


def rope_pair(x1, x2, c, s, *, r1: str, r2: str, r3: str):
    """(x1*cos - x2*sin, x1*sin + x2*cos) with torch's per-operation types (cache.py:35-42)."""
    mul = np.multiply
    p11, p22 = _op(x1, c, r1, mul), _op(x2, s, r2, mul)
    p12, p21 = _op(x1, s, r2, mul), _op(x2, c, r1, mul)
    return _op(p11, p22, r3, np.subtract), _op(p12, p21, r3, np.add)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, *, x_dtype: str, cos_dtype: str, sin_dtype: str,
               interleaved: bool = False) -> np.ndarray:
    """``apply_rope`` (musa_aiter/ops/cache.py:9-42) on numpy inputs (bf16 as uint16 bits)."""
    xf = to_f32(x, x_dtype)
    cf = to_f32(cos, cos_dtype)
    sf = to_f32(sin, sin_dtype)
    r1 = promote_float(x_dtype, cos_dtype, b_is_0dim=np.ndim(cos) == 0)
    r2 = promote_float(x_dtype, sin_dtype, b_is_0dim=np.ndim(sin) == 0)
    r3 = promote_float(r1, r2)
    half = xf.shape[-1] // 2
    if interleaved:
        x1, x2 = xf[..., 0::2], xf[..., 1::2]
    else:
        x1, x2 = xf[..., :half], xf[..., half:]
    x1, x2, cf, sf = np.broadcast_arrays(x1, x2, cf, sf)
    o1, o2 = rope_pair(x1, x2, cf, sf, r1=r1, r2=r2, r3=r3)
    if interleaved:
        out = np.stack((o1, o2), axis=-1).reshape(o1.shape[:-1] + (2 * half,))
    else:
        out = np.concatenate((o1, o2), axis=-1)
    return from_f32(out, x_dtype)


def apply_rope_to_key_cache(key_cache: np.ndarray, slots: np.ndarray, positions: np.ndarray, cos: np.ndarray,
                            sin: np.ndarray, *, cache_dtype: str, cos_dtype: str, sin_dtype: str,
                            interleaved: bool = False) -> None:
    """In place on ``key_cache[NB, NH, HD, BS]``, token by token (musa_aiter/ops/cache.py:84-101)."""
    bs = key_cache.shape[-1]
    for t, slot in enumerate(np.asarray(slots, dtype=np.int64).tolist()):
        if slot < 0:
            continue
        b, o = slot // bs, slot % bs
        pos = int(positions[t])
        crow = cos if cos.ndim == 1 else cos[pos]
        srow = sin if sin.ndim == 1 else sin[pos]
        key_cache[b, :, :, o] = apply_rope(key_cache[b, :, :, o], crow, srow, x_dtype=cache_dtype, cos_dtype=cos_dtype,
                                           sin_dtype=sin_dtype, interleaved=interleaved)


def copy_to_kv_cache(k: np.ndarray, v: np.ndarray, key_cache: np.ndarray, value_cache: np.ndarray, slots) -> None:
    """musa_aiter/ops/cache.py:133-144: token loop, negative slots skipped, last writer wins."""
    bs = key_cache.shape[-1]
    for t, slot in enumerate(np.asarray(slots, dtype=np.int64).tolist()):
        if slot < 0:
            continue
        key_cache[slot // bs, :, :, slot % bs] = k[t]
        value_cache[slot // bs, :, :, slot % bs] = v[t]


# ---------------------------------------------------------------------------
# Flash dense layouts (musa_aiter/ops/kv_transfer.py:1527-1795)
# ---------------------------------------------------------------------------


def flash_slots(block_tables: np.ndarray, seq_lens: np.ndarray, block_size: int, dense_len: int) -> np.ndarray:
    """Per-sequence slot building of kv_transfer.py:1779-1791: [B * dense_len], -1 past seq_len."""
    bt = np.asarray(block_tables, dtype=np.int64)
    lens = np.asarray(seq_lens, dtype=np.int64)
    b = bt.shape[0]
    out = np.full((b, dense_len), -1, dtype=np.int64)
    pos = np.arange(dense_len)
    for i in range(b):
        n = int(lens[i])
        blk = bt[i, pos[:n] // block_size]
        out[i, :n] = blk * block_size + pos[:n] % block_size
    return out.reshape(-1)


def kv_load_and_reshape_flash(k_cache, v_cache, block_tables, seq_lens, max_seq_len=None):
    """kv_transfer.py:1527-1622: dense [B, S, NH, HD] with zero padding."""
    nb, nh, hd, bs = k_cache.shape
    lens = np.asarray(seq_lens, dtype=np.int64)
    dense = int(lens.max()) if max_seq_len is None and lens.size else int(max_seq_len or 0)
    slots = flash_slots(block_tables, lens, bs, dense)
    ok, ov = kv_paged_to_linear(k_cache, v_cache, slots)
    b = lens.shape[0]
    return ok.reshape(b, dense, nh, hd), ov.reshape(b, dense, nh, hd)


def kv_reshape_and_cache_back_flash(dense_k, dense_v, k_cache, v_cache, block_tables, seq_lens) -> None:
    """kv_transfer.py:1625-1726: scatter the first seq_len rows of every sequence (last writer wins)."""
    b, dense, nh, hd = dense_k.shape
    bs = k_cache.shape[3]
    slots = flash_slots(block_tables, seq_lens, bs, dense)
    kv_linear_to_paged(dense_k.reshape(b * dense, nh, hd), dense_v.reshape(b * dense, nh, hd), k_cache, v_cache, slots)


def kv_load_and_dequantize_fp8_flash(k8, v8, block_tables, seq_lens, k_scale, v_scale, *, max_seq_len=None,
                                     out_dtype="bfloat16", fp8_format="e4m3"):
    """kv_transfer.py:1729-1795."""
    nb, nh, hd, bs = k8.shape
    lens = np.asarray(seq_lens, dtype=np.int64)
    dense = int(lens.max()) if max_seq_len is None and lens.size else int(max_seq_len or 0)
    slots = flash_slots(block_tables, lens, bs, dense)
    ok, ov = kv_paged_fp8_to_linear(k8, v8, slots, k_scale, v_scale, out_dtype=out_dtype, fp8_format=fp8_format)
    b = lens.shape[0]
    return ok.reshape(b, dense, nh, hd), ov.reshape(b, dense, nh, hd)


def kv_triton_indexed_to_dense(k_cache, v_cache, indptr, indices, max_seq_len):
    """kv_transfer.py:1291-1366: rows indices[indptr[b] + s] for s < min(len_b, S), zeros elsewhere."""
    indptr = np.asarray(indptr, dtype=np.int64)
    indices = np.asarray(indices, dtype=np.int64)
    b = indptr.shape[0] - 1
    ntok, nh, hd = k_cache.shape
    ok = np.zeros((b, max_seq_len, nh, hd), dtype=k_cache.dtype)
    ov = np.zeros_like(ok)
    for i in range(b):
        n = min(max(int(indptr[i + 1] - indptr[i]), 0), max_seq_len)
        if n <= 0:
            continue
        rows = indices[indptr[i]: indptr[i] + n]
        ok[i, :n] = k_cache[rows]
        ov[i, :n] = v_cache[rows]
    return ok, ov


# ---------------------------------------------------------------------------
# block copies and DSV4 byte rows (kv_transfer.py:1871-2091, 4518-4736)
# ---------------------------------------------------------------------------


def kv_copy_paged_blocks(src_k, src_v, dst_k, dst_v, pairs) -> int:
    """Copy whole blocks pair by pair in order (later pairs overwrite earlier ones); returns the count."""
    pairs = np.asarray(pairs, dtype=np.int64).reshape(-1, 2)
    multi = src_k.ndim == 5
    copied = 0
    for s, d in pairs:
        if s < 0 or d < 0:
            continue
        if multi:
            dst_k[:, d] = src_k[:, s]
            dst_v[:, d] = src_v[:, s]
        else:
            dst_k[d] = src_k[s]
            dst_v[d] = src_v[s]
        copied += 1
    return copied


def kv_copy_paged_rows(src: np.ndarray, dst: np.ndarray, src_idx, dst_idx) -> None:
    """dst.index_copy_(0, dst_idx, src.index_select(0, src_idx)) with in-order overwrite."""
    si = np.asarray(src_idx, dtype=np.int64)
    di = np.asarray(dst_idx, dtype=np.int64)
    keep = last_writer_mask(di)
    dst[di[keep]] = src[si[keep]]


def kv_copy_paged_rows_multi_pool(pools, indices) -> None:
    """kv_transfer.py:4619-4660: every (src, dst) layer pair of every pool copies the rows named
    by the one shared index vector (same index on both sides), in pool and layer order.
    ``pools`` is a list of (src layers, dst layers)."""
    for srcs, dsts in pools:
        for s, d in zip(srcs, dsts):
            kv_copy_paged_rows(s, d, indices, indices)


def hicache_transfer(src_k, dst_k, src_v, dst_v, src_idx, dst_idx, src_layout, dst_layout, start_layer, num_layers):
    """musa_aiter/ops/hicache_transfer.py:254-340: per (page pair, layer) row copies, -1 skips."""
    si = np.asarray(src_idx, dtype=np.int64)
    di = np.asarray(dst_idx, dtype=np.int64)

    def row(t, layout, layer, page):
        return (layer, page) if layout == "layer_first" else (page, layer)

    for s, d in zip(si, di):
        if s < 0 or d < 0:
            continue
        for layer in range(start_layer, start_layer + num_layers):
            dst_k[row(dst_k, dst_layout, layer, d)] = src_k[row(src_k, src_layout, layer, s)]
            if src_v is not None:
                dst_v[row(dst_v, dst_layout, layer, d)] = src_v[row(src_v, src_layout, layer, s)]


def hicache_direct(src_layers, dst_layers, src_idx, dst_idx, page_size: int) -> None:
    """hicache_transfer.py:531-580: per page, ``page_size`` rows from the page's first index."""
    si = np.asarray(src_idx, dtype=np.int64).reshape(-1, page_size)[:, 0]
    di = np.asarray(dst_idx, dtype=np.int64).reshape(-1, page_size)[:, 0]
    for s, d in zip(si, di):
        for src, dst in zip(src_layers, dst_layers):
            dst[d: d + page_size] = src[s: s + page_size]


# ---------------------------------------------------------------------------
# CacheGen codec (kv_transfer.py:1111-1217)
# ---------------------------------------------------------------------------


def kv_cachegen_encode(x_f32: np.ndarray, num_bins: int = 256):
    """Codes, codebook and CDF.  scale = reciprocal(max - min) * (bins - 1) in fp32 (PyTorch's
    ``int / tensor``); codes = clamp(round_half_even((x - min) * scale)); CDF = [0, cumsum(counts) / n]
    accumulated in fp32.  The codebook is torch.linspace on the host (the reference's call)."""
    import torch

    x = np.asarray(x_f32, dtype=np.float32)
    n = x.size
    if n == 0:
        return np.zeros(x.shape, np.uint8), np.zeros(num_bins, np.float32), np.zeros(num_bins + 1, np.float32)
    lo, hi = np.float32(x.min()), np.float32(x.max())
    if lo == hi:
        cdf = np.zeros(num_bins + 1, np.float32)
        cdf[1:] = 1.0
        return np.zeros(x.shape, np.uint8), np.full(num_bins, lo, np.float32), cdf
    with np.errstate(divide="ignore"):
        scale = np.float32(np.float32(1.0) / np.float32(hi - lo)) * np.float32(num_bins - 1)
    q = np.rint(((x - lo).astype(np.float32) * np.float32(scale)).astype(np.float32))
    codes = np.clip(q, 0, num_bins - 1).astype(np.uint8)
    counts = np.bincount(codes.reshape(-1), minlength=num_bins).astype(np.float32)
    cdf = np.zeros(num_bins + 1, np.float32)
    cdf[1:] = np.cumsum(counts, dtype=np.float32) / np.float32(n)
    codebook = torch.linspace(float(lo), float(hi), num_bins, dtype=torch.float32).numpy()
    return codes, codebook, cdf


def kv_cachegen_decode(codes: np.ndarray, codebook: np.ndarray) -> np.ndarray:
    return np.asarray(codebook)[np.asarray(codes).astype(np.int64)]


# ---------------------------------------------------------------------------
# DSV4 strided block transfer (restated from csrc/kvcache/kv_transfer_float.mu:3281-3405;
# the reference has no PyTorch path for it, so this restatement is pinned by reading only)
# ---------------------------------------------------------------------------


def strided_block_transfer(staging: np.ndarray, pages: list[np.ndarray], block_ids, direction: int, idx_start: int,
                           n_valid: int, offset_in_object: int, block_size: int, row_bytes: int, block_stride: int,
                           mode: int, value_bytes: int = 0, scale_bytes: int = 0) -> None:
    """staging: uint8 [NL, staging_tokens, row_bytes]; pages: per-layer uint8 flat page arrays."""
    ids = np.asarray(block_ids, dtype=np.int64)
    for layer, page in enumerate(pages):
        for p in range(n_valid):
            blk = int(ids[idx_start + p])
            if blk < 0:
                continue
            for t in range(block_size):
                st = staging[layer, offset_in_object + p * block_size + t]
                base = blk * block_stride
                if mode == 0:
                    spans = [(base + t * row_bytes, 0, row_bytes)]
                else:
                    spans = [(base + t * value_bytes, 0, value_bytes),
                             (base + block_size * value_bytes + t * scale_bytes, value_bytes, scale_bytes)]
                for poff, soff, nbytes in spans:
                    if direction == 0:
                        page[poff: poff + nbytes] = st[soff: soff + nbytes]
                    else:
                        st[soff: soff + nbytes] = page[poff: poff + nbytes]
