"""Dispatch trace: one stderr line per op call when ``MUSA_AITER_TRACE_DISPATCH`` is set.

Same record fields and line format as the reference (musa_aiter/dispatch.py:9-36),
so tooling that greps ``[MUSA_AITER DISPATCH] op=... backend=...`` keeps working.
This build has exactly one backend, ``cuda-sm100a``.
"""

from __future__ import annotations

import os
import sys
from dataclasses import dataclass
from typing import Any

BACKEND = "cuda-sm100a"


@dataclass(frozen=True)
class DispatchRecord:
    op: str
    backend: str
    device: str
    dtype: str
    reason: str


def trace_enabled() -> bool:
    return os.environ.get("MUSA_AITER_TRACE_DISPATCH", "0") in {"1", "true", "TRUE", "yes", "YES"}


def emit(record: DispatchRecord) -> None:
    if not trace_enabled():
        return
    print(
        f"[MUSA_AITER DISPATCH] op={record.op} backend={record.backend} device={record.device} "
        f"dtype={record.dtype} reason={record.reason}",
        file=sys.stderr,
    )


def tensor_device_dtype(x: Any) -> tuple[str, str]:
    return str(getattr(x, "device", "unknown")), str(getattr(x, "dtype", "unknown"))


def emit_native(op: str, x: Any, reason: str) -> None:
    if trace_enabled():
        device, dtype = tensor_device_dtype(x)
        emit(DispatchRecord(op, BACKEND, device, dtype, reason))
