"""Backend selection for a transfer plan (reference contract: musa_aiter/ops/kv_backend.py:9-84).

The selection rule is the reference's, as a pure function of the plan and the
stated capabilities.  ``native_capabilities()`` states this build's: the
sm_100a kernels are the specialized native backend; there is no reference
(CPU) backend to fall back to.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import Enum

from .kv_transfer_plan import KVTransferPlan, validate_transfer_plan


class KVBackend(str, Enum):
    SPECIALIZED_NATIVE = "specialized_native"
    FUSED_NATIVE = "fused_native"
    DIRECT_BATCH = "direct_batch"
    REFERENCE = "reference"
    REJECTED = "rejected"


@dataclass(frozen=True)
class KVBackendCapabilities:
    specialized_native: bool = False
    fused_native: bool = False
    direct_batch: bool = False
    reference: bool = True


@dataclass(frozen=True)
class KVBackendDecision:
    backend: KVBackend
    accepted: bool
    reason: str
    requires_sync: bool


def native_capabilities() -> KVBackendCapabilities:
    """Capabilities of this build: specialized + fused sm_100a kernels, no reference path."""
    from .. import _native

    ok = _native.is_available()
    return KVBackendCapabilities(specialized_native=ok, fused_native=ok, direct_batch=ok, reference=False)


def select_kv_backend(plan: KVTransferPlan, *, capabilities: KVBackendCapabilities | None = None,
                      require_native: bool = False) -> KVBackendDecision:
    validate_transfer_plan(plan)
    caps = capabilities or KVBackendCapabilities()
    if caps.specialized_native:
        return KVBackendDecision(KVBackend.SPECIALIZED_NATIVE, True, "exact specialized native capability is available", False)
    if caps.fused_native:
        return KVBackendDecision(KVBackend.FUSED_NATIVE, True, "layout transform fused native capability is available", False)
    if plan.direct_eligible and caps.direct_batch:
        return KVBackendDecision(KVBackend.DIRECT_BATCH, True, "affine contiguous transfer is eligible for direct batch copy", False)
    why = plan.direct_reject_reason or "no native backend capability is available"
    if require_native:
        return KVBackendDecision(KVBackend.REJECTED, False, f"native backend required; {why}", False)
    if caps.reference:
        return KVBackendDecision(KVBackend.REFERENCE, True, f"reference fallback: {why}", False)
    return KVBackendDecision(KVBackend.REJECTED, False, f"no acceptable backend: {why}", False)
