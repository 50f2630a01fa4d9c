"""Explicit numerical-precision boundaries.

Parity: ``PrecisionPolicy``, ``resolve_precision_policy``,
``precision_context`` and the compute / accumulation boundaries of
src/representax/precision.py:19-124. The B200 policy differs in mechanism, not
meaning: fp32 master parameters live in one flat buffer with a bf16 compute
copy refreshed by the fused optimizer kernel (instead of a cast per step), and
a ``float8_e4m3fn`` matrix policy routes packed-row linear layers to
tcgen05 FP8 GEMMs with the reference's per-tensor dynamic scaling (E4M3
forward, E5M2 gradients, fp32 accumulation; ``ops.fp8``), or with
``fp8_scaling="block"`` to the MXFP8 GEMMs of ``ops.mxfp8`` (one UE8M0 scale
per 32-value block, applied by the tensor core).
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import contextmanager
from contextvars import ContextVar
from dataclasses import dataclass
from typing import Any

import torch


@dataclass(frozen=True)
class PrecisionPolicy:
    """Resolved dtypes for stored state, forward compute and objectives."""

    parameter_dtype: torch.dtype = torch.float32
    compute_dtype: torch.dtype = torch.float32
    activation_dtype: torch.dtype = torch.float32
    matrix_dtype: torch.dtype = torch.float32
    accumulation_dtype: torch.dtype = torch.float32
    loss_dtype: torch.dtype = torch.float32
    fp8_block_scaled: bool = False  # float8 matrices: MXFP8 (per-32 block) instead of per-tensor scales

    @property
    def communication_dtype(self) -> torch.dtype:
        """Dtype of parameters gathered across ranks (the compute view)."""

        return self.compute_dtype

    @property
    def mixed(self) -> bool:
        return self.compute_dtype != self.parameter_dtype


FP32_POLICY = PrecisionPolicy()
BF16_MIXED_POLICY = PrecisionPolicy(
    compute_dtype=torch.bfloat16, activation_dtype=torch.bfloat16, matrix_dtype=torch.bfloat16
)

_DTYPES = {
    "float32": torch.float32,
    "bfloat16": torch.bfloat16,
    "float8_e4m3fn": torch.float8_e4m3fn,
}

_ACTIVE: ContextVar[PrecisionPolicy | None] = ContextVar("representax_b200_precision", default=None)


def resolve_precision_policy(config: Any) -> PrecisionPolicy:
    """Resolve a validated ``PrecisionConfig`` into torch dtypes."""

    return PrecisionPolicy(
        parameter_dtype=_DTYPES[config.parameter_dtype],
        compute_dtype=_DTYPES[config.compute_dtype],
        activation_dtype=_DTYPES[config.activation_dtype],
        matrix_dtype=_DTYPES[config.resolved_matrix_dtype],
        accumulation_dtype=_DTYPES[config.accumulation_dtype],
        loss_dtype=_DTYPES[config.loss_dtype],
        fp8_block_scaled=getattr(config, "fp8_scaling", "tensor") == "block",
    )


@contextmanager
def precision_context(policy: PrecisionPolicy) -> Iterator[None]:
    """Make one policy visible at model / objective call boundaries."""

    token = _ACTIVE.set(policy)
    try:
        yield
    finally:
        _ACTIVE.reset(token)


def active_policy() -> PrecisionPolicy:
    policy = _ACTIVE.get()
    return FP32_POLICY if policy is None else policy


def active_compute_dtype(fallback: torch.dtype) -> torch.dtype:
    policy = _ACTIVE.get()
    return fallback if policy is None else policy.compute_dtype


def objective_output(value: torch.Tensor) -> torch.Tensor:
    """Cast a representation back to the accumulation dtype."""

    return value.to(active_policy().accumulation_dtype)


def loss_value(value: torch.Tensor) -> torch.Tensor:
    return value.to(active_policy().loss_dtype)


FP8_MIXED_POLICY = PrecisionPolicy(
    compute_dtype=torch.bfloat16, activation_dtype=torch.bfloat16, matrix_dtype=torch.float8_e4m3fn
)
MXFP8_MIXED_POLICY = PrecisionPolicy(
    compute_dtype=torch.bfloat16, activation_dtype=torch.bfloat16, matrix_dtype=torch.float8_e4m3fn,
    fp8_block_scaled=True,
)

__all__ = [
    "BF16_MIXED_POLICY",
    "FP8_MIXED_POLICY",
    "MXFP8_MIXED_POLICY",
    "FP32_POLICY",
    "PrecisionPolicy",
    "active_compute_dtype",
    "active_policy",
    "loss_value",
    "objective_output",
    "precision_context",
    "resolve_precision_policy",
]
