"""Train-state and step-result types (src/representax/train/state.py:12-36)."""

from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class StepMetrics:
    """Device-resident step outputs; read them on the host one step later."""

    loss: torch.Tensor
    gradient_norm: torch.Tensor
    finite: torch.Tensor
    learning_rate: float
    optimizer_step: torch.Tensor
    metrics: dict[str, torch.Tensor] = field(default_factory=dict)
    # Copy of the device status word taken right after the step's kernels were
    # queued (CUDA only). Reading it here, one step late like the other
    # scalars, surfaces a bounded device wait that ran out without a per-step
    # synchronisation.
    device_status: torch.Tensor | None = None

    def to_host(self) -> dict[str, float]:
        if self.device_status is not None:
            code = int(self.device_status[0])
            if code != 0:
                from representax_b200.ops._ext import STATUS_MESSAGES, KernelTimeoutError, status

                if self.device_status.is_cuda:
                    status(self.device_status.device).zero_()  # the live word; this copy stays as read
                raise KernelTimeoutError(f"a kernel of this training step reported: "
                                         f"{STATUS_MESSAGES.get(code, f'status {code}')}")
        out = {
            "loss": float(self.loss),
            "gradient_norm": float(self.gradient_norm),
            "finite": bool(self.finite),
            "learning_rate": self.learning_rate,
            "optimizer_step": int(self.optimizer_step),
        }
        out.update({k: float(v) for k, v in self.metrics.items()})
        return out


@dataclass
class TrainState:
    """Model (with its flat store) plus optimizer scalars and the step count."""

    model: torch.nn.Module
    store: object
    scalars: torch.Tensor  # [8] fp32: clip coef, finite, step, norm, skipped
    # flat buffers of an optimizer other than the fused AdamW (e.g. SGD momentum)
    optimizer_state: dict = field(default_factory=dict)

    @property
    def step(self) -> int:
        return int(self.scalars[2].item())


@dataclass
class StepResult:
    state: TrainState
    metrics: StepMetrics


__all__ = ["StepMetrics", "StepResult", "TrainState"]
