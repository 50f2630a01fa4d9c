"""The training step: loss execution, global norm, clipping, finite gate, AdamW.

Parity: ``init_train_state`` / ``build_train_step`` of
src/representax/train/step.py:36-488: the gradient of the (global) loss is
accumulated in fp32, its global L2 norm computed, clipped by
``min(1, max_norm / (norm + 1e-6))``, the update applied only when the loss,
metrics and gradients are all finite (a skipped update does not advance the
optimizer step), with exact microbatch accumulation for direct execution.

On CUDA the norm, gate and update are three kernels over the flat store with
no host synchronisation; the per-step scalars stay on the device.
"""

from __future__ import annotations

from typing import Any

import torch

from representax_b200.parallel.dist import LOCAL, DistContext, all_reduce_sum_
from representax_b200.precision import PrecisionPolicy, precision_context
from representax_b200.tasks._batch import leading_rows, slice_rows

from .execution import Direct
from .flat import FlatParameterStore
from .optimizer import AdamW, is_flat_optimizer
from .rng import StreamFactory
from .state import StepMetrics, TrainState


def init_train_state(model: torch.nn.Module, *, device, precision: PrecisionPolicy, dist: DistContext = LOCAL,
                     sharded_optimizer: bool = False, fsdp: bool = False) -> TrainState:
    """``sharded_optimizer`` (CUDA, world > 1): AdamW moments sharded over the
    ranks, gradients reduce-scattered and parameters all-gathered by peer
    memory kernels fused with the update (see ``TrainStep``).

    ``fsdp`` (CUDA, world > 1, bf16 compute): fp32 master weights, moments and
    the bf16 owner copy are sharded too; each rank gathers the weights at their
    first use in a step, the forward GEMMs with the gather fused into the
    kernel (``representax_b200.parallel.fsdp``)."""

    model.to(torch.float32)
    group = None
    if (sharded_optimizer or fsdp) and dist.enabled and torch.device(device).type == "cuda":
        from representax_b200.parallel.peer import peer_group

        group = peer_group(dist, torch.device(device))
    elif fsdp and dist.enabled:
        raise ValueError("FSDP runs on CUDA devices (peer memory); use DDP on CPU")
    store = FlatParameterStore(model, device=device, compute_dtype=precision.compute_dtype, peer_group=group,
                               fsdp=fsdp and group is not None)
    scalars = torch.zeros(8, dtype=torch.float32, device=store.device)
    return TrainState(model=model, store=store, scalars=scalars)


class TrainStep:
    """Callable ``step(batch, iteration) -> StepMetrics`` over a train state."""

    def __init__(self, state: TrainState, task: Any, *, optimizer: AdamW, precision: PrecisionPolicy,
                 execution: Any = None, max_gradient_norm: float | None = 1.0, seed: int = 0,
                 accumulation_steps: int = 1, dist: DistContext = LOCAL, stochastic: bool = True) -> None:
        self.state = state
        self.task = task
        self.optimizer = optimizer
        self.precision = precision
        self.execution = execution or Direct()
        self.execution.validate(task)
        self.max_gradient_norm = max_gradient_norm
        self.seed = seed
        self.accumulation_steps = accumulation_steps
        self.dist = dist
        self.stochastic = stochastic
        if accumulation_steps > 1 and not isinstance(self.execution, Direct):
            raise ValueError("gradient accumulation composes only with direct execution")
        store: FlatParameterStore = state.store
        self._norm_sq = torch.zeros(1, dtype=torch.float64, device=store.device)
        self._native = store.device.type == "cuda"

    # ------------------------------------------------------------------
    def _loss_and_grads(self, batch, iteration: int):
        store: FlatParameterStore = self.state.store
        store.zero_grad()
        streams = StreamFactory(store.device, self.seed, iteration, enabled=self.stochastic)
        with precision_context(self.precision):
            if self.accumulation_steps == 1:
                out = self.execution.run(self.task, self.state.model, batch, streams=streams, ctx=self.dist)
                loss, metrics = out.loss, dict(out.metrics)
            else:
                loss, metrics = self._accumulate(batch, streams)
        store.collect_autograd_grads()
        if self.dist.enabled and not store.sharded:
            all_reduce_sum_(store.grad, self.dist)
        return loss, metrics

    def _accumulate(self, batch, streams: StreamFactory):
        rows = leading_rows(getattr(batch, "query", batch))
        steps = self.accumulation_steps
        if rows % steps:
            raise ValueError("batch rows must divide evenly into accumulation microbatches")
        size = rows // steps
        weight_fn = getattr(self.task, "accumulation_weight", None)
        total = None
        metrics: dict[str, torch.Tensor] = {}
        for i in range(steps):
            part = slice_rows(batch, i * size, (i + 1) * size)
            w = 1.0 / steps if weight_fn is None else weight_fn(part, batch)
            sub = StreamFactory(streams.device, *streams.parts, "micro", i, enabled=streams.enabled)
            from representax_b200.core import evaluate_loss

            out = evaluate_loss(self.task, self.state.model, part, generator=sub("direct"))
            (out.loss * w).backward()
            total = out.loss.detach() * w if total is None else total + out.loss.detach() * w
            for k, v in out.metrics.items():
                metrics[k] = metrics.get(k, 0) + v.detach() * w
        return total, metrics

    # ------------------------------------------------------------------
    def _apply_update(self, loss: torch.Tensor, metrics: dict[str, torch.Tensor], lr: float) -> None:
        store: FlatParameterStore = self.state.store
        s = self.state.scalars
        opt = self.optimizer
        max_norm = float(self.max_gradient_norm or 0.0)
        gate = loss.detach().reshape(1).to(torch.float32)
        for v in metrics.values():
            gate = gate + 0.0 * v.detach().reshape(-1)[:1].to(gate.device, torch.float32)
        if not isinstance(opt, AdamW):
            self._flat_update(opt, gate, max_norm, lr)
            return
        if self._native and store.sharded:
            self._sharded_update(gate, max_norm, lr)
            return
        if self._native:
            from representax_b200.ops._ext import ext

            C = ext()
            C.grad_norm_sq(store.grad, self._norm_sq)
            C.finalize_clip(self._norm_sq, s, gate.contiguous(), max_norm, 1)
            C.adamw_step(store.master, store.grad, store.exp_avg, store.exp_avg_sq, store.compute, s,
                         lr, opt.b1, opt.b2, opt.eps, opt.weight_decay)
            return
        # Host / CPU path: the same arithmetic in PyTorch.
        with torch.no_grad():
            norm = torch.linalg.vector_norm(store.grad.double()).float()
            finite = bool(torch.isfinite(norm)) and bool(torch.isfinite(gate).all())
            coef = min(1.0, max_norm / (float(norm) + 1e-6)) if (max_norm > 0 and finite) else 1.0
            s[0] = coef
            s[1] = 1.0 if finite else 0.0
            s[3] = norm
            if not finite:
                s[4] += 1
                return
            s[2] += 1
            step = float(s[2])
            g = store.grad * coef
            store.exp_avg.mul_(opt.b1).add_(g, alpha=1 - opt.b1)
            store.exp_avg_sq.mul_(opt.b2).addcmul_(g, g, value=1 - opt.b2)
            mhat = store.exp_avg / (1 - opt.b1 ** step)
            vhat = store.exp_avg_sq / (1 - opt.b2 ** step)
            update = mhat / (vhat.sqrt() + opt.eps) + opt.weight_decay * store.master
            store.master.add_(update, alpha=-lr)
            store.refresh_compute()

    def _flat_update(self, opt, gate: torch.Tensor, max_norm: float, lr: float) -> None:
        """Norm, clip and finite gate as for AdamW, then ``opt.update`` on the flat fp32 buffers.

        Used for optimizers built from other dotted targets (SGD, Lion, user
        classes); it reads the finite flag on the host once per step.
        """

        store: FlatParameterStore = self.state.store
        if store.sharded:
            raise ValueError("the sharded optimizer layout runs the fused AdamW only; use sharded_optimizer=False "
                             f"for {type(opt).__name__}")
        if not is_flat_optimizer(opt):
            raise TypeError(f"{type(opt).__name__} is not a flat optimizer (lr / init_state / update)")
        s = self.state.scalars
        with torch.no_grad():
            norm = torch.linalg.vector_norm(store.grad.double()).float()
            finite = bool(torch.isfinite(norm)) and bool(torch.isfinite(gate).all())
            coef = min(1.0, max_norm / (float(norm) + 1e-6)) if (max_norm > 0 and finite) else 1.0
            s[0], s[1], s[3] = coef, 1.0 if finite else 0.0, norm
            if not finite:
                s[4] += 1
                return
            s[2] += 1
            if not self.state.optimizer_state:
                self.state.optimizer_state.update(opt.init_state(store.master))
            opt.update(store.master, store.grad * coef, self.state.optimizer_state, lr, int(s[2].item()))
            store.refresh_compute()

    def _sharded_update(self, gate: torch.Tensor, max_norm: float, lr: float) -> None:
        """Fused reduce-scatter -> clipped AdamW on the shard -> all-gather.

        1. device barrier: every rank's gradient accumulator is complete;
        2. this rank sums all ranks' gradients for its shard by peer loads (in
           rank order, deterministic) and accumulates the shard's squared norm;
        3. the squared norm is summed over ranks (8-byte NCCL all-reduce) and
           turned into the clip coefficient and finite gate on the device;
        4. AdamW updates the shard and stores the new fp32 master and bf16
           compute values into every rank's buffers (peer stores);
        5. device barrier: the next forward reads complete parameters.
        """

        import torch.distributed as tdist

        from representax_b200.ops._ext import ext

        C = ext()
        store: FlatParameterStore = self.state.store
        s = self.state.scalars
        opt = self.optimizer
        group = store.group
        if not hasattr(self, "_shard_grad"):
            self._shard_grad = torch.empty(store.shard_numel, dtype=torch.float32, device=store.device)
        group.barrier()
        self._norm_sq.zero_()
        C.sharded_grad_reduce(store.peer_pointers("grad"), group.world, store.shard_offset, store.shard_numel,
                              self._shard_grad, self._norm_sq)
        tdist.all_reduce(self._norm_sq)
        C.finalize_clip(self._norm_sq, s, gate.contiguous(), max_norm, 1)
        if store.fsdp is not None:  # update the owned segments only; peers gather them at next use
            C.sharded_adamw(self._shard_grad, store.shard_offset, store.shard_numel, store.master_ptrs,
                            store.owner_ptrs, 1, 0, store.exp_avg, store.exp_avg_sq, s, lr, opt.b1, opt.b2, opt.eps,
                            opt.weight_decay, store.shard_offset)
            store.fsdp.advance()
        else:
            C.sharded_adamw(self._shard_grad, store.shard_offset, store.shard_numel, store.peer_pointers("master"),
                            store.peer_pointers("compute") if store.mixed else None, group.world, group.rank,
                            store.exp_avg, store.exp_avg_sq, s, lr, opt.b1, opt.b2, opt.eps, opt.weight_decay, 0)
        group.barrier()

    def __call__(self, batch: Any, iteration: int) -> StepMetrics:
        lr = self.optimizer.lr(iteration)
        loss, metrics = self._loss_and_grads(batch, iteration)
        self._apply_update(loss, metrics, lr)
        s = self.state.scalars
        device_status = None
        if self._native:
            from representax_b200.ops._ext import status

            device_status = status(self.state.store.device)[:1].clone()
        return StepMetrics(loss=loss.detach(), gradient_norm=s[3].clone(), finite=s[1].clone() > 0,
                           learning_rate=lr, optimizer_step=s[2].clone(),
                           metrics={k: v.detach() for k, v in metrics.items()}, device_status=device_status)


def build_train_step(state: TrainState, task: Any, **kwargs) -> TrainStep:
    return TrainStep(state, task, **kwargs)


__all__ = ["TrainStep", "build_train_step", "init_train_state"]
