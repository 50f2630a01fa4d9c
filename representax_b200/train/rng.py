"""Counter-based random streams for exact stochastic replay.

Every stochastic op draws from a generator keyed on (seed, iteration, role,
chunk), so the GradCache replay of a chunk sees exactly the dropout masks of
its no-grad pass, and a resumed run sees those of the original run
(the role of ``jax.random.fold_in(base_key, iteration)`` in
src/representax/train/loop.py and the per-chunk keys of
src/representax/train/grad_cache.py:60-107).
"""

from __future__ import annotations

import hashlib

import torch


def stream_seed(*parts: object) -> int:
    digest = hashlib.blake2b("/".join(str(p) for p in parts).encode(), digest_size=8).digest()
    return int.from_bytes(digest, "little") & ((1 << 63) - 1)


def generator(device: torch.device | str, *parts: object) -> torch.Generator:
    device = torch.device(device)
    gen = torch.Generator(device=device if device.type == "cuda" else "cpu")
    gen.manual_seed(stream_seed(*parts))
    return gen


class StreamFactory:
    """Derives per-(role, chunk) generators from one step seed."""

    def __init__(self, device, *parts: object, enabled: bool = True) -> None:
        self.device = device
        self.parts = parts
        self.enabled = enabled

    def __call__(self, *more: object):
        if not self.enabled:
            return None
        return generator(self.device, *self.parts, *more)


__all__ = ["StreamFactory", "generator", "stream_seed"]
