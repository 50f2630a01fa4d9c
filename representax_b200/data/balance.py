"""Token-balanced assignment of a global batch's rows to data-parallel ranks.

Every rank of a data-parallel step waits for the slowest one (at the
cross-rank MNR barrier and at the gradient reduce-scatter), and the work of a
rank grows with the number of tokens it encodes, not with its number of rows.
Splitting a global batch of variable-length rows into contiguous slices leaves
ranks with token counts that differ by a few percent; this module deals the
rows out so that every rank gets the same number of rows and nearly the same
number of tokens. The global batch (its rows, positives and negatives) is
unchanged; only which rank encodes which row changes.

The assignment is a serpentine deal over rows sorted by length (longest
first): ranks 0..N-1, then N-1..0, and so on, which keeps row counts equal and
bounds the token spread by about one row's length. It is deterministic, so
every rank computes the same assignment from the same lengths without
communication.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np


def token_balanced_shards(lengths: Sequence[int], world: int) -> list[np.ndarray]:
    """Row indices of each rank (equal counts; ``len(lengths)`` must divide by ``world``)."""

    n = len(lengths)
    if world < 1 or n % world:
        raise ValueError(f"{n} rows cannot be split evenly over {world} ranks")
    order = np.argsort(-np.asarray(lengths), kind="stable")
    lane = np.arange(n) % (2 * world)
    rank_of = np.where(lane < world, lane, 2 * world - 1 - lane)
    shards = [np.sort(order[rank_of == r]) for r in range(world)]
    return shards


def pair_lengths(query_lengths: Sequence[int], document_lengths: Sequence[int]) -> np.ndarray:
    """Tokens a rank encodes for each (query, document) pair."""

    return np.asarray(query_lengths) + np.asarray(document_lengths)


__all__ = ["pair_lengths", "token_balanced_shards"]
