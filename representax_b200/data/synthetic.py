"""Synthetic retrieval batches with the shapes of the benchmark configurations.

Token ids are uniform in ``[low, vocab)``, the first token is ``[CLS]`` and
the last valid token ``[SEP]``; per-row valid lengths are uniform in
``[min_len, max_len]``; padding uses id 0 with mask 0. Generated on the host
with a seeded NumPy generator so every rank and every resume sees the same
stream.
"""

from __future__ import annotations

import numpy as np
import torch

from representax_b200.models.text_batch import TokenBatch
from representax_b200.tasks.retrieval import RetrievalBatch


def token_batch(rng: np.random.Generator, rows: int, seq: int, *, vocab: int, low: int = 1000,
                min_len: int = 16, max_len: int | None = None, cls_id: int = 101, sep_id: int = 102,
                pack: bool = True) -> TokenBatch:
    max_len = seq if max_len is None else max_len
    ids = rng.integers(low, vocab, size=(rows, seq), dtype=np.int64)
    lengths = rng.integers(min_len, max_len + 1, size=rows)
    mask = np.arange(seq)[None, :] < lengths[:, None]
    ids[:, 0] = cls_id
    ids[np.arange(rows), lengths - 1] = sep_id
    ids = np.where(mask, ids, 0)
    batch = TokenBatch(input_ids=torch.from_numpy(ids.astype(np.int32)),
                       attention_mask=torch.from_numpy(mask.astype(np.int32)))
    return batch.pack() if pack else batch


def retrieval_pairs(rng: np.random.Generator, pairs: int, seq: int, *, vocab: int, low: int = 1000,
                    min_len: int = 16, max_len: int | None = None, pack: bool = True) -> RetrievalBatch:
    q = token_batch(rng, pairs, seq, vocab=vocab, low=low, min_len=min_len, max_len=max_len, pack=pack)
    d = token_batch(rng, pairs, seq, vocab=vocab, low=low, min_len=min_len, max_len=max_len, pack=pack)
    return RetrievalBatch(query=q, document=d, positive_mask=torch.eye(pairs, dtype=torch.bool))


__all__ = ["retrieval_pairs", "token_batch"]
