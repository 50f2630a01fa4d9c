"""End-to-end training mechanics on CPU (BERT-small, MNR)."""

import numpy as np
import pytest
import torch

from representax_b200.data.synthetic import retrieval_pairs
from representax_b200.models.bert import BertConfig, BertEncoder
from representax_b200.precision import FP32_POLICY
from representax_b200.tasks.retrieval import MNRTask
from representax_b200.train.execution import Direct, GradCache
from representax_b200.train.optimizer import AdamW
from representax_b200.train.step import TrainStep, init_train_state


def _tiny(**kw):
    cfg = BertConfig(vocab_size=2000, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                     num_attention_heads=4, max_position_embeddings=64, hidden_dropout_probability=0.0,
                     attention_dropout_probability=0.0, **kw)
    return cfg


def _step(execution, seed=0, steps=3, symmetric=False, lr=1e-3):
    model = BertEncoder(_tiny(), seed=seed)
    state = init_train_state(model, device="cpu", precision=FP32_POLICY)
    step = TrainStep(state, MNRTask(scale=20.0, symmetric=symmetric), optimizer=AdamW(learning_rate=lr),
                     precision=FP32_POLICY, execution=execution, max_gradient_norm=1.0)
    rng = np.random.default_rng(0)
    losses = []
    batch = retrieval_pairs(rng, 8, 32, vocab=2000, low=100, min_len=4)
    for i in range(steps):
        m = step(batch, i)
        losses.append(float(m.loss))
    return state, losses


def test_loss_decreases():
    _, losses = _step(Direct(), steps=8, lr=3e-3)
    assert losses[-1] < losses[0]


@pytest.mark.parametrize("symmetric", [False, True])
def test_grad_cache_matches_direct(symmetric):
    s1, l1 = _step(Direct(), symmetric=symmetric)
    s2, l2 = _step(GradCache(query_chunk_size=3), symmetric=symmetric)
    assert np.allclose(l1, l2, rtol=1e-5, atol=1e-6)
    assert torch.allclose(s1.store.master, s2.store.master, rtol=1e-5, atol=1e-6)


def test_nonfinite_step_keeps_state():
    model = BertEncoder(_tiny(), seed=1)
    state = init_train_state(model, device="cpu", precision=FP32_POLICY)
    step = TrainStep(state, MNRTask(), optimizer=AdamW(learning_rate=1e-3), precision=FP32_POLICY)
    rng = np.random.default_rng(0)
    batch = retrieval_pairs(rng, 4, 16, vocab=2000, low=100, min_len=4)
    step(batch, 0)
    before = state.store.master.clone()
    slot = next(s for s in state.store.slots if s.name == "layers.0.qkv_weight")
    with torch.no_grad():
        state.store.master[slot.offset] = float("nan")
    m = step(batch, 1)
    assert not bool(m.finite)
    assert int(m.optimizer_step) == 1
    after = state.store.master.clone()
    after[slot.offset] = before[slot.offset]
    assert torch.equal(after, before)
