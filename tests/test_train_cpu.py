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


class _HalvingOptimizer:
    """A user optimizer reached through a dotted target: master -= lr * g / 2."""

    def __init__(self, learning_rate=0.1):
        self.learning_rate = learning_rate

    def lr(self, step):
        return self.learning_rate

    def init_state(self, master):
        return {"calls": torch.zeros(1)}

    def update(self, master, grad, state, lr, step):
        state["calls"] += 1
        master.add_(grad, alpha=-lr / 2)


def test_optimizers_from_dotted_targets():
    from representax_b200.config import ComponentConfig, OptimizationConfig
    from representax_b200.train.optimizer import SGD, AdamW, Lion, build_optimizer

    def build(target, schedule=None, **params):
        return build_optimizer(OptimizationConfig(optimizer=ComponentConfig(target=target, parameters=params),
                                                  schedule=schedule))

    assert isinstance(build("optax.adamw", learning_rate=1e-3), AdamW)
    assert build("optax.adam").weight_decay == 0.0
    assert isinstance(build("optax.sgd", learning_rate=0.1, momentum=0.9), SGD)
    assert isinstance(build("optax.lion"), Lion)
    custom = build("tests.test_train_cpu._HalvingOptimizer", learning_rate=0.2)
    assert type(custom).__name__ == "_HalvingOptimizer" and custom.learning_rate == 0.2
    sched = build("optax.sgd", ComponentConfig(target="optax.linear_schedule",
                                               parameters={"init_value": 1.0, "end_value": 0.0,
                                                           "transition_steps": 4}))
    assert sched.lr(2) == 0.5
    with pytest.raises(ValueError, match="both"):
        build("optax.sgd", ComponentConfig(target="optax.constant_schedule", parameters={"value": 1.0}),
              learning_rate=0.1)
    with pytest.raises(TypeError, match="init_state"):
        build("collections.OrderedDict")
    with pytest.raises(ImportError):
        build("no_such_module.factory")


@pytest.mark.parametrize("name", ["sgd", "lion", "custom"])
def test_flat_optimizers_update_rules(name):
    from representax_b200.train.optimizer import SGD, Lion

    torch.manual_seed(0)
    master = torch.randn(10, dtype=torch.float64)
    grads = [torch.randn(10, dtype=torch.float64) for _ in range(3)]
    if name == "sgd":
        opt = SGD(learning_rate=0.1, momentum=0.9, nesterov=True, weight_decay=0.01)
    elif name == "lion":
        opt = Lion(learning_rate=0.01, b1=0.9, b2=0.99, weight_decay=0.1)
    else:
        opt = _HalvingOptimizer(0.2)
    state = opt.init_state(master)
    got = master.clone()
    for step, g in enumerate(grads, start=1):
        opt.update(got, g, state, opt.lr(step), step)
    want, m = master.clone(), torch.zeros(10, dtype=torch.float64)
    for g in grads:
        if name == "sgd":
            g = g + 0.01 * want
            m = 0.9 * m + g
            want = want - 0.1 * (g + 0.9 * m)
        elif name == "lion":
            c = torch.sign(0.9 * m + 0.1 * g)
            want = want - 0.01 * (c + 0.1 * want)
            m = 0.99 * m + 0.01 * g
        else:
            want = want - 0.1 * g
    assert torch.allclose(got, want, atol=1e-12)


def test_train_step_with_sgd_checkpoints_its_state(tmp_path):
    from representax_b200.models.bert import BertConfig, BertEncoder
    from representax_b200.precision import FP32_POLICY
    from representax_b200.tasks.retrieval import MNRTask
    from representax_b200.train.checkpoint import load_training_tensors, training_tensors
    from representax_b200.train.optimizer import SGD
    from representax_b200.train.step import TrainStep, init_train_state
    from representax_b200.data.synthetic import retrieval_pairs

    import numpy as np

    cfg = BertConfig(vocab_size=500, hidden_size=32, intermediate_size=64, num_hidden_layers=1,
                     num_attention_heads=4, max_position_embeddings=64, hidden_dropout_probability=0.0,
                     attention_dropout_probability=0.0)
    state = init_train_state(BertEncoder(cfg, seed=0), device="cpu", precision=FP32_POLICY)
    step = TrainStep(state, MNRTask(scale=20.0), optimizer=SGD(learning_rate=0.5, momentum=0.9),
                     precision=FP32_POLICY)
    batch = retrieval_pairs(np.random.default_rng(0), 4, 16, vocab=500, low=10, min_len=4)
    before = state.store.master.clone()
    m = step(batch, 0)
    assert int(m.optimizer_step) == 1 and not torch.equal(before, state.store.master)
    tensors = training_tensors(state)
    assert "optimizer/flat/trace" in tensors
    state.optimizer_state["trace"].zero_()
    load_training_tensors(state, tensors)
    assert torch.equal(state.optimizer_state["trace"], tensors["optimizer/flat/trace"])
