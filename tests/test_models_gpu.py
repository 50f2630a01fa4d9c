"""Native (packed, sm_100a) BERT path against the PyTorch fp32 reference path."""

import numpy as np
import pytest
import torch

from representax_b200.data.synthetic import retrieval_pairs
from representax_b200.models.bert import BertConfig, BertEncoder
from representax_b200.precision import BF16_MIXED_POLICY, FP32_POLICY, precision_context
from representax_b200.tasks._batch import to_device
from representax_b200.tasks.retrieval import MNRTask
from representax_b200.train.execution import Direct, GradCache
from representax_b200.train.optimizer import AdamW
from representax_b200.train.step import TrainStep, init_train_state

pytestmark = pytest.mark.gpu


def _cfg():
    return BertConfig(vocab_size=3000, hidden_size=256, intermediate_size=1024, num_hidden_layers=2,
                      num_attention_heads=4, max_position_embeddings=128, hidden_dropout_probability=0.0,
                      attention_dropout_probability=0.0)


def _cos(a, b):
    a, b = a.flatten().double(), b.flatten().double()
    return float(a @ b / (a.norm() * b.norm() + 1e-30))


def test_native_encode_matches_reference():
    dev = torch.device("cuda", 0)
    model = BertEncoder(_cfg(), seed=3, compute_dtype=torch.bfloat16).to(dev)
    batch = retrieval_pairs(np.random.default_rng(0), 16, 96, vocab=3000, low=200, min_len=3).query
    batch = to_device(batch, dev)
    with precision_context(BF16_MIXED_POLICY):
        native = model.encode(batch)
    with precision_context(FP32_POLICY):
        unpacked = type(batch)(attention_mask=batch.attention_mask, input_ids=batch.input_ids)
        ref = model.encode(unpacked)
    assert native.shape == ref.shape
    err = (native - ref).abs().max().item()
    assert err < 3e-2, err
    assert min(_cos(native[i], ref[i]) for i in range(16)) > 0.999


@pytest.mark.parametrize("execution", [Direct(), GradCache(query_chunk_size=5)])
def test_native_train_step_matches_reference_gradients(execution):
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(1)
    host = retrieval_pairs(rng, 12, 64, vocab=3000, low=200, min_len=3)
    grads = {}
    losses = {}
    for name, policy in (("native", BF16_MIXED_POLICY), ("reference", FP32_POLICY)):
        model = BertEncoder(_cfg(), seed=5, compute_dtype=policy.compute_dtype)
        state = init_train_state(model, device=dev, precision=policy)
        step = TrainStep(state, MNRTask(scale=20.0, symmetric=True), optimizer=AdamW(learning_rate=0.0),
                         precision=policy, execution=execution, max_gradient_norm=0.0)
        batch = to_device(host, dev)
        if name == "reference":
            batch.query.packed = None
            batch.document.packed = None
        m = step(batch, 0)
        losses[name] = float(m.loss)
        grads[name] = {s.name: state.store.grad[s.offset:s.offset + s.numel].clone() for s in state.store.slots}
    assert abs(losses["native"] - losses["reference"]) < 2e-2 * max(1.0, abs(losses["reference"]))
    for key, ref in grads["reference"].items():
        if ref.norm() < 1e-6:
            continue
        assert _cos(grads["native"][key], ref) > 0.99, key


@pytest.mark.gpu
def test_grad_cache_retention_matches_replay():
    """Keeping first-pass chunk graphs gives the same gradient as replaying every chunk."""

    import numpy as np

    from representax_b200.data.synthetic import retrieval_pairs
    from representax_b200.models.bert import BertConfig, BertEncoder
    from representax_b200.precision import BF16_MIXED_POLICY, precision_context
    from representax_b200.tasks._batch import to_device
    from representax_b200.tasks.retrieval import MNRTask
    from representax_b200.train.execution import GradCache
    from representax_b200.train.rng import StreamFactory
    from representax_b200.train.step import init_train_state

    cfg = BertConfig(vocab_size=1000, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                     intermediate_size=512, max_position_embeddings=128)  # dropout 0.1: replays must match
    dev = torch.device("cuda")
    batch = to_device(retrieval_pairs(np.random.default_rng(0), 64, 64, vocab=1000, low=10, min_len=8, max_len=64),
                      dev)
    grads = []
    for retain in (0, 2 ** 40):
        state = init_train_state(BertEncoder(cfg, seed=0, compute_dtype=torch.bfloat16), device=dev,
                                 precision=BF16_MIXED_POLICY)
        ex = GradCache(query_chunk_size=16, retain_bytes=retain)
        state.store.zero_grad()
        with precision_context(BF16_MIXED_POLICY):
            ex.run(MNRTask(scale=20.0), state.model, batch, streams=StreamFactory(dev, 0, 0, enabled=True))
        state.store.collect_autograd_grads()
        grads.append(state.store.grad.clone())
        assert ex.stats["retained_chunks"] == (0 if retain == 0 else ex.stats["chunks"])
    # fp32 atomics (split-K weight gradients, attention dQ) may sum in a different order
    assert (grads[1] - grads[0]).abs().max() <= 1e-4 * grads[0].abs().max()
