"""MPNet against Hugging Face ``MPNetModel``: forward and gradients (CPU, fp32).

A randomly initialised tiny ``MPNetModel`` is saved as safetensors, loaded
through ``MPNetCheckpointAdapter`` (fused q/k/v, relative-position buckets,
padding-aware positions) and compared token by token on a right-padded batch,
then the gradients of a pooled objective with respect to every parameter are
compared name by name. Parity model: tests/models/mpnet/test_transformers_parity.py
of the reference.
"""

import pytest
import torch

transformers = pytest.importorskip("transformers")


def _hf_model(tmp_path):
    config = transformers.MPNetConfig(vocab_size=120, hidden_size=32, num_hidden_layers=2, num_attention_heads=4,
                                      intermediate_size=64, max_position_embeddings=80,
                                      relative_attention_num_buckets=32, hidden_dropout_prob=0.0,
                                      attention_probs_dropout_prob=0.0, pad_token_id=1)
    torch.manual_seed(0)
    model = transformers.MPNetModel(config, add_pooling_layer=True).eval()
    with torch.no_grad():
        for p in model.parameters():  # non-trivial biases and norms
            p.add_(torch.randn_like(p) * 0.02)
    model.save_pretrained(tmp_path, safe_serialization=True)
    return model


def _batch():
    ids = torch.tensor([[0, 15, 27, 33, 41, 2, 1, 1, 1], [0, 9, 88, 13, 52, 61, 74, 19, 2]])
    mask = (ids != 1).to(torch.int32)
    return ids, mask


def test_mpnet_matches_transformers_forward_and_gradients(tmp_path):
    from representax_b200.models.mpnet import MPNetCheckpointAdapter
    from representax_b200.precision import FP32_POLICY, precision_context

    hf = _hf_model(tmp_path)
    ours = MPNetCheckpointAdapter.load(tmp_path, compute_dtype=torch.float32)
    ids, mask = _batch()
    batch = type(ours).make_batch(input_ids=ids, attention_mask=mask)
    with precision_context(FP32_POLICY):
        h_ours = ours.hidden_states(batch)
    h_hf = hf(input_ids=ids, attention_mask=mask).last_hidden_state
    valid = mask.bool()
    torch.testing.assert_close(h_ours[valid], h_hf[valid], rtol=1e-4, atol=1e-5)

    # gradients of a masked mean-pool objective, parameter by parameter (HF names)
    weights = torch.randn(h_hf.shape[-1], generator=torch.Generator().manual_seed(1))

    def objective(hidden):
        pooled = (hidden * valid[..., None]).sum(1) / valid.sum(1, keepdim=True)
        return (pooled @ weights).square().sum()

    objective(h_hf).backward()
    with precision_context(FP32_POLICY):
        objective(ours.hidden_states(batch)).backward()
    hf_grads = {n: p.grad for n, p in hf.named_parameters() if p.grad is not None}
    ours_grads = MPNetCheckpointAdapter.state_dict(_grad_view(ours))
    compared = 0
    for name, g in hf_grads.items():
        if name.startswith("pooler."):
            continue
        torch.testing.assert_close(ours_grads[name], g, rtol=2e-3, atol=2e-6, msg=lambda m: f"{name}: {m}")
        compared += 1
    assert compared >= 20


def _grad_view(model):
    """A copy of the encoder whose parameters hold the original's gradients."""

    import copy

    view = copy.deepcopy(model)
    with torch.no_grad():
        for (name, p), (_, q) in zip(model.named_parameters(), view.named_parameters()):
            q.copy_(p.grad if p.grad is not None else torch.zeros_like(p))
    return view
