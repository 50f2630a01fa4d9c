"""ModernVBERT numerics against Hugging Face Transformers (fp32, CPU).

A tiny random Transformers ``ModernVBertModel`` is saved as safetensors and
loaded through our checkpoint adapter; hidden states of text-only and
text+image inputs must match the Transformers forward.
"""

from __future__ import annotations

import pytest
import torch

from representax_b200.models.modernvbert import (
    ModernVBERTBatch,
    ModernVBERTCheckpointAdapter,
    ModernVBERTEncoder,
)
from representax_b200.models.text_batch import TokenBatch

IMAGE_TOKEN = 100


def _hf_model(tmp_path):
    from transformers import ModernVBertConfig, ModernVBertModel

    tc = dict(vocab_size=128, hidden_size=64, intermediate_size=96, num_hidden_layers=4, num_attention_heads=2,
              local_attention=4, max_position_embeddings=64, global_attn_every_n_layers=3, pad_token_id=0,
              bos_token_id=1, eos_token_id=2, cls_token_id=1, sep_token_id=2)
    vc = dict(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=2, image_size=32,
              patch_size=8, num_channels=3)
    cfg = ModernVBertConfig(text_config=tc, vision_config=vc, image_token_id=IMAGE_TOKEN, pixel_shuffle_factor=2)
    torch.manual_seed(0)
    hf = ModernVBertModel(cfg).eval()
    with torch.no_grad():  # non-trivial norm weights
        for name, p in hf.named_parameters():
            if "norm" in name and p.dim() == 1:
                p.add_(torch.randn_like(p) * 0.1)
    hf.save_pretrained(str(tmp_path))
    return hf


def test_text_and_image_hidden_states_match_transformers(tmp_path):
    hf = _hf_model(tmp_path)
    model = ModernVBERTCheckpointAdapter.load(tmp_path)
    assert isinstance(model, ModernVBERTEncoder)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(3, 99, (2, 12), generator=g)
    mask = torch.ones_like(ids)
    mask[1, 9:] = 0
    ids[1, 9:] = 0
    # text only
    with torch.no_grad():
        ref = hf(input_ids=ids, attention_mask=mask).last_hidden_state
        got = model.hidden_states(TokenBatch(attention_mask=mask, input_ids=ids))
    torch.testing.assert_close(got[mask.bool()], ref[mask.bool()], rtol=2e-4, atol=2e-4)
    # with one image per record: 4 patches / shuffle 2 -> 4 image tokens
    n_img_tok = model.config.image_sequence_length
    ids_img = ids.clone()
    ids_img[:, 2:2 + n_img_tok] = IMAGE_TOKEN
    pixels = torch.randn(2, 1, 3, 32, 32, generator=g)
    with torch.no_grad():
        ref = hf(input_ids=ids_img, attention_mask=mask, pixel_values=pixels).last_hidden_state
        got = model.hidden_states(ModernVBERTBatch(mask, ids_img, pixels))
    torch.testing.assert_close(got[mask.bool()], ref[mask.bool()], rtol=2e-4, atol=2e-4)


def test_roundtrip_and_encode(tmp_path):
    _hf_model(tmp_path)
    model = ModernVBERTCheckpointAdapter.load(tmp_path)
    out = tmp_path / "resaved"
    ModernVBERTCheckpointAdapter.save(model, out)
    again = ModernVBERTCheckpointAdapter.load(out)
    for (n, a), (_, b) in zip(model.state_dict().items(), again.state_dict().items()):
        torch.testing.assert_close(a, b, msg=n)
    ids = torch.randint(3, 99, (3, 10))
    mask = torch.ones_like(ids)
    e = model.encode(TokenBatch(attention_mask=mask, input_ids=ids))
    assert e.shape == (3, 64)
    torch.testing.assert_close(e.norm(dim=-1), torch.ones(3))


def test_grad_flows_to_all_towers(tmp_path):
    _hf_model(tmp_path)
    model = ModernVBERTCheckpointAdapter.load(tmp_path)
    ids = torch.randint(3, 99, (2, 10))
    ids[:, 1:5] = IMAGE_TOKEN
    mask = torch.ones_like(ids)
    pixels = torch.randn(2, 1, 3, 32, 32)
    model.encode(ModernVBERTBatch(mask, ids, pixels)).sum().backward()
    assert model.vision.layers[0].qkv_w.grad is not None
    assert model.connector.grad is not None
    assert model.text.layers[1].Wqkv.grad is not None
