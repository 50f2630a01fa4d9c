"""CLIP / BGE-VL against Transformers ``CLIPModel`` (fp32, CPU)."""

from __future__ import annotations

import torch

from representax_b200.models.clip import CLIPBatch, CLIPCheckpointAdapter


def test_clip_features_match_transformers(tmp_path):
    from transformers import CLIPConfig, CLIPModel

    cfg = CLIPConfig(text_config=dict(vocab_size=100, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                      num_attention_heads=2, max_position_embeddings=20, eos_token_id=2),
                     vision_config=dict(hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                        num_attention_heads=2, image_size=32, patch_size=8),
                     projection_dim=32)
    torch.manual_seed(0)
    hf = CLIPModel(cfg).eval()
    hf.save_pretrained(str(tmp_path))
    model = CLIPCheckpointAdapter.load(tmp_path)
    ids = torch.randint(3, 90, (3, 12))
    mask = torch.ones_like(ids)
    ids[:, 8] = 99           # legacy EOS = arg-max id
    mask[:, 9:] = 0
    ids[:, 9:] = 0
    pixels = torch.randn(3, 3, 32, 32)
    with torch.no_grad():
        t_ref = hf.get_text_features(input_ids=ids, attention_mask=mask)
        i_ref = hf.get_image_features(pixel_values=pixels)
        t_ref = getattr(t_ref, "pooler_output", t_ref)
        i_ref = getattr(i_ref, "pooler_output", i_ref)
        t = model.text_features(ids, mask)
        i = model.image_features(pixels)
    torch.testing.assert_close(t, t_ref, rtol=2e-4, atol=2e-4)
    torch.testing.assert_close(i, i_ref, rtol=2e-4, atol=2e-4)
    both = model.encode(CLIPBatch(ids, mask, torch.tensor([True, False, True]), pixels,
                                  torch.tensor([True, True, False])))
    want = torch.stack([t_ref[0] + i_ref[0], i_ref[1], t_ref[2]])
    torch.testing.assert_close(both, torch.nn.functional.normalize(want, dim=-1), rtol=2e-4, atol=2e-4)
