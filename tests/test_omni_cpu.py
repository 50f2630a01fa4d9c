"""Qwen2.5-Omni thinker (text + image + audio) against Transformers (fp32, CPU)."""

from __future__ import annotations

import torch

IMG, AUD, VS, AS = 250, 251, 252, 253


def _tiny(tmp_path):
    from transformers import Qwen2_5OmniThinkerConfig
    from transformers.models.qwen2_5_omni.modeling_qwen2_5_omni import Qwen2_5OmniThinkerForConditionalGeneration

    tc = dict(vocab_size=256, hidden_size=64, intermediate_size=96, num_hidden_layers=2, num_attention_heads=4,
              num_key_value_heads=2, max_position_embeddings=512, rope_theta=10000.0,
              rope_scaling={"type": "default", "mrope_section": [2, 3, 3]})
    vc = dict(depth=3, hidden_size=32, intermediate_size=64, num_heads=2, patch_size=4, spatial_merge_size=2,
              temporal_patch_size=2, out_hidden_size=64, fullatt_block_indexes=[1], window_size=16, in_channels=3)
    ac = dict(num_mel_bins=16, encoder_layers=2, encoder_attention_heads=2, encoder_ffn_dim=64, d_model=32,
              output_dim=64, max_source_positions=100, n_window=5)
    cfg = Qwen2_5OmniThinkerConfig(text_config=tc, vision_config=vc, audio_config=ac, image_token_index=IMG,
                                   audio_token_index=AUD, vision_start_token_id=VS, audio_start_token_id=AS)
    torch.manual_seed(0)
    hf = Qwen2_5OmniThinkerForConditionalGeneration(cfg).eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if ("norm" in n or "ln_" in n) and p.dim() == 1:
                p.add_(0.1 * torch.randn_like(p))
    hf.save_pretrained(str(tmp_path))
    return hf


def test_omni_matches_transformers(tmp_path):
    from representax_b200.models.qwen2_5_omni import Qwen2_5OmniBatch, Qwen2_5OmniCheckpointAdapter

    hf = _tiny(tmp_path)
    cfg_path = tmp_path / "config.json"
    model = Qwen2_5OmniCheckpointAdapter.load(tmp_path)
    g = torch.Generator().manual_seed(5)
    # image grid 1 x 8 x 12 patches -> 4 x 6 merged = 24 tokens, 2 windows wide (window 16 px = 2 merged)
    grid = torch.tensor([[1, 8, 12]])
    n_img = 24
    # audio: 23 mel frames -> chunks 10, 10, 3 -> after conv 5, 5, 2 = 12 -> pooled 6 tokens
    frames = 23
    n_aud = 6
    seq = [5, 6, VS] + [IMG] * n_img + [VS + 0, 7, AS] + [AUD] * n_aud + [254, 8, 9]
    ids = torch.tensor([seq, seq])
    mask = torch.ones_like(ids)
    mask[1, -2:] = 0
    pixels = torch.randn(8 * 12, 3 * 2 * 4 * 4, generator=g)
    pixels = torch.cat([pixels, pixels])
    grid2 = torch.cat([grid, grid])
    feats = torch.randn(2, 16, frames, generator=g)
    fmask = torch.ones(2, frames, dtype=torch.long)
    with torch.no_grad():
        out = hf(input_ids=ids, attention_mask=mask, pixel_values=pixels, image_grid_thw=grid2,
                 input_features=feats, feature_attention_mask=fmask, output_hidden_states=True)
        ref = out.hidden_states[-1]
        batch = Qwen2_5OmniBatch(ids, mask, pixels, grid2, feats.permute(1, 0, 2).reshape(16, -1),
                                 torch.tensor([frames, frames]))
        got = model.hidden_states(batch)
    torch.testing.assert_close(got[mask.bool()], ref[mask.bool()], rtol=5e-4, atol=5e-4)
