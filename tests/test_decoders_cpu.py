"""Qwen3-family decoders against Hugging Face Transformers (fp32, CPU)."""

from __future__ import annotations

import torch

from representax_b200.models.jina_v5 import JinaV5CheckpointAdapter
from representax_b200.models.text_batch import TokenBatch


def _tiny_qwen3(tmp_path):
    from transformers import Qwen3Config, Qwen3Model

    cfg = Qwen3Config(vocab_size=200, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16, max_position_embeddings=128,
                      rope_theta=10000.0, pad_token_id=0)
    torch.manual_seed(0)
    hf = Qwen3Model(cfg).eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if "norm" in n:
                p.add_(0.1 * torch.randn_like(p))
    state = {"language_model." + k: v for k, v in hf.state_dict().items()}
    from safetensors.torch import save_file

    tmp_path.mkdir(exist_ok=True)
    save_file({k: v.contiguous() for k, v in state.items()}, str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text(cfg.to_json_string())
    return hf


def test_jina_v5_text_matches_qwen3(tmp_path):
    hf = _tiny_qwen3(tmp_path)
    model = JinaV5CheckpointAdapter.load(tmp_path, output_dimension=32)
    ids = torch.randint(1, 200, (3, 11))
    mask = torch.ones_like(ids)
    mask[1, 7:] = 0
    ids[1, 7:] = 0
    with torch.no_grad():
        ref = hf(input_ids=ids, attention_mask=mask).last_hidden_state
        got = model.hidden_states(TokenBatch(attention_mask=mask, input_ids=ids))
    torch.testing.assert_close(got[mask.bool()], ref[mask.bool()], rtol=2e-4, atol=2e-4)
    e = model.encode(TokenBatch(attention_mask=mask, input_ids=ids))
    last = mask.sum(1) - 1
    want = ref[torch.arange(3), last, :32]
    torch.testing.assert_close(e, torch.nn.functional.normalize(want, dim=-1), rtol=2e-4, atol=2e-4)


def _tiny_qwen3_vl(tmp_path):
    from transformers import Qwen3VLConfig, Qwen3VLModel

    tc = dict(vocab_size=256, hidden_size=64, intermediate_size=96, num_hidden_layers=3, num_attention_heads=4,
              num_key_value_heads=2, head_dim=16, max_position_embeddings=256, pad_token_id=0,
              rope_parameters={"rope_type": "default", "rope_theta": 10000.0, "mrope_section": [2, 3, 3],
                               "mrope_interleaved": True})
    vc = dict(depth=3, hidden_size=32, intermediate_size=64, num_heads=2, patch_size=4, spatial_merge_size=2,
              temporal_patch_size=2, out_hidden_size=64, num_position_embeddings=16, deepstack_visual_indexes=[0, 1],
              in_channels=3)
    cfg = Qwen3VLConfig(text_config=tc, vision_config=vc, image_token_id=250, video_token_id=251,
                        vision_start_token_id=252)
    torch.manual_seed(0)
    hf = Qwen3VLModel(cfg).eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if "norm" in n and p.dim() == 1:
                p.add_(0.1 * torch.randn_like(p))
    hf.save_pretrained(str(tmp_path))
    return hf


def test_qwen3_vl_matches_transformers(tmp_path):
    from representax_b200.models.qwen3_vl import Qwen3VLBatch, Qwen3VLCheckpointAdapter, Qwen3VLReranker

    hf = _tiny_qwen3_vl(tmp_path)
    model = Qwen3VLCheckpointAdapter.load(tmp_path)
    g = torch.Generator().manual_seed(3)
    # record 0: text, 4 image tokens (grid 1x4x4 -> 2x2 merged), text ; record 1: 2 images (4x4 and 4x8)
    ids = torch.randint(1, 240, (2, 20), generator=g)
    mask = torch.ones_like(ids)
    ids[0, 3:7] = 250
    ids[1, 1:5] = 250
    ids[1, 8:16] = 250
    mask[0, 15:] = 0
    ids[0, 15:] = 0
    grid = torch.tensor([[1, 4, 4], [1, 4, 4], [1, 4, 8]])
    patches = int((grid[:, 0] * grid[:, 1] * grid[:, 2]).sum())
    pixels = torch.randn(patches, 3 * 2 * 4 * 4, generator=g)
    mm = (ids == 250).long()
    with torch.no_grad():
        ref = hf(input_ids=ids, attention_mask=mask, pixel_values=pixels, image_grid_thw=grid,
                 mm_token_type_ids=mm).last_hidden_state
        got = model.hidden_states(Qwen3VLBatch(ids, mask, pixels, grid))
    torch.testing.assert_close(got[mask.bool()], ref[mask.bool()], rtol=3e-4, atol=3e-4)
    # text only
    with torch.no_grad():
        ref = hf(input_ids=ids.clamp_max(240), attention_mask=mask).last_hidden_state
        got = model.hidden_states(Qwen3VLBatch(ids.clamp_max(240), mask))
    torch.testing.assert_close(got[mask.bool()], ref[mask.bool()], rtol=3e-4, atol=3e-4)
    s = Qwen3VLReranker(model, true_token_id=5, false_token_id=6).score(Qwen3VLBatch(ids, mask, pixels, grid))
    assert s.shape == (2,) and bool(((s > 0) & (s < 1)).all())


def test_family_catalog_and_pinned_loaders(tmp_path):
    from representax_b200.integrations import families as F
    from representax_b200.integrations.pinned import load_modernvbert_text_encoder
    from representax_b200.models.modernvbert import ModernVBERTCheckpointAdapter, ModernVBERTTextEncoder
    from representax_b200.models.modernvbert.config import ModernVBERTTextConfig

    assert F.get_model_type_family("qwen3_vl").name == "qwen3_vl"
    arch = F.get_hugging_face_architecture("bert")
    assert arch.family == "bert" and arch.has_auto_model
    assert F.get_hugging_face_architecture("llama").support is F.ArchitectureSupport.CATALOGUED
    for fam in F.MODEL_FAMILIES.values():
        assert F.resolve_native_loader(fam.model_types[0]) is not None
    text = ModernVBERTTextEncoder(ModernVBERTTextConfig(vocab_size=64, hidden_size=32, intermediate_size=48,
                                                        num_hidden_layers=2, num_attention_heads=2,
                                                        pad_token_id=0))
    ModernVBERTCheckpointAdapter.save(text, tmp_path)
    loaded = load_modernvbert_text_encoder(tmp_path)
    for a, b in zip(text.parameters(), loaded.parameters()):
        torch.testing.assert_close(a, b)


def test_quantized_lora_on_qwen3_vl_trains_only_adapters():
    from representax_b200.models.adapters import QuantizedLoRAWeight, apply_quantized_lora, merge_quantized_lora
    from representax_b200.models.qwen3 import Qwen3TextConfig
    from representax_b200.models.qwen3_vl import Qwen3VLBatch, Qwen3VLConfig, Qwen3VLEncoder, Qwen3VLVisionConfig

    cfg = Qwen3VLConfig(text=Qwen3TextConfig(vocab_size=128, hidden_size=64, intermediate_size=96, num_hidden_layers=2,
                                             num_attention_heads=4, num_key_value_heads=2, head_dimension=16,
                                             mrope_section=(2, 3, 3), pad_token_id=0),
                        vision=Qwen3VLVisionConfig(depth=1, hidden_size=32, intermediate_size=64, num_heads=2,
                                                   patch_size=4, out_hidden_size=64, num_position_embeddings=16,
                                                   deepstack_visual_indexes=()),
                        image_token_id=120)
    model = Qwen3VLEncoder(cfg, seed=0)
    apply_quantized_lora(model, rank=4, alpha=8.0, target_pattern=r"text\.layers\..*(qkv|o_proj|gate_up|down)$")
    adapters = [m for m in model.modules() if isinstance(m, QuantizedLoRAWeight)]
    assert len(adapters) == 8
    ids = torch.randint(1, 100, (2, 9))
    batch = Qwen3VLBatch(ids, torch.ones_like(ids))
    e0 = model.encode(batch)
    e0.sum().backward()
    trained = {n for n, p in model.named_parameters() if p.grad is not None}
    assert trained and all("lora_" in n for n in trained)
    with torch.no_grad():
        for a in adapters:
            a.lora_b.normal_()
    e1 = model.encode(batch)
    merged = merge_quantized_lora(model)
    torch.testing.assert_close(merged.encode(batch), e1, rtol=1e-4, atol=1e-5)


def test_qwen3_vl_batch_rows_slice_images(tmp_path):
    """Row slices carry their own images' patches, so chunked encoding equals whole-batch encoding."""
    from representax_b200.models.qwen3_vl import Qwen3VLBatch, Qwen3VLCheckpointAdapter

    _tiny_qwen3_vl(tmp_path)
    model = Qwen3VLCheckpointAdapter.load(tmp_path)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(1, 240, (3, 20), generator=g)
    mask = torch.ones_like(ids)
    ids[0, 3:7] = 250             # one 4x4 image
    ids[1, 1:5] = 250             # two images: 4x4 and 4x8
    ids[1, 8:16] = 250
    ids[2, 2:10] = 250            # one 4x8 image
    mask[2, 17:] = 0
    grid = torch.tensor([[1, 4, 4], [1, 4, 4], [1, 4, 8], [1, 4, 8]])
    patches = int((grid[:, 0] * grid[:, 1] * grid[:, 2]).sum())
    pixels = torch.randn(patches, 3 * 2 * 4 * 4, generator=g)
    full = Qwen3VLBatch(ids, mask, pixels, grid).prepare(model.config)
    assert full.images_per_row.tolist() == [1, 2, 1]
    part = full.rows(1, 3)
    assert part.image_grid_thw.tolist() == [[1, 4, 4], [1, 4, 8], [1, 4, 8]]
    assert part.pixel_values.shape[0] == 16 + 32 + 32
    torch.testing.assert_close(part.pixel_values, pixels[16:])
    with torch.no_grad():
        whole = model.encode(full)
        chunks = torch.cat([model.encode(full.rows(0, 1)), model.encode(full.rows(1, 3))])
    torch.testing.assert_close(chunks, whole, rtol=1e-5, atol=1e-5)
