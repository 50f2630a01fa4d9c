"""Host inference surface: processors, sentence modules, the ST loader, embed().

The Sentence-Transformers artifact is written here from a random tiny BERT;
the oracle is Hugging Face ``transformers.BertModel`` on the same weights
(fp32, CPU) followed by a plain re-statement of the pooling / Dense /
Normalize chain.
"""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from representax_b200 import Route, TextEmbeddingModel, embed
from representax_b200.data.artifact import Artifact, read_artifact
from representax_b200.models import (
    BertCheckpointAdapter,
    BertConfig,
    BertEncoder,
    SentencePooling,
    make_image_processor,
    select_static_shape_bucket,
)

WORDS = ["hello", "world", "query", "passage", "the", "a", "cat", "dog", "sat", "on", "mat", "search", ":"]


def test_shape_buckets():
    assert select_static_shape_bucket((3,), [(8,), (4,), (16,)]) == (4,)
    assert select_static_shape_bucket((2, 3), [(4, 4), (8, 8)]) == (4, 4)
    with pytest.raises(ValueError, match="incomparable"):
        select_static_shape_bucket((2, 2), [(4, 8), (8, 4)])
    with pytest.raises(ValueError, match="exceeds"):
        select_static_shape_bucket((9,), [(8,)])


def test_media_processor_is_deterministic_per_seed():
    def probe(artifact, *, route):
        return artifact.metadata["hw"]

    def prepare(artifact, *, bucket, route, rng):
        noise = rng.standard_normal(bucket).astype(np.float32)
        return {"pixels": noise}

    proc = make_image_processor(admitted_shapes=[(4, 4), (8, 8)], probe=probe, prepare=prepare,
                                batch_builder=lambda pixels: pixels, configuration={"mean": 0.5})
    arts = [Artifact.inline("image", b"x", metadata={"hw": (3, 4)}), Artifact.inline("image", b"y", metadata={"hw": (2, 2)})]
    a = proc(arts, seed=7)
    b = proc(arts, seed=7)
    assert a.shape == (2, 4, 4)
    np.testing.assert_array_equal(a, b)
    assert proc.data_contract()["schema_version"] == "representax-media-processor-v1"


def test_artifact_reads_range_member_and_checksum(tmp_path):
    import hashlib
    import zipfile

    f = tmp_path / "blob.bin"
    f.write_bytes(b"0123456789")
    art = Artifact.ref("text", uri=str(f), byte_range=(2, 5),
                       checksum="sha256:" + hashlib.sha256(b"234").hexdigest())
    assert read_artifact(art) == b"234"
    z = tmp_path / "a.zip"
    with zipfile.ZipFile(z, "w") as handle:
        handle.writestr("inner.txt", b"abcdef")
    assert read_artifact(Artifact.ref("text", uri=str(z), archive_member="inner.txt", byte_range=(1, 3))) == b"bc"
    bad = Artifact.ref("text", uri=str(f), checksum="sha256:" + "0" * 64)
    with pytest.raises(ValueError, match="checksum"):
        read_artifact(bad)


@pytest.mark.parametrize("modes", [("mean",), ("cls", "max"), ("mean_sqrt_len_tokens",), ("weightedmean",),
                                   ("lasttoken",)])
def test_sentence_pooling_modes(modes):
    g = torch.Generator().manual_seed(0)
    h = torch.randn(3, 5, 4, generator=g)
    mask = torch.tensor([[1, 1, 1, 0, 0], [1, 1, 1, 1, 1], [0, 1, 1, 0, 0]])
    out = SentencePooling(4, modes)(h, mask)
    parts = []
    m = mask[..., None].float()
    for mode in modes:
        if mode == "cls":
            parts.append(torch.stack([h[i, int(mask[i].nonzero()[0])] for i in range(3)]))
        elif mode == "max":
            parts.append(h.masked_fill(m == 0, -1e30).amax(1))
        elif mode == "mean":
            parts.append((h * m).sum(1) / m.sum(1))
        elif mode == "mean_sqrt_len_tokens":
            parts.append((h * m).sum(1) / m.sum(1).sqrt())
        elif mode == "weightedmean":
            w = m * torch.arange(1, 6).float()[None, :, None]
            parts.append((h * w).sum(1) / w.sum(1))
        else:
            parts.append(torch.stack([h[i, int(mask[i].nonzero()[-1])] for i in range(3)]))
    torch.testing.assert_close(out, torch.cat(parts, -1))


def _write_st_artifact(root, *, prompts=None, include_prompt=True):
    from transformers import BertTokenizerFast

    vocab = ["[PAD]", "[UNK]", "[CLS]", "[SEP]", "[MASK]"] + WORDS
    (root / "vocab.txt").write_text("\n".join(vocab) + "\n")
    tok = BertTokenizerFast(vocab_file=str(root / "vocab.txt"), do_lower_case=True)
    tok.save_pretrained(str(root))
    cfg = BertConfig(vocab_size=len(vocab), hidden_size=32, num_hidden_layers=2, num_attention_heads=2,
                     intermediate_size=64, max_position_embeddings=64)
    model = BertEncoder(cfg, seed=3)
    BertCheckpointAdapter.save(model, root)
    (root / "modules.json").write_text(json.dumps([
        {"idx": 0, "name": "0", "path": "", "type": "sentence_transformers.models.Transformer"},
        {"idx": 1, "name": "1", "path": "1_Pooling", "type": "sentence_transformers.models.Pooling"},
        {"idx": 2, "name": "2", "path": "2_Dense", "type": "sentence_transformers.models.Dense"},
        {"idx": 3, "name": "3", "path": "3_Normalize", "type": "sentence_transformers.models.Normalize"},
    ]))
    (root / "sentence_bert_config.json").write_text(json.dumps({"max_seq_length": 16, "do_lower_case": True}))
    (root / "config_sentence_transformers.json").write_text(json.dumps(
        {"prompts": prompts or {}, "similarity_fn_name": "cosine"}))
    (root / "1_Pooling").mkdir()
    (root / "1_Pooling" / "config.json").write_text(json.dumps(
        {"word_embedding_dimension": 32, "pooling_mode_mean_tokens": True, "include_prompt": include_prompt}))
    (root / "2_Dense").mkdir()
    (root / "2_Dense" / "config.json").write_text(json.dumps(
        {"in_features": 32, "out_features": 16, "bias": True,
         "activation_function": "torch.nn.modules.activation.Tanh"}))
    g = torch.Generator().manual_seed(5)
    dense = {"linear.weight": torch.randn(16, 32, generator=g) * 0.1, "linear.bias": torch.randn(16, generator=g) * 0.1}
    from safetensors.torch import save_file

    save_file(dense, str(root / "2_Dense" / "model.safetensors"))
    (root / "3_Normalize").mkdir()
    return tok, dense


def _oracle(root, tok, dense, texts, prefix=""):
    from transformers import BertModel

    hf = BertModel.from_pretrained(str(root), local_files_only=True).eval()
    enc = tok([prefix + t for t in texts], padding=True, truncation=True, max_length=16, return_tensors="pt")
    with torch.no_grad():
        h = hf(**enc).last_hidden_state
    m = enc["attention_mask"][..., None].float()
    pooled = (h * m).sum(1) / m.sum(1)
    out = torch.tanh(pooled @ dense["linear.weight"].T + dense["linear.bias"])
    return torch.nn.functional.normalize(out, dim=-1).numpy()


def test_sentence_transformer_loader_matches_transformers(tmp_path):
    from representax_b200.integrations.sentence_transformers import (
        SentenceTransformerGraphKind,
        load_sentence_transformer,
        load_sentence_transformer_graph,
    )

    tok, dense = _write_st_artifact(tmp_path)
    assert load_sentence_transformer_graph(tmp_path).kind is SentenceTransformerGraphKind.DENSE_EMBEDDING
    model = load_sentence_transformer(tmp_path)
    assert isinstance(model, TextEmbeddingModel)
    texts = ["hello world", "the cat sat on the mat", "dog"]
    got = embed(model, texts, batch_size=2)  # exercises the padded last chunk
    assert got.shape == (3, 16)
    np.testing.assert_allclose(got, _oracle(tmp_path, tok, dense, texts), rtol=1e-4, atol=1e-5)
    sim = model.similarity(got, got)
    np.testing.assert_allclose(np.diag(sim), 1.0, rtol=1e-5)


def test_route_prompts_and_prompt_exclusion(tmp_path):
    from representax_b200.integrations.sentence_transformers import load_sentence_transformer

    tok, dense = _write_st_artifact(tmp_path, prompts={"query": "query : ", "document": "passage : "})
    model = load_sentence_transformer(tmp_path)
    got = model.embed(["cat"], route=Route.QUERY)
    np.testing.assert_allclose(got, _oracle(tmp_path, tok, dense, ["cat"], prefix="query : "), rtol=1e-4, atol=1e-5)
    batch = model.preprocess(["cat"], route=Route.DOCUMENT)
    assert batch.input_ids[0, 1].item() == tok.convert_tokens_to_ids("passage")


def test_prompt_excluded_from_pooling(tmp_path):
    from representax_b200.integrations.sentence_transformers import load_sentence_transformer
    from representax_b200.models import SentenceBatch

    _write_st_artifact(tmp_path, prompts={"query": "query : "}, include_prompt=False)
    model = load_sentence_transformer(tmp_path)
    batch = model.preprocess(["cat dog"], route=Route.QUERY)
    assert isinstance(batch, SentenceBatch)
    # [CLS] query : cat dog [SEP] -> the first 3 tokens are prompt (CLS + 2)
    assert batch.pooling_mask[0].tolist()[:6] == [0, 0, 0, 1, 1, 1]
    assert model.embed(["cat dog"], route=Route.QUERY).shape == (1, 16)


def test_public_api_surface():
    import representax_b200 as rx

    for name in rx.__all__:
        assert hasattr(rx, name), name
