"""ModernVBERT: ModernBERT text tower, SigLIP vision tower, pixel-shuffle connector.

All towers run on packed rows (no padding FLOPs) through ``ops.nn``: on
bf16 CUDA tensors every GEMM, norm, RoPE, attention (global or sliding
window) and GeGLU is an sm_100a kernel; elsewhere the same code runs the
PyTorch statement of each op.

Parity:
  * text tower — src/representax/models/modernvbert/model.py:137-687 (fused
    Wqkv, RoPE with separate theta for global and sliding layers, symmetric
    local window of radius local_attention // 2, GeGLU, bias-free
    LayerNorms, identity attention norm in layer 0, final norm, mean pool +
    L2 normalisation);
  * vision tower — src/representax/models/modernvbert/vision.py:23-285
    (patch embedding, learned positions, pre-LN blocks with tanh-GELU MLP,
    post LayerNorm);
  * connector / merge — vision.py:286-307 (pixel shuffle),
    multimodal.py:87-132 (image features scattered into image-token
    positions, valid images first, record-major).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import nn

from representax_b200.core.model import EncoderMetadata, Modality, Route
from representax_b200.models.text_batch import PackedTokens, TokenBatch, pack_tokens, packed_segments
from representax_b200.ops import nn as N
from representax_b200.precision import active_compute_dtype

from .config import ModernVBERTConfig, ModernVBERTTextConfig, SigLIPVisionConfig


def _normal(shape, std, g):
    return nn.Parameter(torch.randn(*shape, generator=g) * std)


def _embed(ids: torch.Tensor, table: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    return torch.nn.functional.embedding(ids.long(), table).to(dtype)


# --------------------------------------------------------------- text tower
class ModernBertLayer(nn.Module):
    def __init__(self, cfg: ModernVBERTTextConfig, index: int, g: torch.Generator) -> None:
        super().__init__()
        h, i, std = cfg.hidden_size, cfg.intermediate_size, cfg.initializer_range
        self.index = index
        self.layer_type = cfg.layer_type(index)
        self.attn_norm = nn.Parameter(torch.ones(h)) if index > 0 else None
        self.Wqkv = _normal((3 * h, h), std, g)
        self.Wo = _normal((h, h), std, g)
        self.mlp_norm = nn.Parameter(torch.ones(h))
        self.Wi = _normal((2 * i, h), std, g)
        self.mlp_Wo = _normal((h, i), std, g)

    def forward(self, h, seg, pos, inv_freq, cfg: ModernVBERTTextConfig):
        x = h if self.attn_norm is None else N.layer_norm(h, self.attn_norm, None, cfg.norm_epsilon)
        qkv = N.linear(x, self.Wqkv)
        window = cfg.local_attention // 2 if self.layer_type == "sliding_attention" else -1
        a = N.qkv_attention(qkv, seg, heads=cfg.num_attention_heads, pos=pos, inv_freq=inv_freq, window=window)
        h = N.linear(a, self.Wo, residual=h)
        x = N.layer_norm(h, self.mlp_norm, None, cfg.norm_epsilon)
        g = N.gated_activation(N.linear(x, self.Wi), cfg.hidden_activation)
        return N.linear(g, self.mlp_Wo, residual=h)


class ModernBertTextTower(nn.Module):
    def __init__(self, cfg: ModernVBERTTextConfig, g: torch.Generator) -> None:
        super().__init__()
        self.config = cfg
        emb = torch.randn(cfg.vocab_size, cfg.hidden_size, generator=g) * cfg.initializer_range
        if 0 <= cfg.pad_token_id < cfg.vocab_size:
            emb[cfg.pad_token_id] = 0
        self.tok_embeddings = nn.Parameter(emb)
        self.emb_norm = nn.Parameter(torch.ones(cfg.hidden_size))
        self.layers = nn.ModuleList(ModernBertLayer(cfg, i, g) for i in range(cfg.num_hidden_layers))
        self.final_norm = nn.Parameter(torch.ones(cfg.hidden_size))
        d = cfg.head_dimension
        self.register_buffer("inv_freq_full", N.rope_inv_freq(d, cfg.full_attention_rope_theta), persistent=False)
        self.register_buffer("inv_freq_sliding", N.rope_inv_freq(d, cfg.sliding_attention_rope_theta),
                             persistent=False)

    def token_embeddings(self, ids: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        return _embed(ids, self.tok_embeddings, dtype)

    def forward(self, emb: torch.Tensor, seg: N.Segments, pos: torch.Tensor, *, all_layers: bool = False):
        cfg = self.config
        h = N.layer_norm(emb, self.emb_norm, None, cfg.norm_epsilon)
        states = [h]
        for layer in self.layers:
            f = self.inv_freq_full if layer.layer_type == "full_attention" else self.inv_freq_sliding
            h = layer(h, seg, pos, f, cfg)
            if all_layers:
                states.append(h)
        h = N.layer_norm(h, self.final_norm, None, cfg.norm_epsilon)
        if all_layers:
            states[-1] = h
            return states
        return h


class ModernVBERTTextEncoder(nn.Module):
    """Text-only ModernBERT encoder (mean pool + L2)."""

    def __init__(self, config: ModernVBERTTextConfig, *, seed: int = 0, model_id: str = "representax/modernbert",
                 revision: str = "random-init", compute_dtype: torch.dtype = torch.float32) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.config = config
        self.tower = ModernBertTextTower(config, g)
        self.compute_dtype = compute_dtype
        self.metadata = EncoderMetadata(model_id=model_id, revision=revision, output_dimension=config.hidden_size,
                                        routes=frozenset(Route), modalities=frozenset({Modality.TEXT}))

    @staticmethod
    def make_batch(*, input_ids, attention_mask, token_type_ids=None) -> TokenBatch:
        del token_type_ids
        return TokenBatch.from_arrays(input_ids=input_ids, attention_mask=attention_mask)

    def _packed(self, batch: TokenBatch):
        dtype = active_compute_dtype(self.compute_dtype)
        pk, seg = packed_segments(batch, self.tower.tok_embeddings.device)
        return pk, seg, self.tower.token_embeddings(pk.input_ids, dtype)

    def packed_hidden(self, batch: TokenBatch, *, all_layers: bool = False):
        pk, seg, emb = self._packed(batch)
        return self.tower(emb, seg, pk.position_ids, all_layers=all_layers), seg

    def hidden_states(self, inputs: TokenBatch, *, generator=None) -> torch.Tensor:
        h, seg = self.packed_hidden(inputs)
        return _unpack(h, inputs.attention_mask)

    def hidden_states_by_layer(self, inputs: TokenBatch, *, generator=None) -> torch.Tensor:
        states, seg = self.packed_hidden(inputs, all_layers=True)
        return torch.stack([_unpack(s, inputs.attention_mask) for s in states])

    def encode(self, inputs: TokenBatch, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        h, seg = self.packed_hidden(inputs)
        return N.pool_rows(h, seg, "mean", True)

    def encode_layers(self, inputs: TokenBatch, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        states, seg = self.packed_hidden(inputs, all_layers=True)
        return torch.stack([N.pool_rows(s, seg, "mean", True) for s in states])


def _unpack(h: torch.Tensor, mask: torch.Tensor) -> torch.Tensor:
    m = mask.to(h.device).bool()
    out = h.new_zeros(m.shape + (h.shape[-1],))
    out[m] = h
    return out


# ------------------------------------------------------------- vision tower
class VisionLayer(nn.Module):
    """Pre-LN transformer block (fused q/k/v) used by the SigLIP and CLIP towers."""

    def __init__(self, hidden: int, inter: int, g: torch.Generator, std: float = 0.02) -> None:
        super().__init__()
        self.ln1_w, self.ln1_b = nn.Parameter(torch.ones(hidden)), nn.Parameter(torch.zeros(hidden))
        self.qkv_w, self.qkv_b = _normal((3 * hidden, hidden), std, g), nn.Parameter(torch.zeros(3 * hidden))
        self.out_w, self.out_b = _normal((hidden, hidden), std, g), nn.Parameter(torch.zeros(hidden))
        self.ln2_w, self.ln2_b = nn.Parameter(torch.ones(hidden)), nn.Parameter(torch.zeros(hidden))
        self.fc1_w, self.fc1_b = _normal((inter, hidden), std, g), nn.Parameter(torch.zeros(inter))
        self.fc2_w, self.fc2_b = _normal((hidden, inter), std, g), nn.Parameter(torch.zeros(hidden))

    def forward(self, h, seg, heads: int, eps: float, act: str, causal: bool = False):
        x = N.layer_norm(h, self.ln1_w, self.ln1_b, eps)
        a = N.qkv_attention(N.linear(x, self.qkv_w, self.qkv_b), seg, heads=heads, causal=causal)
        h = N.linear(a, self.out_w, self.out_b, residual=h)
        x = N.layer_norm(h, self.ln2_w, self.ln2_b, eps)
        m = N.activation(N.linear(x, self.fc1_w, self.fc1_b), act)
        return N.linear(m, self.fc2_w, self.fc2_b, residual=h)


def patchify(pixels: torch.Tensor, patch: int) -> torch.Tensor:
    """[N, C, H, W] -> [N * (H/p) * (W/p), C * p * p], patches row-major, (c, y, x) inside."""

    n, c, hh, ww = pixels.shape
    gh, gw = hh // patch, ww // patch
    x = pixels.reshape(n, c, gh, patch, gw, patch).permute(0, 2, 4, 1, 3, 5)
    return x.reshape(n * gh * gw, c * patch * patch)


class SigLIPVisionTower(nn.Module):
    def __init__(self, cfg: SigLIPVisionConfig, g: torch.Generator, std: float = 0.02) -> None:
        super().__init__()
        self.config = cfg
        k = cfg.num_channels * cfg.patch_size ** 2
        self.patch_w = _normal((cfg.hidden_size, k), std, g)  # conv weight [out, C, p, p] flattened
        self.patch_b = nn.Parameter(torch.zeros(cfg.hidden_size))
        self.position = _normal((cfg.num_patches, cfg.hidden_size), std, g)
        self.layers = nn.ModuleList(VisionLayer(cfg.hidden_size, cfg.intermediate_size, g, std)
                                    for _ in range(cfg.num_hidden_layers))
        self.post_w, self.post_b = nn.Parameter(torch.ones(cfg.hidden_size)), nn.Parameter(torch.zeros(cfg.hidden_size))

    def forward(self, pixels: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """[N, C, H, W] -> [N, patches, hidden]."""

        cfg = self.config
        n = pixels.shape[0]
        patches = patchify(pixels.to(dtype), cfg.patch_size)
        pos = self.position.to(dtype).repeat(n, 1)
        h = N.linear(patches, self.patch_w, self.patch_b, residual=pos)
        seg = N.Segments.from_lengths([cfg.num_patches] * n, pixels.device)
        for layer in self.layers:
            h = layer(h, seg, cfg.num_attention_heads, cfg.norm_epsilon, cfg.hidden_activation)
        h = N.layer_norm(h, self.post_w, self.post_b, cfg.norm_epsilon)
        return h.reshape(n, cfg.num_patches, cfg.hidden_size)


def pixel_shuffle(x: torch.Tensor, factor: int) -> torch.Tensor:
    """Space-to-depth on the patch grid: [N, S, E] -> [N, S / r^2, E r^2].

    Row-major patch grid (h = w = sqrt(S)); groups of r consecutive columns
    are folded first, then groups of r rows, the same element order as the
    Transformers Idefics3 / ModernVBERT connector.
    """

    n, s, e = x.shape
    side = int(round(s ** 0.5))
    if side * side != s or side % factor:
        raise ValueError("pixel shuffle needs a square patch grid divisible by the factor")
    x = x.reshape(n, side, side // factor, e * factor)
    x = x.permute(0, 2, 1, 3).reshape(n, side // factor, side // factor, e * factor * factor)
    x = x.permute(0, 2, 1, 3)
    return x.reshape(n, s // factor ** 2, e * factor ** 2)


# --------------------------------------------------------------- multimodal
@dataclass
class ModernVBERTBatch:
    """Text tokens plus optional images ``[batch, images, C, H, W]``."""

    attention_mask: torch.Tensor
    input_ids: torch.Tensor
    pixel_values: torch.Tensor | None = None
    image_valid: torch.Tensor | None = None
    packed: PackedTokens | None = None

    def __post_init__(self) -> None:
        if self.input_ids.shape != self.attention_mask.shape:
            raise ValueError("input_ids and attention_mask must align")
        if self.pixel_values is not None:
            if self.pixel_values.ndim != 5 or self.pixel_values.shape[0] != self.input_ids.shape[0]:
                raise ValueError("pixel_values must have shape [batch, images, channels, H, W]")
            if self.image_valid is not None and tuple(self.image_valid.shape) != tuple(self.pixel_values.shape[:2]):
                raise ValueError("image_valid must have shape [batch, images]")
        elif self.image_valid is not None:
            raise ValueError("image masks require pixel_values")

    @property
    def batch_size(self) -> int:
        return self.input_ids.shape[0]

    def pack(self) -> "ModernVBERTBatch":
        return ModernVBERTBatch(self.attention_mask, self.input_ids, self.pixel_values, self.image_valid,
                                pack_tokens(self.input_ids, self.attention_mask))

    def text_batch(self) -> TokenBatch:
        return TokenBatch(attention_mask=self.attention_mask, input_ids=self.input_ids, packed=self.packed)

    def map_tensors(self, fn) -> "ModernVBERTBatch":
        opt = lambda t: None if t is None else fn(t)  # noqa: E731
        return ModernVBERTBatch(fn(self.attention_mask), fn(self.input_ids), opt(self.pixel_values),
                                opt(self.image_valid), None if self.packed is None else self.packed.map_tensors(fn))

    def rows(self, start: int, stop: int) -> "ModernVBERTBatch":
        opt = lambda t: None if t is None else t[start:stop]  # noqa: E731
        return ModernVBERTBatch(self.attention_mask[start:stop], self.input_ids[start:stop],
                                opt(self.pixel_values), opt(self.image_valid),
                                None if self.packed is None else self.packed.rows(start, stop))


def merge_image_features(packed_ids: torch.Tensor, seg: N.Segments, embeddings: torch.Tensor,
                         features: torch.Tensor, image_token_id: int,
                         image_valid: torch.Tensor | None = None) -> torch.Tensor:
    """Write image features into the image-token rows of packed embeddings.

    ``features`` is ``[batch, images, tokens, hidden]``; per record, the
    valid images' tokens are consumed in order by that record's image-token
    positions; image tokens beyond the valid features keep their embedding
    row replaced by zeros (the reference's padding behaviour).
    """

    b, n_img, n_tok, hidden = features.shape
    if image_valid is None:
        image_valid = torch.ones(b, n_img, dtype=torch.bool, device=features.device)
    order = torch.argsort((~image_valid.bool()).to(torch.int8), dim=1, stable=True)
    ordered = torch.gather(features, 1, order[:, :, None, None].expand_as(features)).reshape(b, n_img * n_tok, hidden)
    ordered = torch.cat([ordered, ordered.new_zeros(b, 1, hidden)], 1)
    valid_count = image_valid.sum(1) * n_tok
    is_img = packed_ids == image_token_id
    rec = torch.repeat_interleave(torch.arange(b, device=packed_ids.device),
                                  torch.as_tensor(seg.lengths(), device=packed_ids.device))
    # index of each image token among its record's image tokens
    csum = torch.cumsum(is_img.long(), 0)
    start = torch.as_tensor(seg.cu_host[:-1], device=packed_ids.device)
    before = torch.where(start > 0, csum[(start - 1).clamp_min(0)], torch.zeros_like(start))
    local = csum - 1 - before[rec]
    local = torch.where(is_img & (local < valid_count[rec]), local, torch.full_like(local, n_img * n_tok))
    gathered = ordered[rec, local.clamp_min(0)]
    return torch.where(is_img[:, None], gathered.to(embeddings.dtype), embeddings)


class ModernVBERTEncoder(nn.Module):
    """Text + image retriever: images -> SigLIP -> shuffle -> projection -> text tower."""

    def __init__(self, config: ModernVBERTConfig, *, seed: int = 0, model_id: str = "representax/modernvbert",
                 revision: str = "random-init", compute_dtype: torch.dtype = torch.float32) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.config = config
        self.text = ModernBertTextTower(config.text, g)
        self.vision = SigLIPVisionTower(config.vision, g)
        r = config.pixel_shuffle_factor
        self.connector = _normal((config.text.hidden_size, config.vision.hidden_size * r * r),
                                 config.text.initializer_range, g)
        self.compute_dtype = compute_dtype
        self.metadata = EncoderMetadata(model_id=model_id, revision=revision,
                                        output_dimension=config.text.hidden_size, routes=frozenset(Route),
                                        modalities=frozenset({Modality.TEXT, Modality.IMAGE}))

    @staticmethod
    def make_batch(*, input_ids, attention_mask, token_type_ids=None, pixel_values=None, image_valid=None):
        t = lambda v: None if v is None else torch.as_tensor(v)  # noqa: E731
        return ModernVBERTBatch(t(attention_mask).long(), t(input_ids).long(), t(pixel_values), t(image_valid))

    def image_features(self, pixel_values: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        b, n = pixel_values.shape[:2]
        hidden = self.vision(pixel_values.reshape(b * n, *pixel_values.shape[2:]), dtype)
        shuffled = pixel_shuffle(hidden, self.config.pixel_shuffle_factor)
        flat = shuffled.reshape(-1, shuffled.shape[-1])
        out = N.linear(flat, self.connector)
        return out.reshape(b, n, self.config.image_sequence_length, self.config.text.hidden_size)

    def packed_hidden(self, inputs, *, all_layers: bool = False):
        if isinstance(inputs, TokenBatch):
            inputs = ModernVBERTBatch(inputs.attention_mask, inputs.input_ids, packed=inputs.packed)
        dtype = active_compute_dtype(self.compute_dtype)
        device = self.text.tok_embeddings.device
        pk, seg = packed_segments(inputs.text_batch(), device)
        emb = self.text.token_embeddings(pk.input_ids, dtype)
        if inputs.pixel_values is not None:
            feats = self.image_features(inputs.pixel_values.to(device), dtype)
            valid = None if inputs.image_valid is None else inputs.image_valid.to(device)
            emb = merge_image_features(pk.input_ids, seg, emb, feats, self.config.image_token_id, valid)
        return self.text(emb, seg, pk.position_ids, all_layers=all_layers), seg

    def hidden_states(self, inputs, *, generator=None) -> torch.Tensor:
        h, _ = self.packed_hidden(inputs)
        return _unpack(h, inputs.attention_mask)

    def hidden_states_by_layer(self, inputs, *, generator=None) -> torch.Tensor:
        states, _ = self.packed_hidden(inputs, all_layers=True)
        return torch.stack([_unpack(s, inputs.attention_mask) for s in states])

    def encode(self, inputs, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        h, seg = self.packed_hidden(inputs)
        return N.pool_rows(h, seg, "mean", True)

    def encode_layers(self, inputs, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        states, seg = self.packed_hidden(inputs, all_layers=True)
        return torch.stack([N.pool_rows(s, seg, "mean", True) for s in states])


__all__ = ["ModernBertLayer", "ModernBertTextTower", "ModernVBERTBatch", "ModernVBERTEncoder",
           "ModernVBERTTextEncoder", "SigLIPVisionTower", "VisionLayer", "merge_image_features", "patchify",
           "pixel_shuffle"]
