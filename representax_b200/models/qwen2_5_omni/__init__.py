"""Qwen2.5-Omni thinker as a text / image / audio / video embedder.

* Text: Qwen2.5 decoder (q/k/v biases, no q/k norm) with sectioned M-RoPE
  (the first ``mrope_section[0]`` frequencies rotate with the temporal
  position, the next ``[1]`` with height, the last ``[2]`` with width).
* Vision: flattened (t, p, p) patches -> bias-free projection -> blocks of
  RMSNorm / fused-q/k/v attention with 2-D RoPE / RMSNorm / SwiGLU MLP.
  Most blocks attend inside windows of ``window_size`` pixels (patches are
  re-ordered window by window, as merged 2x2 units); ``fullatt_block_indexes``
  attend over whole frames. Merger: RMSNorm -> 2x2 concat -> fc -> GELU -> fc,
  then the window order is undone.
* Audio: log-mel frames in chunks of ``2 * n_window``: conv(k3) -> GELU ->
  conv(k3, stride 2) -> GELU (both as im2col GEMMs) + sinusoidal positions,
  pre-LN blocks attending within each chunk, 2x average pooling, LayerNorm,
  projection.
* Multimodal positions: text, audio and marker tokens advance all axes by
  one; an image spans its (t * 25, h, w) merged grid from the running
  position and the next token starts at the grid maximum plus one.
* Representation: last (or mean) valid token, L2-normalised.

Parity: src/representax/models/qwen2_5_omni/{config,text,vision,audio,model,
checkpoint}.py (M11). Video frames use the image path (one grid per frame
group); the audio-interleaved video position scheme is not implemented.
"""

from __future__ import annotations

import json
import os
from collections.abc import Mapping, Sequence
from dataclasses import dataclass
from pathlib import Path
from typing import Any

import numpy as np
import torch
from torch import nn

from representax_b200._config import FrozenConfig
from representax_b200.core.model import EncoderMetadata, Modality, Route
from representax_b200.integrations.huggingface import load_hf_config, load_safetensor_subset, save_safetensors
from representax_b200.models.qwen3 import (
    Qwen3TextConfig,
    Qwen3TextTower,
    last_token_rows,
    load_qwen3_tower,
    qwen3_tower_state,
)
from representax_b200.models.qwen3_vl import vision_layout
from representax_b200.models.text_batch import PackedTokens, pack_tokens
from representax_b200.ops import nn as N
from representax_b200.precision import active_compute_dtype


class OmniVisionConfig(FrozenConfig):
    depth: int = 32
    hidden_size: int = 1280
    intermediate_size: int = 3420
    num_heads: int = 16
    in_channels: int = 3
    patch_size: int = 14
    temporal_patch_size: int = 2
    spatial_merge_size: int = 2
    out_hidden_size: int = 2048
    window_size: int = 112
    fullatt_block_indexes: tuple[int, ...] = (7, 15, 23, 31)
    hidden_activation: str = "silu"

    @property
    def patch_dim(self) -> int:
        return self.in_channels * self.temporal_patch_size * self.patch_size ** 2

    @property
    def merger_window(self) -> int:
        return self.window_size // self.spatial_merge_size // self.patch_size


class OmniAudioConfig(FrozenConfig):
    num_mel_bins: int = 128
    d_model: int = 1280
    encoder_layers: int = 32
    encoder_attention_heads: int = 20
    encoder_ffn_dim: int = 5120
    output_dim: int = 2048
    max_source_positions: int = 1500
    n_window: int = 100


class Qwen2_5OmniConfig(FrozenConfig):
    text: Qwen3TextConfig = Qwen3TextConfig(qkv_bias=True, qk_norm=False, mrope_section=(16, 24, 24),
                                            mrope_interleaved=False)
    vision: OmniVisionConfig = OmniVisionConfig()
    audio: OmniAudioConfig = OmniAudioConfig()
    image_token_id: int = 151655
    video_token_id: int = 151656
    audio_token_id: int = 151646
    position_id_per_seconds: int = 25
    pooling: str = "last"

    @classmethod
    def from_hf_config(cls, value: Mapping[str, Any]) -> "Qwen2_5OmniConfig":
        v = value.get("thinker_config", value)
        text = Qwen3TextConfig.from_hf_config(v["text_config"], qkv_bias=True, qk_norm=False, mrope_interleaved=False)
        vc, ac = v["vision_config"], v["audio_config"]
        return cls(
            text=text,
            vision=OmniVisionConfig(depth=int(vc["depth"]), hidden_size=int(vc["hidden_size"]),
                                    intermediate_size=int(vc["intermediate_size"]), num_heads=int(vc["num_heads"]),
                                    in_channels=int(vc.get("in_channels", 3)), patch_size=int(vc["patch_size"]),
                                    temporal_patch_size=int(vc.get("temporal_patch_size", 2)),
                                    spatial_merge_size=int(vc.get("spatial_merge_size", 2)),
                                    out_hidden_size=int(vc["out_hidden_size"]), window_size=int(vc["window_size"]),
                                    fullatt_block_indexes=tuple(int(i) for i in vc.get("fullatt_block_indexes", ())),
                                    hidden_activation=str(vc.get("hidden_act", "silu"))),
            audio=OmniAudioConfig(num_mel_bins=int(ac["num_mel_bins"]), d_model=int(ac["d_model"]),
                                  encoder_layers=int(ac["encoder_layers"]),
                                  encoder_attention_heads=int(ac["encoder_attention_heads"]),
                                  encoder_ffn_dim=int(ac["encoder_ffn_dim"]), output_dim=int(ac["output_dim"]),
                                  max_source_positions=int(ac.get("max_source_positions", 1500)),
                                  n_window=int(ac.get("n_window", 100))),
            image_token_id=int(v.get("image_token_index", v.get("image_token_id", 151655))),
            video_token_id=int(v.get("video_token_index", v.get("video_token_id", 151656))),
            audio_token_id=int(v.get("audio_token_index", v.get("audio_token_id", 151646))),
            position_id_per_seconds=int(v.get("position_id_per_seconds", 25)))


# --------------------------------------------------------------- host prep
def window_order(grid_thw: Sequence[Sequence[int]], merge: int, window: int):
    """Permutation of merged 2x2 units into window order, and window lengths (in patches)."""

    order, lengths, base = [], [], 0
    for t, h, w in grid_thw:
        gh, gw = int(h) // merge, int(w) // merge
        idx = np.arange(int(t) * gh * gw).reshape(int(t), gh, gw)
        nh, nw = -(-gh // window), -(-gw // window)
        for f in range(int(t)):
            for a in range(nh):
                for b in range(nw):
                    block = idx[f, a * window:(a + 1) * window, b * window:(b + 1) * window].reshape(-1)
                    if block.size:
                        order.append(block + base)
                        lengths.append(block.size * merge * merge)
        base += int(t) * gh * gw
    return np.concatenate(order) if order else np.zeros(0, np.int64), lengths


def omni_positions(input_ids: np.ndarray, attention_mask: np.ndarray, grid_thw: Sequence[Sequence[int]],
                   image_token_id: int, merge: int, per_second: int) -> np.ndarray:
    b, s = input_ids.shape
    out = np.zeros((3, b, s), dtype=np.int64)
    grids = iter([tuple(int(v) for v in g) for g in grid_thw])
    for i in range(b):
        valid = np.nonzero(attention_mask[i])[0]
        ids = input_ids[i, valid]
        pos = np.zeros((3, len(ids)), dtype=np.int64)
        nxt, j = 0, 0
        while j < len(ids):
            if ids[j] == image_token_id:
                t, h, w = next(grids)
                gh, gw = h // merge, w // merge
                n = t * gh * gw
                tt = np.repeat(np.arange(t) * per_second, gh * gw)
                hh = np.tile(np.repeat(np.arange(gh), gw), t)
                ww = np.tile(np.arange(gw), gh * t)
                grid = np.stack([tt, hh, ww]) + nxt
                pos[:, j:j + n] = grid
                nxt = int(grid.max()) + 1
                j += n
            else:
                pos[:, j] = nxt
                nxt += 1
                j += 1
        out[:, i, valid] = pos
    return out


@dataclass
class Qwen2_5OmniBatch:
    input_ids: torch.Tensor
    attention_mask: torch.Tensor
    pixel_values: torch.Tensor | None = None      # [patches, C * T * p * p]
    image_grid_thw: torch.Tensor | None = None    # [images, 3]
    input_features: torch.Tensor | None = None    # [mel, frames of all audios]
    feature_lens: torch.Tensor | None = None      # [audios]
    packed: PackedTokens | None = None
    packed_positions: torch.Tensor | None = None

    @property
    def batch_size(self) -> int:
        return self.input_ids.shape[0]

    def prepare(self, config: Qwen2_5OmniConfig) -> "Qwen2_5OmniBatch":
        ids = self.input_ids.cpu().numpy()
        mask = self.attention_mask.cpu().numpy().astype(bool)
        grids = [] if self.image_grid_thw is None else self.image_grid_thw.tolist()
        pos = omni_positions(ids, mask, grids, config.image_token_id, config.vision.spatial_merge_size,
                             config.position_id_per_seconds)
        rows, cols = np.nonzero(mask)
        return Qwen2_5OmniBatch(self.input_ids, self.attention_mask, self.pixel_values, self.image_grid_thw,
                                self.input_features, self.feature_lens, pack_tokens(self.input_ids, self.attention_mask),
                                torch.from_numpy(np.ascontiguousarray(pos[:, rows, cols]).astype(np.int32)))

    def map_tensors(self, fn) -> "Qwen2_5OmniBatch":
        opt = lambda t: None if t is None else fn(t)  # noqa: E731
        return Qwen2_5OmniBatch(fn(self.input_ids), fn(self.attention_mask), opt(self.pixel_values),
                                self.image_grid_thw, opt(self.input_features), self.feature_lens,
                                None if self.packed is None else self.packed.map_tensors(fn),
                                opt(self.packed_positions))


def _normal(shape, std, g):
    return nn.Parameter(torch.randn(*shape, generator=g) * std)


# ------------------------------------------------------------------ vision
class _OmniVisionBlock(nn.Module):
    def __init__(self, cfg: OmniVisionConfig, g) -> None:
        super().__init__()
        h, i = cfg.hidden_size, cfg.intermediate_size
        self.n1, self.n2 = nn.Parameter(torch.ones(h)), nn.Parameter(torch.ones(h))
        self.qkv_w, self.qkv_b = _normal((3 * h, h), 0.02, g), nn.Parameter(torch.zeros(3 * h))
        self.proj_w, self.proj_b = _normal((h, h), 0.02, g), nn.Parameter(torch.zeros(h))
        self.gate_up_w, self.gate_up_b = _normal((2 * i, h), 0.02, g), nn.Parameter(torch.zeros(2 * i))
        self.down_w, self.down_b = _normal((h, i), 0.02, g), nn.Parameter(torch.zeros(h))

    def forward(self, h, seg, pos, axis, inv, cfg: OmniVisionConfig):
        x = N.rms_norm(h, self.n1, 1e-6)
        a = N.qkv_attention(N.linear(x, self.qkv_w, self.qkv_b), seg, heads=cfg.num_heads, pos=pos, inv_freq=inv,
                            axis_of=axis)
        h = N.linear(a, self.proj_w, self.proj_b, residual=h)
        x = N.rms_norm(h, self.n2, 1e-6)
        m = N.gated_activation(N.linear(x, self.gate_up_w, self.gate_up_b), cfg.hidden_activation)
        return N.linear(m, self.down_w, self.down_b, residual=h)


class OmniVisionTower(nn.Module):
    def __init__(self, cfg: OmniVisionConfig, g) -> None:
        super().__init__()
        self.config = cfg
        self.patch_w = _normal((cfg.hidden_size, cfg.patch_dim), 0.02, g)
        self.blocks = nn.ModuleList(_OmniVisionBlock(cfg, g) for _ in range(cfg.depth))
        wide = cfg.hidden_size * cfg.spatial_merge_size ** 2
        self.ln_q = nn.Parameter(torch.ones(cfg.hidden_size))
        self.fc1_w, self.fc1_b = _normal((wide, wide), 0.02, g), nn.Parameter(torch.zeros(wide))
        self.fc2_w, self.fc2_b = _normal((cfg.out_hidden_size, wide), 0.02, g), nn.Parameter(torch.zeros(cfg.out_hidden_size))
        d = cfg.hidden_size // cfg.num_heads
        inv = N.rope_inv_freq(d // 2, 10000.0)
        self.register_buffer("inv_freq", torch.cat([inv, inv]), persistent=False)
        self.register_buffer("axis_of", torch.tensor([0] * (d // 4) + [1] * (d // 4), dtype=torch.int32),
                             persistent=False)

    def forward(self, pixels: torch.Tensor, grid_thw: Sequence[Sequence[int]], dtype: torch.dtype) -> torch.Tensor:
        cfg = self.config
        dev = pixels.device
        unit = cfg.spatial_merge_size ** 2
        rc, _, _, frames = vision_layout(grid_thw, cfg.spatial_merge_size, 1)
        order, win_lengths = window_order(grid_thw, cfg.spatial_merge_size, cfg.merger_window)
        order_t = torch.from_numpy(order).to(dev)
        h = N.linear(pixels.to(dtype), self.patch_w)
        n = h.shape[0]
        h = h.reshape(n // unit, unit, -1)[order_t].reshape(n, -1)
        pos = torch.from_numpy(rc).to(dev).reshape(2, n // unit, unit)[:, order_t].reshape(2, n)
        full = N.Segments.from_lengths(frames, dev)
        windows = N.Segments.from_lengths(win_lengths, dev)
        for i, blk in enumerate(self.blocks):
            h = blk(h, full if i in cfg.fullatt_block_indexes else windows, pos, self.axis_of, self.inv_freq, cfg)
        x = N.rms_norm(h, self.ln_q, 1e-6).reshape(n // unit, -1)
        merged = N.linear(N.activation(N.linear(x, self.fc1_w, self.fc1_b), "gelu"), self.fc2_w, self.fc2_b)
        return merged[torch.argsort(order_t)]


# ------------------------------------------------------------------- audio
def _conv1d(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, stride: int) -> torch.Tensor:
    """x [chunks, L, C_in] -> [chunks, L_out, C_out]; kernel 3, padding 1, as an im2col GEMM."""

    c, L, cin = x.shape
    xp = torch.nn.functional.pad(x, (0, 0, 1, 1))
    cols = xp.unfold(1, 3, stride)                       # [c, L_out, C_in, 3]
    lout = cols.shape[1]
    y = N.linear(cols.reshape(c * lout, cin * 3), weight.reshape(weight.shape[0], -1), bias)
    return y.reshape(c, lout, -1)


class OmniAudioTower(nn.Module):
    def __init__(self, cfg: OmniAudioConfig, g) -> None:
        super().__init__()
        self.config = cfg
        d = cfg.d_model
        self.conv1_w, self.conv1_b = _normal((d, cfg.num_mel_bins, 3), 0.02, g), nn.Parameter(torch.zeros(d))
        self.conv2_w, self.conv2_b = _normal((d, d, 3), 0.02, g), nn.Parameter(torch.zeros(d))
        from representax_b200.models.modernvbert.model import VisionLayer

        self.layers = nn.ModuleList(VisionLayer(d, cfg.encoder_ffn_dim, g) for _ in range(cfg.encoder_layers))
        self.ln_post_w, self.ln_post_b = nn.Parameter(torch.ones(d)), nn.Parameter(torch.zeros(d))
        self.proj_w, self.proj_b = _normal((cfg.output_dim, d), 0.02, g), nn.Parameter(torch.zeros(cfg.output_dim))
        self.register_buffer("positions", N.sinusoid_table(cfg.max_source_positions, d), persistent=False)

    def forward(self, features: torch.Tensor, lengths: Sequence[int], dtype: torch.dtype) -> torch.Tensor:
        """features [mel, frames]; returns audio tokens of all clips, concatenated."""

        cfg = self.config
        dev = features.device
        span = 2 * cfg.n_window
        chunks = []
        for n in lengths:
            full, rest = divmod(int(n), span)
            chunks += [span] * full + ([rest] if rest else [])
        cmax = max(chunks)
        x = torch.zeros(len(chunks), cmax, cfg.num_mel_bins, dtype=dtype, device=dev)
        mask = torch.zeros(len(chunks), cmax, 1, dtype=dtype, device=dev)
        frames = features.T.to(dtype)
        off = 0
        for i, n in enumerate(chunks):
            x[i, :n] = frames[off:off + n]
            mask[i, :n] = 1
            off += n
        h = N.activation(_conv1d(x, self.conv1_w, self.conv1_b, 1).reshape(-1, cfg.d_model), "gelu")
        h = h.reshape(len(chunks), cmax, -1) * mask
        h = _conv1d(h, self.conv2_w, self.conv2_b, 2)
        h = N.activation(h.reshape(-1, cfg.d_model), "gelu").reshape(len(chunks), -1, cfg.d_model)
        h = h + self.positions[: h.shape[1]].to(dtype)
        after = [(n - 1) // 2 + 1 for n in chunks]
        rows = torch.cat([torch.arange(a, device=dev) + i * h.shape[1] for i, a in enumerate(after)])
        h = h.reshape(-1, cfg.d_model)[rows]
        seg = N.Segments.from_lengths(after, dev)
        for layer in self.layers:
            h = layer(h, seg, cfg.encoder_attention_heads, 1e-5, "gelu")
        outs, off = [], 0
        per_clip = [(int(n) - 1) // 2 + 1 for n in lengths]
        for n in per_clip:
            clip = h[off:off + n]
            off += n
            m = n // 2
            outs.append((clip[: 2 * m].reshape(m, 2, -1).float().mean(1)).to(dtype))
        h = torch.cat(outs)
        h = N.layer_norm(h, self.ln_post_w, self.ln_post_b, 1e-5)
        return N.linear(h, self.proj_w, self.proj_b)


# ------------------------------------------------------------------- model
class Qwen2_5OmniEncoder(nn.Module):
    def __init__(self, config: Qwen2_5OmniConfig, *, seed: int = 0, model_id: str = "representax/qwen2.5-omni",
                 revision: str = "random-init", compute_dtype: torch.dtype = torch.float32) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.config = config
        self.text = Qwen3TextTower(config.text, g)
        self.vision = OmniVisionTower(config.vision, g)
        self.audio = OmniAudioTower(config.audio, g)
        self.compute_dtype = compute_dtype
        self.metadata = EncoderMetadata(model_id=model_id, revision=revision,
                                        output_dimension=config.text.hidden_size, routes=frozenset(Route),
                                        modalities=frozenset({Modality.TEXT, Modality.IMAGE, Modality.AUDIO,
                                                              Modality.VIDEO}))

    def packed_hidden(self, inputs: Qwen2_5OmniBatch):
        dtype = active_compute_dtype(self.compute_dtype)
        dev = self.text.embed_tokens.device
        if inputs.packed is None:
            inputs = inputs.prepare(self.config)
        pk = inputs.packed.map_tensors(lambda t: t.to(dev, non_blocking=True))
        seg = N.Segments([int(v) for v in pk.cu_host.tolist()], pk.cu_seqlens.to(dev, torch.int32))
        emb = self.text.token_embeddings(pk.input_ids, dtype)
        if inputs.pixel_values is not None:
            feats = self.vision(inputs.pixel_values.to(dev), inputs.image_grid_thw.tolist(), dtype)
            rows = torch.nonzero(pk.input_ids == self.config.image_token_id).flatten()
            emb = emb.index_copy(0, rows, feats.to(dtype))
        if inputs.input_features is not None:
            feats = self.audio(inputs.input_features.to(dev), [int(n) for n in inputs.feature_lens.tolist()], dtype)
            rows = torch.nonzero(pk.input_ids == self.config.audio_token_id).flatten()
            emb = emb.index_copy(0, rows, feats.to(dtype))
        return self.text(emb, seg, inputs.packed_positions.to(dev)), seg

    def hidden_states(self, inputs: Qwen2_5OmniBatch, *, generator=None) -> torch.Tensor:
        h, _ = self.packed_hidden(inputs)
        m = inputs.attention_mask.to(h.device).bool()
        out = h.new_zeros(m.shape + (h.shape[-1],))
        out[m] = h
        return out

    def encode(self, inputs: Qwen2_5OmniBatch, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        h, seg = self.packed_hidden(inputs)
        if self.config.pooling == "mean":
            return N.pool_rows(h, seg, "mean", True)
        v = h[last_token_rows(seg)].float()
        return v / v.norm(dim=-1, keepdim=True).clamp_min(1e-12)


# -------------------------------------------------------------- checkpoint
def _omni_extra(model: Qwen2_5OmniEncoder, vp: str, ap: str):
    """(hf name, tensor, native shape) for the vision and audio towers."""

    v, a = model.vision, model.audio
    vc = model.config.vision
    yield vp + "patch_embed.proj.weight", v.patch_w, (vc.hidden_size, vc.in_channels, vc.temporal_patch_size,
                                                      vc.patch_size, vc.patch_size)
    for i, b in enumerate(v.blocks):
        q = f"{vp}blocks.{i}."
        yield q + "norm1.weight", b.n1, None
        yield q + "norm2.weight", b.n2, None
        yield q + "attn.proj.weight", b.proj_w, None
        yield q + "attn.proj.bias", b.proj_b, None
        yield q + "mlp.down_proj.weight", b.down_w, None
        yield q + "mlp.down_proj.bias", b.down_b, None
    yield vp + "merger.ln_q.weight", v.ln_q, None
    yield vp + "merger.mlp.0.weight", v.fc1_w, None
    yield vp + "merger.mlp.0.bias", v.fc1_b, None
    yield vp + "merger.mlp.2.weight", v.fc2_w, None
    yield vp + "merger.mlp.2.bias", v.fc2_b, None
    for name, t in (("conv1.weight", a.conv1_w), ("conv1.bias", a.conv1_b), ("conv2.weight", a.conv2_w),
                    ("conv2.bias", a.conv2_b), ("ln_post.weight", a.ln_post_w), ("ln_post.bias", a.ln_post_b),
                    ("proj.weight", a.proj_w), ("proj.bias", a.proj_b)):
        yield ap + name, t, None
    for i, layer in enumerate(a.layers):
        q = f"{ap}layers.{i}."
        for attr, name in (("out", "self_attn.out_proj"), ("fc1", "fc1"), ("fc2", "fc2"),
                           ("ln1", "self_attn_layer_norm"), ("ln2", "final_layer_norm")):
            yield q + name + ".weight", getattr(layer, attr + "_w"), None
            yield q + name + ".bias", getattr(layer, attr + "_b"), None


class Qwen2_5OmniCheckpointAdapter:
    PREFIXES = (("thinker.model.", "thinker.visual.", "thinker.audio_tower."), ("model.", "visual.", "audio_tower."))

    @classmethod
    def state_dict(cls, model: Qwen2_5OmniEncoder) -> dict[str, torch.Tensor]:
        tp, vp, ap = cls.PREFIXES[1]
        out = qwen3_tower_state(model.text, tp)
        for name, t, shape in _omni_extra(model, vp, ap):
            out[name] = t.detach().reshape(shape) if shape else t.detach()
        for i, b in enumerate(model.vision.blocks):
            q = f"{vp}blocks.{i}."
            h = model.config.vision.hidden_size
            inter = model.config.vision.intermediate_size
            for j, n in enumerate(("q", "k", "v")):
                out[q + f"attn.{n}.weight"] = b.qkv_w.detach()[j * h:(j + 1) * h]
                out[q + f"attn.{n}.bias"] = b.qkv_b.detach()[j * h:(j + 1) * h]
            out[q + "mlp.gate_proj.weight"] = b.gate_up_w.detach()[:inter]
            out[q + "mlp.up_proj.weight"] = b.gate_up_w.detach()[inter:]
            out[q + "mlp.gate_proj.bias"] = b.gate_up_b.detach()[:inter]
            out[q + "mlp.up_proj.bias"] = b.gate_up_b.detach()[inter:]
        d = model.config.audio.d_model
        for i, layer in enumerate(model.audio.layers):
            q = f"{ap}layers.{i}."
            for j, n in enumerate(("q_proj", "k_proj", "v_proj")):
                out[q + f"self_attn.{n}.weight"] = layer.qkv_w.detach()[j * d:(j + 1) * d]
                if n != "k_proj":
                    out[q + f"self_attn.{n}.bias"] = layer.qkv_b.detach()[j * d:(j + 1) * d]
        return {k: v.float().cpu().contiguous() for k, v in out.items()}

    @classmethod
    def from_state_dict(cls, model: Qwen2_5OmniEncoder, t: Mapping[str, torch.Tensor]) -> Qwen2_5OmniEncoder:
        tp, vp, ap = next(p for p in cls.PREFIXES if p[0] + "embed_tokens.weight" in t)
        load_qwen3_tower(model.text, t, tp)
        with torch.no_grad():
            for name, target, shape in _omni_extra(model, vp, ap):
                target.copy_(t[name].reshape(target.shape))
            vc, d = model.config.vision, model.config.audio.d_model
            for i, b in enumerate(model.vision.blocks):
                q = f"{vp}blocks.{i}."
                b.qkv_w.copy_(torch.cat([t[q + f"attn.{n}.weight"] for n in "qkv"]))
                b.qkv_b.copy_(torch.cat([t[q + f"attn.{n}.bias"] for n in "qkv"]))
                b.gate_up_w.copy_(torch.cat([t[q + "mlp.gate_proj.weight"], t[q + "mlp.up_proj.weight"]]))
                b.gate_up_b.copy_(torch.cat([t[q + "mlp.gate_proj.bias"], t[q + "mlp.up_proj.bias"]]))
            for i, layer in enumerate(model.audio.layers):
                q = f"{ap}layers.{i}."
                layer.qkv_w.copy_(torch.cat([t[q + f"self_attn.{n}.weight"] for n in ("q_proj", "k_proj", "v_proj")]))
                layer.qkv_b.copy_(torch.cat([t[q + "self_attn.q_proj.bias"], torch.zeros(d),
                                             t[q + "self_attn.v_proj.bias"]]))
        return model

    @classmethod
    def load(cls, path: str | os.PathLike, *, compute_dtype: torch.dtype = torch.float32, **kwargs):
        path = Path(path)
        kwargs.setdefault("model_id", path.name)
        kwargs.setdefault("revision", "local")
        model = Qwen2_5OmniEncoder(Qwen2_5OmniConfig.from_hf_config(load_hf_config(path)),
                                   compute_dtype=compute_dtype, **kwargs)
        from safetensors import safe_open

        from representax_b200.integrations.huggingface import _weight_files

        names = set()
        for file in _weight_files(path):
            with safe_open(str(file), framework="pt") as handle:
                names |= set(handle.keys())
        return cls.from_state_dict(model, load_safetensor_subset(path, names))

    @classmethod
    def save(cls, model: Qwen2_5OmniEncoder, path: str | os.PathLike) -> None:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        save_safetensors(cls.state_dict(model), path / "model.safetensors")


def build_qwen2_5_omni(*, seed: int = 0, compute_dtype: str = "float32", **config) -> Qwen2_5OmniEncoder:
    return Qwen2_5OmniEncoder(Qwen2_5OmniConfig(**config), seed=seed, compute_dtype=getattr(torch, compute_dtype))


__all__ = ["OmniAudioConfig", "OmniAudioTower", "OmniVisionConfig", "OmniVisionTower", "Qwen2_5OmniBatch",
           "Qwen2_5OmniCheckpointAdapter", "Qwen2_5OmniConfig", "Qwen2_5OmniEncoder", "build_qwen2_5_omni",
           "omni_positions", "window_order"]
