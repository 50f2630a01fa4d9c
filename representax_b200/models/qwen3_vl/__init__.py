"""Qwen3-VL embedder and reranker: ViT with 2-D RoPE + DeepStack, M-RoPE decoder.

Vision: flattened (t, p, p) patches -> patch projection + bilinearly
interpolated learned positions -> pre-LN blocks (fused q/k/v, 2-D rotary
embedding over (row, column), attention within each frame, tanh-GELU MLP)
-> 2x2 spatial merger (LayerNorm -> fc -> GELU -> fc); DeepStack mergers tap
chosen blocks and their outputs are added to the visual-token rows of the
first decoder layers. Text: the Qwen3 decoder with interleaved M-RoPE
positions (text tokens advance all three axes together; an image occupies
a (t, h, w) grid offset by the running position). Embeddings pool the
last valid token; the reranker scores sigmoid(h_last . (E[yes] - E[no])).

Parity: src/representax/models/qwen3_vl/{config,vision,text,model,
checkpoint,processing}.py (M10).
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
from representax_b200.models.text_batch import PackedTokens, pack_tokens
from representax_b200.ops import nn as N
from representax_b200.precision import active_compute_dtype


class Qwen3VLVisionConfig(FrozenConfig):
    depth: int = 24
    hidden_size: int = 1024
    intermediate_size: int = 4096
    num_heads: int = 16
    in_channels: int = 3
    patch_size: int = 16
    temporal_patch_size: int = 2
    spatial_merge_size: int = 2
    out_hidden_size: int = 2048
    num_position_embeddings: int = 2304
    deepstack_visual_indexes: tuple[int, ...] = (5, 11, 17)
    hidden_activation: str = "gelu_pytorch_tanh"
    rope_theta: float = 10000.0

    @property
    def head_dimension(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def patch_dim(self) -> int:
        return self.in_channels * self.temporal_patch_size * self.patch_size ** 2

    @classmethod
    def from_hf_config(cls, value: Mapping[str, Any]) -> "Qwen3VLVisionConfig":
        v = value.get("vision_config", value)
        return cls(depth=int(v["depth"]), hidden_size=int(v["hidden_size"]),
                   intermediate_size=int(v["intermediate_size"]), num_heads=int(v["num_heads"]),
                   in_channels=int(v.get("in_channels", 3)), patch_size=int(v["patch_size"]),
                   temporal_patch_size=int(v.get("temporal_patch_size", 2)),
                   spatial_merge_size=int(v.get("spatial_merge_size", 2)), out_hidden_size=int(v["out_hidden_size"]),
                   num_position_embeddings=int(v["num_position_embeddings"]),
                   deepstack_visual_indexes=tuple(int(i) for i in v.get("deepstack_visual_indexes", ())),
                   hidden_activation=str(v.get("hidden_act", "gelu_pytorch_tanh")))

    def to_hf_config(self) -> dict[str, Any]:
        return {"depth": self.depth, "hidden_size": self.hidden_size, "intermediate_size": self.intermediate_size,
                "num_heads": self.num_heads, "in_channels": self.in_channels, "patch_size": self.patch_size,
                "temporal_patch_size": self.temporal_patch_size, "spatial_merge_size": self.spatial_merge_size,
                "out_hidden_size": self.out_hidden_size, "num_position_embeddings": self.num_position_embeddings,
                "deepstack_visual_indexes": list(self.deepstack_visual_indexes), "hidden_act": self.hidden_activation}


class Qwen3VLConfig(FrozenConfig):
    text: Qwen3TextConfig = Qwen3TextConfig(mrope_section=(24, 20, 20))
    vision: Qwen3VLVisionConfig = Qwen3VLVisionConfig()
    image_token_id: int = 151655
    video_token_id: int = 151656
    vision_start_token_id: int = 151652

    @classmethod
    def from_hf_config(cls, value: Mapping[str, Any]) -> "Qwen3VLConfig":
        return cls(text=Qwen3TextConfig.from_hf_config(value), vision=Qwen3VLVisionConfig.from_hf_config(value),
                   image_token_id=int(value.get("image_token_id", 151655)),
                   video_token_id=int(value.get("video_token_id", 151656)),
                   vision_start_token_id=int(value.get("vision_start_token_id", 151652)))

    def to_hf_config(self) -> dict[str, Any]:
        return {"model_type": "qwen3_vl", "text_config": {"model_type": "qwen3_vl_text", **self.text.to_hf_config()},
                "vision_config": {"model_type": "qwen3_vl", **self.vision.to_hf_config()},
                "image_token_id": self.image_token_id, "video_token_id": self.video_token_id,
                "vision_start_token_id": self.vision_start_token_id,
                "tie_word_embeddings": self.text.tie_word_embeddings}


# --------------------------------------------------------------- host prep
def vision_layout(grid_thw: Sequence[Sequence[int]], merge: int, grid_side: int):
    """Per-patch (row, col) rotary positions, 4-corner interpolation indices /
    weights into the learned ``grid_side^2`` position table, and frame lengths,
    all in the processor's patch order (t, row block, col block, m, m)."""

    rows, cols, idx, wts, frames = [], [], [[] for _ in range(4)], [[] for _ in range(4)], []
    for t, h, w in grid_thw:
        t, h, w = int(t), int(h), int(w)
        r = np.arange(h).reshape(h // merge, merge)[:, None, :, None]
        c = np.arange(w).reshape(w // merge, merge)[None, :, None, :]
        rr = np.broadcast_to(r, (h // merge, w // merge, merge, merge)).reshape(-1)
        cc = np.broadcast_to(c, (h // merge, w // merge, merge, merge)).reshape(-1)
        rows += [rr] * t
        cols += [cc] * t
        hs = np.linspace(0, grid_side - 1, h, dtype=np.float32)
        ws = np.linspace(0, grid_side - 1, w, dtype=np.float32)
        h0, w0 = hs.astype(np.int64), ws.astype(np.int64)
        h1, w1 = np.minimum(h0 + 1, grid_side - 1), np.minimum(w0 + 1, grid_side - 1)
        dh, dw = hs - h0, ws - w0
        corners = [(h0, w0, (1 - dh)[:, None] * (1 - dw)[None]), (h0, w1, (1 - dh)[:, None] * dw[None]),
                   (h1, w0, dh[:, None] * (1 - dw)[None]), (h1, w1, dh[:, None] * dw[None])]
        for k, (hh, ww, wt) in enumerate(corners):
            grid_idx = hh[:, None] * grid_side + ww[None]           # [h, w] row-major
            ordered = grid_idx[rr, cc]                               # merge-window order
            ordered_w = wt[rr, cc]
            idx[k] += [ordered] * t
            wts[k] += [ordered_w] * t
        frames += [h * w] * t
    cat = lambda xs: np.concatenate(xs) if xs else np.zeros(0)  # noqa: E731
    return (np.stack([cat(rows), cat(cols)]).astype(np.int32), np.stack([cat(i) for i in idx]).astype(np.int64),
            np.stack([cat(x) for x in wts]).astype(np.float32), frames)


def rope_positions(input_ids: np.ndarray, attention_mask: np.ndarray, grid_thw: Sequence[Sequence[int]],
                   image_token_id: int, merge: int) -> np.ndarray:
    """[3, B, S] M-RoPE positions (0 at padding): text advances all axes by one;
    each image run spans its (t, h/m, w/m) grid and advances by max(h, w)/m."""

    b, s = input_ids.shape
    out = np.zeros((3, b, s), dtype=np.int64)
    grids = iter([tuple(int(v) for v in g) for g in grid_thw])
    for i in range(b):
        valid = np.nonzero(attention_mask[i])[0]
        ids = input_ids[i, valid]
        pos, cur, j = [], 0, 0
        while j < len(ids):
            if ids[j] == image_token_id:
                t, h, w = next(grids)
                gh, gw = h // merge, w // merge
                n = t * gh * gw
                tt = np.full(n, cur)
                hh = cur + np.repeat(np.arange(gh), gw * t)
                ww = cur + np.tile(np.arange(gw), gh * t)
                pos.append(np.stack([tt, hh, ww]))
                cur += max(h, w) // merge
                j += n
            else:
                k = j
                while k < len(ids) and ids[k] != image_token_id:
                    k += 1
                run = np.arange(cur, cur + k - j)
                pos.append(np.stack([run, run, run]))
                cur += k - j
                j = k
        if pos:
            out[:, i, valid] = np.concatenate(pos, 1)
    return out


@dataclass
class Qwen3VLBatch:
    """Token ids / mask plus optional flattened image patches and their grids."""

    input_ids: torch.Tensor
    attention_mask: torch.Tensor
    pixel_values: torch.Tensor | None = None       # [patches, C * T * p * p]
    image_grid_thw: torch.Tensor | None = None     # [images, 3]
    position_ids: torch.Tensor | None = None       # [3, B, S]
    packed: PackedTokens | None = None
    packed_positions: torch.Tensor | None = None   # [3, T] int32
    images_per_row: torch.Tensor | None = None     # [B] int64 on the host (set by prepare)

    def __post_init__(self) -> None:
        if self.input_ids.shape != self.attention_mask.shape:
            raise ValueError("attention_mask and input_ids must align")
        if (self.pixel_values is None) != (self.image_grid_thw is None):
            raise ValueError("pixel_values and image_grid_thw go together")

    @property
    def batch_size(self) -> int:
        return self.input_ids.shape[0]

    def prepare(self, config: Qwen3VLConfig) -> "Qwen3VLBatch":
        """Host-side packing and M-RoPE positions (call before moving to the device)."""

        ids = self.input_ids.cpu().numpy()
        mask = self.attention_mask.cpu().numpy().astype(bool)
        if self.position_ids is not None:
            pos = self.position_ids.cpu().numpy()
        else:
            grids = [] if self.image_grid_thw is None else self.image_grid_thw.tolist()
            pos = rope_positions(ids, mask, grids, config.image_token_id, config.vision.spatial_merge_size)
        packed = pack_tokens(self.input_ids, self.attention_mask)
        rows, cols = np.nonzero(mask)
        ppos = torch.from_numpy(np.ascontiguousarray(pos[:, rows, cols]).astype(np.int32))
        per_row = None
        if self.image_grid_thw is not None:
            # Images are consumed in order by the rows' image-token runs.
            merge = config.vision.spatial_merge_size ** 2
            tokens = [int(t * h * w) // merge for t, h, w in self.image_grid_thw.tolist()]
            counts = ((ids == config.image_token_id) & mask).sum(1)
            per_row = np.zeros(len(counts), dtype=np.int64)
            image = 0
            for r, need in enumerate(counts.tolist()):
                while need > 0 and image < len(tokens):
                    need -= tokens[image]
                    image += 1
                    per_row[r] += 1
            per_row = torch.from_numpy(per_row)
        return Qwen3VLBatch(self.input_ids, self.attention_mask, self.pixel_values, self.image_grid_thw,
                            torch.from_numpy(pos), packed, ppos, per_row)

    def rows(self, start: int, stop: int) -> "Qwen3VLBatch":
        """Rows [start, stop) with their images' patches (for chunked encoders such as GradCache)."""

        if self.packed is None or self.packed_positions is None:
            raise ValueError("call prepare() before slicing a Qwen3-VL batch")
        t0, t1 = int(self.packed.cu_host[start]), int(self.packed.cu_host[stop])
        pixels, grid, per_row = None, None, None
        if self.image_grid_thw is not None:
            if self.images_per_row is None:
                raise ValueError("prepare() did not record the images of each row")
            first = int(self.images_per_row[:start].sum())
            last = first + int(self.images_per_row[start:stop].sum())
            patches = (self.image_grid_thw[:, 0] * self.image_grid_thw[:, 1] * self.image_grid_thw[:, 2]).tolist()
            p0, p1 = int(sum(patches[:first])), int(sum(patches[:last]))
            pixels = self.pixel_values[p0:p1]
            grid = self.image_grid_thw[first:last]
            per_row = self.images_per_row[start:stop]
            if last == first:
                pixels, grid = None, None
        pos = None if self.position_ids is None else self.position_ids[:, start:stop]
        return Qwen3VLBatch(self.input_ids[start:stop], self.attention_mask[start:stop], pixels, grid, pos,
                            self.packed.rows(start, stop), self.packed_positions[:, t0:t1], per_row)

    def map_tensors(self, fn) -> "Qwen3VLBatch":
        opt = lambda t: None if t is None else fn(t)  # noqa: E731
        return Qwen3VLBatch(fn(self.input_ids), fn(self.attention_mask), opt(self.pixel_values),
                            self.image_grid_thw, opt(self.position_ids),
                            None if self.packed is None else self.packed.map_tensors(fn), opt(self.packed_positions),
                            self.images_per_row)


# ------------------------------------------------------------------ vision
def _normal(shape, std, g):
    return nn.Parameter(torch.randn(*shape, generator=g) * std)


class _Merger(nn.Module):
    def __init__(self, cfg: Qwen3VLVisionConfig, postshuffle: bool, g) -> None:
        super().__init__()
        wide = cfg.hidden_size * cfg.spatial_merge_size ** 2
        self.postshuffle = postshuffle
        norm_width = wide if postshuffle else cfg.hidden_size
        self.norm_w, self.norm_b = nn.Parameter(torch.ones(norm_width)), nn.Parameter(torch.zeros(norm_width))
        self.fc1_w, self.fc1_b = _normal((wide, wide), 0.02, g), nn.Parameter(torch.zeros(wide))
        self.fc2_w, self.fc2_b = _normal((cfg.out_hidden_size, wide), 0.02, g), nn.Parameter(torch.zeros(cfg.out_hidden_size))
        self.wide = wide

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.postshuffle:
            x = N.layer_norm(x.reshape(-1, self.wide), self.norm_w, self.norm_b, 1e-6)
        else:
            x = N.layer_norm(x, self.norm_w, self.norm_b, 1e-6).reshape(-1, self.wide)
        return N.linear(N.activation(N.linear(x, self.fc1_w, self.fc1_b), "gelu"), self.fc2_w, self.fc2_b)


class _VisionBlock(nn.Module):
    def __init__(self, cfg: Qwen3VLVisionConfig, g) -> None:
        super().__init__()
        h, i = cfg.hidden_size, cfg.intermediate_size
        self.n1_w, self.n1_b = nn.Parameter(torch.ones(h)), nn.Parameter(torch.zeros(h))
        self.qkv_w, self.qkv_b = _normal((3 * h, h), 0.02, g), nn.Parameter(torch.zeros(3 * h))
        self.proj_w, self.proj_b = _normal((h, h), 0.02, g), nn.Parameter(torch.zeros(h))
        self.n2_w, self.n2_b = nn.Parameter(torch.ones(h)), nn.Parameter(torch.zeros(h))
        self.fc1_w, self.fc1_b = _normal((i, h), 0.02, g), nn.Parameter(torch.zeros(i))
        self.fc2_w, self.fc2_b = _normal((h, i), 0.02, g), nn.Parameter(torch.zeros(h))

    def forward(self, h, seg, pos, axis, inv, cfg: Qwen3VLVisionConfig):
        x = N.layer_norm(h, self.n1_w, self.n1_b, 1e-6)
        a = N.qkv_attention(N.linear(x, self.qkv_w, self.qkv_b), seg, heads=cfg.num_heads, pos=pos, inv_freq=inv,
                            axis_of=axis)
        h = N.linear(a, self.proj_w, self.proj_b, residual=h)
        x = N.layer_norm(h, self.n2_w, self.n2_b, 1e-6)
        m = N.activation(N.linear(x, self.fc1_w, self.fc1_b), cfg.hidden_activation)
        return N.linear(m, self.fc2_w, self.fc2_b, residual=h)


class Qwen3VLVisionTower(nn.Module):
    def __init__(self, cfg: Qwen3VLVisionConfig, g) -> None:
        super().__init__()
        self.config = cfg
        self.patch_w = _normal((cfg.hidden_size, cfg.patch_dim), 0.02, g)
        self.patch_b = nn.Parameter(torch.zeros(cfg.hidden_size))
        self.pos_embed = _normal((cfg.num_position_embeddings, cfg.hidden_size), 0.02, g)
        self.blocks = nn.ModuleList(_VisionBlock(cfg, g) for _ in range(cfg.depth))
        self.merger = _Merger(cfg, False, g)
        self.deepstack = nn.ModuleList(_Merger(cfg, True, g) for _ in cfg.deepstack_visual_indexes)
        d = cfg.head_dimension
        quarter = d // 4
        inv = N.rope_inv_freq(d // 2, cfg.rope_theta)                # d/4 frequencies
        self.register_buffer("inv_freq", torch.cat([inv, inv]), persistent=False)
        self.register_buffer("axis_of", torch.tensor([0] * quarter + [1] * quarter, dtype=torch.int32),
                             persistent=False)

    def forward(self, pixels: torch.Tensor, grid_thw: Sequence[Sequence[int]], dtype: torch.dtype):
        cfg = self.config
        side = int(round(cfg.num_position_embeddings ** 0.5))
        rc, idx, wts, frames = vision_layout(grid_thw, cfg.spatial_merge_size, side)
        dev = pixels.device
        idx_t = torch.from_numpy(idx).to(dev)
        w_t = torch.from_numpy(wts).to(dev)
        pos_emb = (self.pos_embed[idx_t] * w_t[..., None]).sum(0).to(dtype)
        h = N.linear(pixels.to(dtype), self.patch_w, self.patch_b, residual=pos_emb)
        seg = N.Segments.from_lengths(frames, dev)
        pos = torch.from_numpy(rc).to(dev)
        deep = []
        for i, blk in enumerate(self.blocks):
            h = blk(h, seg, pos, self.axis_of, self.inv_freq, cfg)
            if i in cfg.deepstack_visual_indexes:
                deep.append(self.deepstack[cfg.deepstack_visual_indexes.index(i)](h))
        return self.merger(h), deep


# ------------------------------------------------------------------- model
class Qwen3VLEncoder(nn.Module):
    def __init__(self, config: Qwen3VLConfig, *, seed: int = 0, model_id: str = "representax/qwen3-vl",
                 revision: str = "random-init", compute_dtype: torch.dtype = torch.float32,
                 output_dimension: int | None = None) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.config = config
        self.text = Qwen3TextTower(config.text, g)
        self.vision = Qwen3VLVisionTower(config.vision, g)
        self.compute_dtype = compute_dtype
        out = output_dimension or config.text.hidden_size
        self.metadata = EncoderMetadata(model_id=model_id, revision=revision, output_dimension=out,
                                        routes=frozenset(Route), modalities=frozenset({Modality.TEXT, Modality.IMAGE}))

    @staticmethod
    def make_batch(*, input_ids, attention_mask, token_type_ids=None, pixel_values=None, image_grid_thw=None):
        t = lambda v: None if v is None else torch.as_tensor(v)  # noqa: E731
        return Qwen3VLBatch(t(input_ids).long(), t(attention_mask).long(), t(pixel_values), t(image_grid_thw))

    def packed_hidden(self, inputs: Qwen3VLBatch, *, all_layers: bool = False):
        dtype = active_compute_dtype(self.compute_dtype)
        dev = self.text.embed_tokens.device
        if inputs.packed is None:
            inputs = inputs.prepare(self.config)
        pk = inputs.packed.map_tensors(lambda t: t.to(dev, non_blocking=True))
        seg = N.Segments([int(v) for v in pk.cu_host.tolist()], pk.cu_seqlens.to(dev, torch.int32))
        pos = inputs.packed_positions.to(dev)
        emb = self.text.token_embeddings(pk.input_ids, dtype)
        deep, rows = (), None
        if inputs.pixel_values is not None:
            merged, deep = self.vision(inputs.pixel_values.to(dev), inputs.image_grid_thw.tolist(), dtype)
            rows = torch.nonzero(pk.input_ids == self.config.image_token_id).flatten()
            if rows.numel() != merged.shape[0]:
                raise ValueError(f"{rows.numel()} image tokens but {merged.shape[0]} visual features")
            emb = emb.index_copy(0, rows, merged.to(dtype))
        return self.text(emb, seg, pos, deepstack=deep, visual_rows=rows, all_layers=all_layers), seg

    def hidden_states(self, inputs: Qwen3VLBatch, *, generator=None) -> torch.Tensor:
        h, _ = self.packed_hidden(inputs)
        m = inputs.attention_mask.to(h.device).bool()
        out = h.new_zeros(m.shape + (h.shape[-1],))
        out[m] = h
        return out

    def _pool(self, h, seg):
        v = h[last_token_rows(seg), : self.metadata.output_dimension].float()
        return v / v.norm(dim=-1, keepdim=True).clamp_min(1e-12)

    def encode(self, inputs: Qwen3VLBatch, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        h, seg = self.packed_hidden(inputs)
        return self._pool(h, seg)

    def encode_layers(self, inputs: Qwen3VLBatch, *, route: Route = Route.GENERIC, generator=None):
        states, seg = self.packed_hidden(inputs, all_layers=True)
        return torch.stack([self._pool(s, seg) for s in states])


class Qwen3VLReranker(nn.Module):
    """Relevance = sigmoid(last hidden . (E[true] - E[false])) with the tied embedding rows."""

    def __init__(self, model: Qwen3VLEncoder, true_token_id: int = 9693, false_token_id: int = 2152) -> None:
        super().__init__()
        self.model = model
        self.true_token_id, self.false_token_id = true_token_id, false_token_id
        self.metadata = model.metadata

    def score(self, inputs: Qwen3VLBatch) -> torch.Tensor:
        h, seg = self.model.packed_hidden(inputs)
        last = h[last_token_rows(seg)].float()
        emb = self.model.text.embed_tokens
        direction = (emb[self.true_token_id] - emb[self.false_token_id]).float()
        return torch.sigmoid(last @ direction)


# -------------------------------------------------------------- checkpoint
def _vision_state(v: Qwen3VLVisionTower, p: str) -> dict[str, torch.Tensor]:
    cfg = v.config
    out = {p + "patch_embed.proj.weight": v.patch_w.detach().reshape(
        cfg.hidden_size, cfg.in_channels, cfg.temporal_patch_size, cfg.patch_size, cfg.patch_size),
        p + "patch_embed.proj.bias": v.patch_b.detach(), p + "pos_embed.weight": v.pos_embed.detach()}
    for i, b in enumerate(v.blocks):
        q = f"{p}blocks.{i}."
        for attr, name in (("n1", "norm1"), ("n2", "norm2"), ("qkv", "attn.qkv"), ("proj", "attn.proj"),
                           ("fc1", "mlp.linear_fc1"), ("fc2", "mlp.linear_fc2")):
            out[q + name + ".weight"] = getattr(b, attr + "_w").detach()
            out[q + name + ".bias"] = getattr(b, attr + "_b").detach()
    for prefix, m in [(p + "merger.", v.merger)] + [(f"{p}deepstack_merger_list.{i}.", d)
                                                  for i, d in enumerate(v.deepstack)]:
        for attr, name in (("norm", "norm"), ("fc1", "linear_fc1"), ("fc2", "linear_fc2")):
            out[prefix + name + ".weight"] = getattr(m, attr + "_w").detach()
            out[prefix + name + ".bias"] = getattr(m, attr + "_b").detach()
    return out


class Qwen3VLCheckpointAdapter:
    TEXT_PREFIXES = ("model.language_model.", "language_model.")
    VISION_PREFIXES = ("model.visual.", "visual.")

    @classmethod
    def state_dict(cls, model: Qwen3VLEncoder) -> dict[str, torch.Tensor]:
        out = qwen3_tower_state(model.text, "model.language_model.")
        out.update(_vision_state(model.vision, "model.visual."))
        return {k: v.float().cpu().contiguous() for k, v in out.items()}

    @classmethod
    def from_state_dict(cls, model: Qwen3VLEncoder, tensors: Mapping[str, torch.Tensor]) -> Qwen3VLEncoder:
        tp = next((p for p in cls.TEXT_PREFIXES if p + "embed_tokens.weight" in tensors), None)
        vp = next((p for p in cls.VISION_PREFIXES if p + "pos_embed.weight" in tensors), None)
        if tp is None or vp is None:
            raise KeyError("checkpoint lacks the Qwen3-VL text or vision tower")
        load_qwen3_tower(model.text, tensors, tp)
        want = _vision_state(model.vision, vp)
        params = dict(_vision_params(model.vision, vp))
        with torch.no_grad():
            for name, ref in want.items():
                target, shape = params[name]
                target.copy_(tensors[name].reshape(shape))
        return model

    @classmethod
    def load(cls, path: str | os.PathLike, *, compute_dtype: torch.dtype = torch.float32, **kwargs) -> Qwen3VLEncoder:
        path = Path(path)
        cfg = Qwen3VLConfig.from_hf_config(load_hf_config(path))
        kwargs.setdefault("model_id", path.name)
        kwargs.setdefault("revision", "local")
        model = Qwen3VLEncoder(cfg, compute_dtype=compute_dtype, **kwargs)
        names = set()
        for tp in cls.TEXT_PREFIXES:
            names |= set(qwen3_tower_state(model.text, tp))
        for vp in cls.VISION_PREFIXES:
            names |= set(_vision_state(model.vision, vp))
        return cls.from_state_dict(model, load_safetensor_subset(path, names))

    @classmethod
    def save(cls, model: Qwen3VLEncoder, path: str | os.PathLike) -> None:
        path = Path(path)
        path.mkdir(parents=True, exist_ok=True)
        with open(path / "config.json", "w") as handle:
            json.dump(model.config.to_hf_config(), handle, indent=2, sort_keys=True)
        save_safetensors(cls.state_dict(model), path / "model.safetensors")


def _vision_params(v: Qwen3VLVisionTower, p: str):
    yield p + "patch_embed.proj.weight", (v.patch_w, v.patch_w.shape)
    yield p + "patch_embed.proj.bias", (v.patch_b, v.patch_b.shape)
    yield p + "pos_embed.weight", (v.pos_embed, v.pos_embed.shape)
    for i, b in enumerate(v.blocks):
        q = f"{p}blocks.{i}."
        for attr, name in (("n1", "norm1"), ("n2", "norm2"), ("qkv", "attn.qkv"), ("proj", "attn.proj"),
                           ("fc1", "mlp.linear_fc1"), ("fc2", "mlp.linear_fc2")):
            for kind in ("w", "b"):
                t = getattr(b, f"{attr}_{kind}")
                yield q + name + (".weight" if kind == "w" else ".bias"), (t, t.shape)
    for prefix, m in [(p + "merger.", v.merger)] + [(f"{p}deepstack_merger_list.{i}.", d)
                                                  for i, d in enumerate(v.deepstack)]:
        for attr, name in (("norm", "norm"), ("fc1", "linear_fc1"), ("fc2", "linear_fc2")):
            for kind in ("w", "b"):
                t = getattr(m, f"{attr}_{kind}")
                yield prefix + name + (".weight" if kind == "w" else ".bias"), (t, t.shape)


def build_qwen3_vl(*, seed: int = 0, compute_dtype: str = "float32", **config) -> Qwen3VLEncoder:
    return Qwen3VLEncoder(Qwen3VLConfig(**config), seed=seed, compute_dtype=getattr(torch, compute_dtype))


__all__ = ["Qwen3VLBatch", "Qwen3VLCheckpointAdapter", "Qwen3VLConfig", "Qwen3VLEncoder", "Qwen3VLReranker",
           "Qwen3VLVisionConfig", "Qwen3VLVisionTower", "build_qwen3_vl", "rope_positions", "vision_layout"]
