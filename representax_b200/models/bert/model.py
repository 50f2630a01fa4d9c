"""BERT encoder (post-LN) with a native packed path and a PyTorch reference path.

Parity: ``BertEmbeddings``, ``BertLayer``, ``BertTower`` and ``BertEncoder`` of
src/representax/models/bert/model.py:31-591 (embeddings with padding-row
gradient suppression, QKV/O attention, GELU MLP, mean pooling + L2 in
``encode``, tanh pooler, layerwise ``encode_layers``).

The query/key/value projections are held as one fused ``[3H, H]`` parameter
(split back into Hugging Face names by the checkpoint adapter) so the native
path runs them as one tcgen05 GEMM.

Execution: when the batch is packed and on a CUDA device, the compute dtype is
bf16 and dropout is inactive, every op runs in the sm_100a extension on packed
tokens (no padding FLOPs). Otherwise the padded PyTorch reference path runs
(CPU tests, fp32 policies, dropout-active training).
"""

from __future__ import annotations

import torch
from torch import nn

from representax_b200.core import EncoderMetadata, Modality, Route
from representax_b200.models import components as cmp
from representax_b200.models.text_batch import TokenBatch
from representax_b200.precision import active_compute_dtype

from .config import BertConfig

BertBatch = TokenBatch


def _param(t: torch.Tensor) -> nn.Parameter:
    return nn.Parameter(t)


class BertEmbeddings(nn.Module):
    def __init__(self, config: BertConfig, generator: torch.Generator | None = None) -> None:
        super().__init__()
        r = config.initializer_range
        h = config.hidden_size
        word = torch.randn(config.vocab_size, h, generator=generator) * r
        word[config.pad_token_id] = 0
        self.word = _param(word)
        self.position = _param(torch.randn(config.max_position_embeddings, h, generator=generator) * r)
        self.token_type = _param(torch.randn(config.type_vocab_size, h, generator=generator) * r)
        self.norm_weight = _param(torch.ones(h))
        self.norm_bias = _param(torch.zeros(h))


class BertLayer(nn.Module):
    def __init__(self, config: BertConfig, generator: torch.Generator | None = None) -> None:
        super().__init__()
        h, f, r = config.hidden_size, config.intermediate_size, config.initializer_range
        self.qkv_weight = _param(torch.randn(3 * h, h, generator=generator) * r)
        self.qkv_bias = _param(torch.zeros(3 * h))
        self.out_weight = _param(torch.randn(h, h, generator=generator) * r)
        self.out_bias = _param(torch.zeros(h))
        self.attn_norm_weight = _param(torch.ones(h))
        self.attn_norm_bias = _param(torch.zeros(h))
        self.ffn_in_weight = _param(torch.randn(f, h, generator=generator) * r)
        self.ffn_in_bias = _param(torch.zeros(f))
        self.ffn_out_weight = _param(torch.randn(h, f, generator=generator) * r)
        self.ffn_out_bias = _param(torch.zeros(h))
        self.out_norm_weight = _param(torch.ones(h))
        self.out_norm_bias = _param(torch.zeros(h))


class BertEncoder(nn.Module):
    """Native bidirectional BERT plus representation pooling."""

    def __init__(self, config: BertConfig, *, seed: int = 0, model_id: str = "representax/bert",
                 revision: str = "random-init", compute_dtype: torch.dtype = torch.float32,
                 pooling: str = "mean", normalize: bool = True) -> None:
        super().__init__()
        generator = torch.Generator().manual_seed(seed)
        self.config = config
        self.embeddings = BertEmbeddings(config, generator)
        self.layers = nn.ModuleList(BertLayer(config, generator) for _ in range(config.num_hidden_layers))
        self.pooler_weight = _param(torch.randn(config.hidden_size, config.hidden_size, generator=generator)
                                    * config.initializer_range)
        self.pooler_bias = _param(torch.zeros(config.hidden_size))
        self.metadata = EncoderMetadata(
            model_id=model_id,
            revision=revision,
            output_dimension=config.hidden_size,
            routes=frozenset(Route),
            modalities=frozenset({Modality.TEXT}),
        )
        self.compute_dtype = compute_dtype
        self.pooling = pooling
        self.normalize = normalize

    @classmethod
    def init(cls, config: BertConfig, **kwargs) -> "BertEncoder":
        return cls(config, **kwargs)

    @staticmethod
    def make_batch(*, input_ids, attention_mask, token_type_ids=None) -> TokenBatch:
        return TokenBatch.from_arrays(input_ids=input_ids, attention_mask=attention_mask,
                                      token_type_ids=token_type_ids)

    # ------------------------------------------------------------ dispatch
    def _dtype(self) -> torch.dtype:
        return active_compute_dtype(self.compute_dtype)

    def _native(self, batch: TokenBatch, generator) -> bool:
        packed = batch.packed
        if packed is None or not packed.input_ids.is_cuda:
            return False
        if self._dtype() != torch.bfloat16 or self.config.head_dimension != 64:
            return False
        if self.config.hidden_activation != "gelu":
            return False
        from representax_b200.ops import _ext

        _ext.ext()  # raises loudly if the extension is missing on a GPU box
        return True

    # ------------------------------------------------------------ native path
    def _native_hidden(self, batch: TokenBatch, all_layers: bool = False, generator=None):
        from representax_b200.ops import functional as Fn

        cfg = self.config
        pk = batch.packed
        packed = Fn.Packed(cu_seqlens=pk.cu_seqlens, max_len=pk.max_len, total=pk.total)
        e = self.embeddings
        # Dropout masks come from counter-based Philox streams keyed by the
        # generator's seed, so GradCache replays reproduce them exactly.
        p_h, p_a = cfg.hidden_dropout_probability, cfg.attention_dropout_probability
        seed = generator.initial_seed() if generator is not None and (p_h > 0 or p_a > 0) else None

        def drop(site: int):
            return None if seed is None else Fn.Dropout(seed, site, p_a, p_h)

        h = Fn.embed_layer_norm(pk.input_ids, pk.position_ids, pk.token_type_ids, e.word, e.position,
                                e.token_type, e.norm_weight, e.norm_bias, cfg.norm_epsilon, cfg.pad_token_id,
                                dropout=drop(0))
        states = [h] if all_layers else None
        fused_bias = seed is None or p_h == 0  # norm-fused bias gradient needs the undropped gradient
        for i, layer in enumerate(self.layers):
            site = 16 * (i + 1)
            s1 = Fn.attention_block(h, layer.qkv_weight, layer.qkv_bias, layer.out_weight, layer.out_bias,
                                    packed, heads=cfg.num_attention_heads, out_bias_grad_fused=fused_bias,
                                    dropout=drop(site))
            h1 = Fn.layer_norm(s1, layer.attn_norm_weight, layer.attn_norm_bias, cfg.norm_epsilon,
                               producer_bias=layer.out_bias if fused_bias else None)
            s2 = Fn.mlp_block(h1, layer.ffn_in_weight, layer.ffn_in_bias, layer.ffn_out_weight, layer.ffn_out_bias,
                              out_bias_grad_fused=fused_bias, dropout=drop(site))
            h = Fn.layer_norm(s2, layer.out_norm_weight, layer.out_norm_bias, cfg.norm_epsilon,
                              producer_bias=layer.ffn_out_bias if fused_bias else None)
            if all_layers:
                states.append(h)
        return (h, packed) if not all_layers else (states, packed)

    # ------------------------------------------------------------ reference path
    def _reference_embeddings(self, batch: TokenBatch, generator, dtype):
        cfg = self.config
        e = self.embeddings
        seq = batch.attention_mask.shape[1]
        if seq > cfg.max_position_embeddings:
            raise ValueError("sequence exceeds max_position_embeddings")
        if batch.input_ids is None:
            hidden = batch.inputs_embeds.to(torch.float32)
        else:
            ids = batch.input_ids.long()
            hidden = e.word[ids]
            pad = (ids == cfg.pad_token_id)[..., None]
            hidden = torch.where(pad, hidden.detach(), hidden)
        pos_ids = batch.position_ids
        if pos_ids is None:
            pos_ids = torch.arange(seq, device=batch.attention_mask.device)[None, :]
        types = batch.token_type_ids
        if types is None:
            types = torch.zeros_like(batch.attention_mask, dtype=torch.long)
        hidden = hidden + e.position[pos_ids.long()] + e.token_type[types.long()]
        hidden = cmp.layer_norm(hidden, e.norm_weight, e.norm_bias, cfg.norm_epsilon)
        hidden = cmp.dropout(hidden, cfg.hidden_dropout_probability, generator)
        return hidden.to(dtype)

    def _reference_layer(self, layer: BertLayer, hidden, mask, generator, dtype):
        cfg = self.config
        b, s, h = hidden.shape
        heads = cfg.num_attention_heads
        w = lambda p: p.to(dtype)  # noqa: E731
        qkv = torch.nn.functional.linear(hidden, w(layer.qkv_weight), w(layer.qkv_bias))
        q, k, v = qkv.split(h, dim=-1)
        shape = (b, s, heads, cfg.head_dimension)
        att = cmp.dot_product_attention(q.reshape(shape), k.reshape(shape), v.reshape(shape), key_mask=mask,
                                        dropout_p=cfg.attention_dropout_probability, generator=generator)
        att = torch.nn.functional.linear(att.reshape(b, s, h), w(layer.out_weight), w(layer.out_bias))
        att = cmp.dropout(att, cfg.hidden_dropout_probability, generator)
        hidden = cmp.layer_norm(hidden + att, w(layer.attn_norm_weight), w(layer.attn_norm_bias), cfg.norm_epsilon)
        mid = cmp.activate(torch.nn.functional.linear(hidden, w(layer.ffn_in_weight), w(layer.ffn_in_bias)),
                           cfg.hidden_activation)
        out = torch.nn.functional.linear(mid, w(layer.ffn_out_weight), w(layer.ffn_out_bias))
        out = cmp.dropout(out, cfg.hidden_dropout_probability, generator)
        return cmp.layer_norm(hidden + out, w(layer.out_norm_weight), w(layer.out_norm_bias), cfg.norm_epsilon)

    def hidden_states(self, inputs: TokenBatch, *, generator=None) -> torch.Tensor:
        """Padded ``[batch, sequence, hidden]`` final hidden states."""

        if not isinstance(inputs, TokenBatch):
            raise TypeError("BERT inputs must be TokenBatch")
        if self._native(inputs, generator):
            h, _ = self._native_hidden(inputs, generator=generator)
            return _unpack(h, inputs)
        dtype = self._dtype()
        mask = inputs.attention_mask.bool()
        hidden = self._reference_embeddings(inputs, generator, dtype)
        for layer in self.layers:
            hidden = self._reference_layer(layer, hidden, mask, generator, dtype)
        return hidden

    def hidden_states_by_layer(self, inputs: TokenBatch, *, generator=None) -> torch.Tensor:
        dtype = self._dtype()
        mask = inputs.attention_mask.bool()
        hidden = self._reference_embeddings(inputs, generator, dtype)
        states = [hidden]
        for layer in self.layers:
            hidden = self._reference_layer(layer, hidden, mask, generator, dtype)
            states.append(hidden)
        return torch.stack(states)

    def encode(self, inputs: TokenBatch, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        del route
        if not isinstance(inputs, TokenBatch):
            raise TypeError("BERT inputs must be TokenBatch")
        if self._native(inputs, generator):
            from representax_b200.ops import functional as Fn

            h, packed = self._native_hidden(inputs, generator=generator)
            return Fn.pool(h, packed, self.pooling, self.normalize)
        hidden = self.hidden_states(inputs, generator=generator)
        pooled = self._pool_reference(hidden, inputs.attention_mask)
        return cmp.l2_normalize(pooled) if self.normalize else pooled

    def _pool_reference(self, hidden, mask):
        if self.pooling == "mean":
            return cmp.mean_pool(hidden, mask)
        if self.pooling in {"cls", "first"}:
            return hidden[:, 0].float()
        if self.pooling in {"last", "lasttoken"}:
            return cmp.last_token_pool(hidden, mask)
        raise ValueError(f"unknown pooling {self.pooling!r}")

    def encode_layers(self, inputs: TokenBatch, *, route: Route = Route.GENERIC, generator=None) -> torch.Tensor:
        del route
        if inputs.packed is not None and self._native(inputs, generator):
            from representax_b200.ops import functional as Fn

            states, packed = self._native_hidden(inputs, all_layers=True, generator=generator)
            return torch.stack([Fn.pool(s, packed, self.pooling, True) for s in states])
        hidden = self.hidden_states_by_layer(inputs, generator=generator)
        pooled = torch.stack([self._pool_reference(h, inputs.attention_mask) for h in hidden])
        return cmp.l2_normalize(pooled)

    def pooler_output(self, inputs: TokenBatch, *, generator=None) -> torch.Tensor:
        hidden = self.hidden_states(inputs, generator=generator)
        return torch.tanh(torch.nn.functional.linear(hidden[:, 0].float(), self.pooler_weight, self.pooler_bias))

    def fused_parameter_groups(self):
        """Parameter name groups the flat store keeps adjacent (none needed: QKV is fused)."""

        return []


def _unpack(h: torch.Tensor, batch: TokenBatch) -> torch.Tensor:
    """Scatter packed rows back to a zero-padded [batch, sequence, hidden] tensor."""

    mask = batch.attention_mask.to(h.device).bool()
    out = torch.zeros(mask.shape + (h.shape[-1],), dtype=h.dtype, device=h.device)
    out[mask] = h
    return out


__all__ = ["BertBatch", "BertEmbeddings", "BertEncoder", "BertLayer"]
