from .checkpoint import BertCheckpointAdapter, bert_weight_names
from .config import BertConfig
from .model import BertBatch, BertEmbeddings, BertEncoder, BertLayer

__all__ = ["BertBatch", "BertCheckpointAdapter", "BertConfig", "BertEmbeddings", "BertEncoder", "BertLayer",
           "bert_weight_names"]


def build_bert(*, seed: int = 0, compute_dtype: str = "float32", model_id: str = "representax/bert",
               pooling: str = "mean", **config):
    """Dotted-target factory for job files: ``BertConfig`` fields as parameters."""

    import torch

    return BertEncoder(BertConfig(**config), seed=seed, model_id=model_id,
                       compute_dtype=getattr(torch, compute_dtype), pooling=pooling)


__all__.append("build_bert")
