from .checkpoint import BertCheckpointAdapter, bert_weight_names
from .config import BertConfig
from .model import BertBatch, BertEmbeddings, BertEncoder, BertLayer

__all__ = ["BertBatch", "BertCheckpointAdapter", "BertConfig", "BertEmbeddings", "BertEncoder", "BertLayer",
           "bert_weight_names"]
