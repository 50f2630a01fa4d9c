"""Native encoders, compositions and host processors.

Parity: the re-exports of src/representax/models/__init__.py.
"""

from .adapters import (
    QuantizedLoRAWeight,
    apply_quantized_lora,
    lora_parameter_filter,
    merge_quantized_lora,
    pack_int4_rows,
    unpack_int4_rows,
)
from .bert import BertBatch, BertCheckpointAdapter, BertConfig, BertEncoder, build_bert
from .composition import DenoisingAutoEncoder, EncoderPair, PairClassifier, TokenReconstructionDecoder
from .dense import DenseEncoder
from .mpnet import MPNetCheckpointAdapter, MPNetConfig, MPNetEncoder, build_mpnet
from .processing import (
    Processor,
    make_audio_processor,
    make_image_processor,
    make_media_processor,
    make_text_processor,
    make_video_processor,
    select_static_shape_bucket,
)
from .sentence import (
    POOLING_MODES,
    SentenceBatch,
    SentenceDense,
    SentenceEncoder,
    SentenceNormalize,
    SentencePooling,
)
from .text_batch import PackedTokens, TokenBatch, pack_tokens

__all__ = [
    "BertBatch", "BertCheckpointAdapter", "BertConfig", "BertEncoder", "DenoisingAutoEncoder", "DenseEncoder",
    "EncoderPair", "MPNetCheckpointAdapter", "MPNetConfig", "MPNetEncoder", "POOLING_MODES", "PackedTokens",
    "PairClassifier", "Processor", "QuantizedLoRAWeight", "SentenceBatch", "SentenceDense", "SentenceEncoder",
    "SentenceNormalize", "SentencePooling", "TokenBatch", "TokenReconstructionDecoder", "apply_quantized_lora",
    "build_bert", "build_mpnet", "lora_parameter_filter", "make_audio_processor", "make_image_processor",
    "make_media_processor", "make_text_processor", "make_video_processor", "merge_quantized_lora", "pack_int4_rows",
    "pack_tokens", "select_static_shape_bucket", "unpack_int4_rows",
]
