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
from .clip import CLIPBatch, CLIPCheckpointAdapter, CLIPConfig, CLIPEncoder, build_clip
from .jina_v5 import JinaV5CheckpointAdapter, JinaV5TextEncoder, load_jina_v5_small_text_encoder
from .modernvbert import (
    ModernVBERTBatch,
    ModernVBERTCheckpointAdapter,
    ModernVBERTConfig,
    ModernVBERTEncoder,
    ModernVBERTTextEncoder,
    build_modernvbert,
)
from .qwen2_5_omni import Qwen2_5OmniBatch, Qwen2_5OmniCheckpointAdapter, Qwen2_5OmniConfig, Qwen2_5OmniEncoder
from .qwen3 import Qwen3TextConfig, Qwen3TextTower
from .qwen3_vl import Qwen3VLBatch, Qwen3VLCheckpointAdapter, Qwen3VLConfig, Qwen3VLEncoder, Qwen3VLReranker
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
    "CLIPBatch", "CLIPCheckpointAdapter", "CLIPConfig", "CLIPEncoder", "JinaV5CheckpointAdapter", "JinaV5TextEncoder",
    "ModernVBERTBatch", "ModernVBERTCheckpointAdapter", "ModernVBERTConfig", "ModernVBERTEncoder",
    "ModernVBERTTextEncoder", "Qwen2_5OmniBatch", "Qwen2_5OmniCheckpointAdapter", "Qwen2_5OmniConfig",
    "Qwen2_5OmniEncoder", "Qwen3TextConfig", "Qwen3TextTower", "Qwen3VLBatch", "Qwen3VLCheckpointAdapter",
    "Qwen3VLConfig", "Qwen3VLEncoder", "Qwen3VLReranker", "build_clip", "build_modernvbert",
    "load_jina_v5_small_text_encoder",
    "BertBatch", "BertCheckpointAdapter", "BertConfig", "BertEncoder", "DenoisingAutoEncoder", "DenseEncoder",
    "EncoderPair", "MPNetCheckpointAdapter", "MPNetConfig", "MPNetEncoder", "POOLING_MODES", "PackedTokens",
    "PairClassifier", "Processor", "QuantizedLoRAWeight", "SentenceBatch", "SentenceDense", "SentenceEncoder",
    "SentenceNormalize", "SentencePooling", "TokenBatch", "TokenReconstructionDecoder", "apply_quantized_lora",
    "build_bert", "build_mpnet", "lora_parameter_filter", "make_audio_processor", "make_image_processor",
    "make_media_processor", "make_text_processor", "make_video_processor", "merge_quantized_lora", "pack_int4_rows",
    "pack_tokens", "select_static_shape_bucket", "unpack_int4_rows",
]
