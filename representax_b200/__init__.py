"""representax_b200: representation learning on B200 (sm_100a).

PyTorch is the framework layer; the hot ops are hand-written sm_100a CUDA
kernels in ``representax_b200._C``; multi-GPU paths run one process per GPU
with NCCL plus peer-memory kernels over NVLink / NVSwitch.

Parity: the public surface of src/representax/__init__.py.
"""

from . import data, evaluation, integrations, models, planning, tasks, train
from .config import JobConfig, PrecisionConfig, QuantizedLoRAConfig
from .core import (
    BoundEncoder,
    Encoder,
    EncoderMetadata,
    LossOutput,
    Modality,
    Route,
    Task,
    bind,
    encode,
    evaluate_loss,
)
from .export import InferenceBundle, export_inference_bundle, load_inference_bundle
from .inference import TextEmbeddingModel, embed
from .models import Processor
from .precision import PrecisionPolicy

__all__ = [
    "BoundEncoder", "Encoder", "EncoderMetadata", "InferenceBundle", "JobConfig", "LossOutput", "Modality",
    "PrecisionConfig", "PrecisionPolicy", "Processor", "QuantizedLoRAConfig", "Route", "Task", "TextEmbeddingModel",
    "bind", "data", "embed", "encode", "evaluate_loss", "evaluation", "export_inference_bundle", "integrations",
    "load_inference_bundle", "models", "planning", "tasks", "train",
]
