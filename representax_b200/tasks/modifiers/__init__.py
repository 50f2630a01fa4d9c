from .config import AdaptiveLayerModifierConfig, Matryoshka2dModifierConfig, MatryoshkaModifierConfig
from .task import AdaptiveLayerTask, Matryoshka2dTask, MatryoshkaTask

__all__ = ["AdaptiveLayerModifierConfig", "AdaptiveLayerTask", "Matryoshka2dModifierConfig", "Matryoshka2dTask",
           "MatryoshkaModifierConfig", "MatryoshkaTask"]
