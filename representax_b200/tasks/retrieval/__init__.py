from .batch import ProcessLocalRetrievalBatch, RetrievalBatch, RetrievalCollator, retrieval_batch
from .config import MNRConfig, RetrievalConfig
from .mnr import MNRLossTerms, MNRTask, mnr_loss_terms

__all__ = [
    "MNRConfig",
    "MNRLossTerms",
    "MNRTask",
    "ProcessLocalRetrievalBatch",
    "RetrievalBatch",
    "RetrievalCollator",
    "RetrievalConfig",
    "mnr_loss_terms",
    "retrieval_batch",
]
