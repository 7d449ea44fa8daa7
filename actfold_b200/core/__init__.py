"""Branch Folding engine (drop-in for ``actfold.core``)."""

from actfold_b200.core.activation_cache import ActivationCache
from actfold_b200.core.cache_factory import ActivationCacheType, make_activation_cache
from actfold_b200.core.chunked_cache import ChunkedActivationCache
from actfold_b200.core.folded_transformer import FoldedTransformerLayer
from actfold_b200.core.folding_context import FOLDING_CONTEXT, folding_scope
from actfold_b200.core.folding_scheduler import FoldingScheduler
from actfold_b200.core.fused_ops import gather_cached_activations, merge_stable_divergent
from actfold_b200.core.model_wrapper import FoldedModel
from actfold_b200.core.similarity_gate import SimilarityGate

__all__ = [
    "ActivationCache",
    "ActivationCacheType",
    "ChunkedActivationCache",
    "FOLDING_CONTEXT",
    "FoldedModel",
    "FoldedTransformerLayer",
    "FoldingScheduler",
    "SimilarityGate",
    "folding_scope",
    "gather_cached_activations",
    "make_activation_cache",
    "merge_stable_divergent",
]
