"""B200 (sm_100a) forward pass of the TikTok TechJam 2026 Track 3 Transformer encoder stack.

Drop-in for the reference benchmark's `UserOptimizedTransformer` slot: same constructor, weight
names, forward signature and mask semantics; computation in hand-written tcgen05/TMA CUDA kernels
(libb200tx.so, C-ABI in include/b200tx.h).
"""

from .cases import BASELINE_CONFIGS, TransformerConfig, Workload, config_from
from .correctness import AccuracyResult, GateResult, baseline_gate, compare_outputs
from .models import UserOptimizedTransformer, copy_model_weights

__all__ = [
    "AccuracyResult",
    "BASELINE_CONFIGS",
    "GateResult",
    "TransformerConfig",
    "UserOptimizedTransformer",
    "Workload",
    "baseline_gate",
    "compare_outputs",
    "config_from",
    "copy_model_weights",
]
