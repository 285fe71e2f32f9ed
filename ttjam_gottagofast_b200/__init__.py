"""B200 (sm_100a) implementation of the reference's pre-norm Transformer forward.

Public surface, mirroring the reference contract (torch_transformer_benchmark.py):
`TransformerConfig`, `UserOptimizedTransformer`, `generate_random_case`,
`compare_outputs`, `copy_model_weights`, `derive_user_optimized` (the
contract's `UserOptimizedTransformer(BaselineTransformer)` over a caller's
base class), and the harness candidate hooks
`build_model` / `load_from_baseline`.
"""
from .config import TransformerConfig, WORKLOADS, MODEL_SEED, TIMING_DATA_SEED
from .contract import generate_random_case, compare_outputs, AccuracyResult, RTOL, ATOL
from .model import UserOptimizedTransformer, derive_user_optimized
from .candidate import build_model, load_from_baseline, copy_model_weights

__all__ = [
    "TransformerConfig", "WORKLOADS", "MODEL_SEED", "TIMING_DATA_SEED",
    "generate_random_case", "compare_outputs", "AccuracyResult", "RTOL", "ATOL",
    "UserOptimizedTransformer", "derive_user_optimized", "build_model", "load_from_baseline", "copy_model_weights",
]
