"""rustwood_b200: B200-native oblivious-tree boosting hot path (librwgpu) with a host
mirror of rustwood's Booster/Config API.

The GPU library is loaded on import; there is no CPU fallback for any GPU entry point.
"""
from .config import Config  # noqa: F401
from . import _native  # noqa: F401  (loads librwgpu.so or raises)
from .booster import (Booster, Context, Dataset, base_score, compute_boundaries,  # noqa: F401
                      fit_dataset, train_params)

__all__ = ["Config", "Booster", "Context", "Dataset", "compute_boundaries", "base_score",
           "fit_dataset", "train_params"]
