"""scao_b200 -- B200-native (sm_100a) implementation of the SCAO optimizer step.

Drop-in for ``scao.SCAO`` of whispering3/scao: same constructor, ``step``,
callbacks and checkpoint schema; the step runs as batched CUDA kernels from
``libscao_b200.so`` (C ABI in include/scao_b200.h).
"""
from .optimizer import SCAO
from . import logging as scao_logging
from .sparse_preconditioner import SparsePreconditioner
from .presets import scao_sub1b, scao_1b, scao_3b, scao_7b, scao_40b, scao_125b
from .utils import (adaptive_rank, low_rank_matrix_power_neg_quarter, matrix_power_neg_quarter,
                    newton_schulz_root_inv)

__version__ = "0.1.0"

__all__ = ["SCAO", "SparsePreconditioner", "scao_logging", "adaptive_rank", "matrix_power_neg_quarter", "newton_schulz_root_inv",
           "low_rank_matrix_power_neg_quarter", "scao_sub1b", "scao_1b", "scao_3b", "scao_7b",
           "scao_40b", "scao_125b", "__version__"]
