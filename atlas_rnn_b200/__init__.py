"""atlas_rnn_b200: B200-native memory-update hot path of Atlas-RNN.

Public API mirrors atlas_pytorch/rnn_memory.py (RNNMemoryCell, OmegaRNNMemoryCell,
RNNMemory, OmegaRNNMemory, RNNMemState, state_detach, PolynomialFeatureMap), the LMM
language model of atlas_pytorch/rnn_transformer.py (RNNMemoryTransformer with
block_type 'lmm', LMMBlock, LongTermMemoryModel), plus the
functional ``memory_recurrence``, the GPU drop-in for the third-party
``assoc_scan.AssocScan`` (``AssocScan``, ``assoc_scan``) and the multi-GPU helpers in ``parallel``.
"""
from .ops import memory_recurrence, MemoryRecurrenceFn
from ._lib import check_device_status
from .scan import AssocScan, assoc_scan
from .omega_store import omega_store_update
from .affine_scan import affine_associative_scan
from .rnn_memory import (RNNMemState, state_detach, PolynomialFeatureMap, MultiheadRMSNorm,
                         RNNMemoryCell, OmegaRNNMemoryCell, RNNMemory, OmegaRNNMemory)
from .rnn_transformer import LMMBlock, LongTermMemoryModel, RNNMemoryTransformer

__all__ = ["memory_recurrence", "MemoryRecurrenceFn", "check_device_status", "AssocScan", "assoc_scan", "omega_store_update", "affine_associative_scan", "RNNMemState", "state_detach",
           "PolynomialFeatureMap", "MultiheadRMSNorm", "RNNMemoryCell", "OmegaRNNMemoryCell",
           "RNNMemory", "OmegaRNNMemory", "LMMBlock", "LongTermMemoryModel", "RNNMemoryTransformer"]
