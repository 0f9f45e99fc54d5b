"""atlas_rnn_b200: B200-native memory-update hot path of Atlas-RNN.

Public API mirrors atlas_pytorch/rnn_memory.py (RNNMemoryCell, OmegaRNNMemoryCell,
RNNMemory, OmegaRNNMemory, RNNMemState, state_detach, PolynomialFeatureMap) plus the
functional ``memory_recurrence`` and the multi-GPU helpers in ``parallel``.
"""
from .ops import memory_recurrence, MemoryRecurrenceFn
from .rnn_memory import (RNNMemState, state_detach, PolynomialFeatureMap, MultiheadRMSNorm,
                         RNNMemoryCell, OmegaRNNMemoryCell, RNNMemory, OmegaRNNMemory)

__all__ = ["memory_recurrence", "MemoryRecurrenceFn", "RNNMemState", "state_detach",
           "PolynomialFeatureMap", "MultiheadRMSNorm", "RNNMemoryCell", "OmegaRNNMemoryCell",
           "RNNMemory", "OmegaRNNMemory"]
