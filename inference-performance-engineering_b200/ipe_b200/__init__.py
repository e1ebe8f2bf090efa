"""ipe_b200: a B200-native (sm_100a) implementation of the dense Qwen3 prefill/decode hot path.

Drop-in for the reference engine's API (`ipe.engine.Engine`, `ipe.forward.forward_full`); see
`ipe_b200.engine` and `ipe_b200.forward`. All compute runs in hand-written CUDA kernels loaded from
`ipe_b200/lib/libipe_b200.so` through the C-ABI of `include/ipe_b200.h`; there is no CPU path.
"""

from ipe_b200.config import QWEN3_0_6B, QWEN3_1_7B, Qwen3Config
from ipe_b200.engine import Engine, Generation, sample
from ipe_b200.forward import final_hidden, forward_full, lm_logits
from ipe_b200.weights import LayerWeights, LoadedCheckpoint, Qwen3Weights, TieRecord

__all__ = ["Engine", "Generation", "sample", "forward_full", "final_hidden", "lm_logits", "Qwen3Config",
           "QWEN3_0_6B", "QWEN3_1_7B", "LayerWeights", "Qwen3Weights", "TieRecord", "LoadedCheckpoint"]
