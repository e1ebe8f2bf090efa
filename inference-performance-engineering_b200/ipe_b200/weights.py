"""The weight interface the hot path consumes.

Field names, order and layout ([out, in]) follow the reference's dataclasses
(`src/ipe/weights.py:38-75`): a `LoadedCheckpoint` built by the reference's loader can be passed
to this package unchanged, and the reverse. `lm_head is embed_tokens` whenever the head is tied.
Loading safetensors files is not part of this package; see `ipe_b200.synthetic` for the
random-init models the benchmarks use.
"""

from dataclasses import dataclass

import torch

from ipe_b200.config import Qwen3Config

DTYPES = (torch.bfloat16, torch.float32, torch.float64)

LAYER_FIELDS = ("input_layernorm", "q_proj", "k_proj", "v_proj", "q_norm", "k_norm", "o_proj",
                "post_attention_layernorm", "gate_proj", "up_proj", "down_proj")


@dataclass(frozen=True, slots=True)
class LayerWeights:
    input_layernorm: torch.Tensor
    q_proj: torch.Tensor
    k_proj: torch.Tensor
    v_proj: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    o_proj: torch.Tensor
    post_attention_layernorm: torch.Tensor
    gate_proj: torch.Tensor
    up_proj: torch.Tensor
    down_proj: torch.Tensor


@dataclass(frozen=True, slots=True)
class Qwen3Weights:
    embed_tokens: torch.Tensor
    layers: tuple[LayerWeights, ...]
    norm: torch.Tensor
    lm_head: torch.Tensor  # the same object as embed_tokens whenever tied


@dataclass(frozen=True, slots=True)
class TieRecord:
    stored: bool
    tied: bool
    max_abs_diff: float | None


@dataclass(frozen=True, slots=True)
class LoadedCheckpoint:
    config: Qwen3Config
    weights: Qwen3Weights
    tie: TieRecord
