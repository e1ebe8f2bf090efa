"""The synthetic models the golden vectors were made from (tests/golden/make_golden.py), rebuilt
with the same seeds, plus helpers shared by the test modules."""

import dataclasses

import torch

from ipe_b200.config import QWEN3_0_6B, QWEN3_1_7B, Qwen3Config
from ipe_b200.synthetic import random_model

CASES = {
    "small": (Qwen3Config(2048, 256, 512, 2, 4, 2, 128, 8192, 1e-5, 1e4), {"seed": 1, "std": 0.06, "norm_jitter": 0.1}),
    "mqa": (Qwen3Config(512, 128, 384, 3, 4, 1, 128, 8192, 1e-6, 1e6), {"seed": 2, "std": 0.08, "norm_jitter": 0.1}),
    "qwen3-0.6b-2layer": (dataclasses.replace(QWEN3_0_6B, num_hidden_layers=2), {"seed": 0, "std": 0.02}),
    "qwen3-1.7b-2layer": (dataclasses.replace(QWEN3_1_7B, num_hidden_layers=2), {"seed": 0, "std": 0.02}),
}


def build(name, device="cpu"):
    config, init = CASES[name]
    return random_model(config, device=device, **init)


def to_device(loaded, device):
    """The same model with every tensor moved to `device` (the tie is kept)."""
    from ipe_b200.weights import LayerWeights, LoadedCheckpoint, Qwen3Weights

    w = loaded.weights
    embed = w.embed_tokens.to(device)
    layers = tuple(LayerWeights(**{f: getattr(layer, f).to(device) for f in layer.__slots__}) for layer in w.layers)
    return LoadedCheckpoint(loaded.config, Qwen3Weights(embed, layers, w.norm.to(device), embed), loaded.tie)


def same_bits(actual, expected):
    return actual.dtype == expected.dtype and actual.shape == expected.shape and torch.equal(
        actual.contiguous().view(torch.uint8), expected.contiguous().view(torch.uint8))
