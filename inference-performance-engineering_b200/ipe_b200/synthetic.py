"""Random-initialised Qwen3 models for the benchmark workloads and tests.

The benchmark model: every matrix, the tied embedding included, is N(0, std^2) with std 0.02, and
every RMSNorm weight is 1.0. One generator seeded with `seed` draws the embedding first, then each
layer's matrices in LayerWeights field order. Prompts are `torch.randint(0, vocab, (B, P))` from a
generator seeded 0. With `generator_device="cpu"` the values are those of the reference's CPU
generator; `"cuda"` draws on the GPU (different values, much faster for the 1.7B model).

`norm_jitter` > 0 draws the norm weights as 1 + jitter * N(0, 1) instead, which makes the weight
multiply's rounding visible in parity tests.
"""

import torch

from ipe_b200.config import Qwen3Config
from ipe_b200.weights import LAYER_FIELDS, LayerWeights, LoadedCheckpoint, Qwen3Weights, TieRecord

_NORMS = ("input_layernorm", "q_norm", "k_norm", "post_attention_layernorm")


def layer_shapes(c: Qwen3Config) -> dict[str, tuple[int, ...]]:
    q, kv = c.num_attention_heads * c.head_dim, c.num_key_value_heads * c.head_dim
    return {"input_layernorm": (c.hidden_size,), "q_proj": (q, c.hidden_size), "k_proj": (kv, c.hidden_size),
            "v_proj": (kv, c.hidden_size), "q_norm": (c.head_dim,), "k_norm": (c.head_dim,),
            "o_proj": (c.hidden_size, q), "post_attention_layernorm": (c.hidden_size,),
            "gate_proj": (c.intermediate_size, c.hidden_size), "up_proj": (c.intermediate_size, c.hidden_size),
            "down_proj": (c.hidden_size, c.intermediate_size)}


def random_model(config: Qwen3Config, *, seed: int = 0, std: float = 0.02, dtype=torch.bfloat16,
                 device="cpu", generator_device="cpu", norm_jitter: float = 0.0) -> LoadedCheckpoint:
    gen = torch.Generator(generator_device).manual_seed(seed)

    def matrix(shape):
        value = torch.randn(shape, generator=gen, device=generator_device, dtype=torch.float32) * std
        return value.to(dtype).to(device)

    def norm(size):
        if norm_jitter == 0:
            return torch.ones(size, dtype=dtype, device=device)
        value = 1 + norm_jitter * torch.randn(size, generator=gen, device=generator_device, dtype=torch.float32)
        return value.to(dtype).to(device)

    embed = matrix((config.vocab_size, config.hidden_size))
    shapes = layer_shapes(config)
    layers = []
    for _ in range(config.num_hidden_layers):
        fields = {name: (norm(shapes[name][0]) if name in _NORMS else matrix(shapes[name])) for name in LAYER_FIELDS}
        layers.append(LayerWeights(**fields))
    weights = Qwen3Weights(embed, tuple(layers), norm(config.hidden_size), embed)
    return LoadedCheckpoint(config, weights, TieRecord(stored=False, tied=True, max_abs_diff=None))


def random_prompts(config: Qwen3Config, batch: int, length: int, *, seed: int = 0) -> torch.Tensor:
    """Token IDs uniform in [0, vocab) from a CPU generator, int64 [batch, length]."""
    return torch.randint(0, config.vocab_size, (batch, length), generator=torch.Generator().manual_seed(seed))
