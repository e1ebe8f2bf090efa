"""Dense Qwen3 structure the CUDA path is built for.

`Qwen3Config` has the ten fields, names and meaning of the reference's frozen dataclass
(`src/ipe/config.py:20-33`), so a reference config object and this one are interchangeable. Config
file admission (`validate_config`, `load_config`) is not part of the hot path; configs are built
directly, as the synthetic benchmark models are.
"""

from dataclasses import dataclass


@dataclass(frozen=True, slots=True)
class Qwen3Config:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    max_position_embeddings: int
    rms_norm_eps: float
    rope_theta: float


# The two published dense sizes the benchmark workloads use (hidden, intermediate, layers, heads).
QWEN3_0_6B = Qwen3Config(151936, 1024, 3072, 28, 16, 8, 128, 40960, 1e-6, 1e6)
QWEN3_1_7B = Qwen3Config(151936, 2048, 6144, 28, 16, 8, 128, 40960, 1e-6, 1e6)


def check_supported(config) -> None:
    """Raise ValueError unless the CUDA kernels cover this shape.

    The kernels are specialised for what every dense Qwen3 size uses: head_dim 128, grouped
    query heads, and hidden / intermediate widths that are multiples of 128.
    """
    problems = []
    if config.head_dim != 128:
        problems.append(f"head_dim {config.head_dim} (kernels are built for 128)")
    if config.num_attention_heads % config.num_key_value_heads:
        problems.append("num_attention_heads must be a multiple of num_key_value_heads")
    elif config.num_attention_heads // config.num_key_value_heads > 8:
        problems.append("more than 8 query heads per KV head")
    for name in ("hidden_size", "intermediate_size"):
        if getattr(config, name) % 128:
            problems.append(f"{name} {getattr(config, name)} is not a multiple of 128")
    if config.hidden_size > 8192 or config.intermediate_size > 32768:
        problems.append("hidden_size above 8192 or intermediate_size above 32768")
    if problems:
        raise ValueError("config not supported by the CUDA path: " + "; ".join(problems))
