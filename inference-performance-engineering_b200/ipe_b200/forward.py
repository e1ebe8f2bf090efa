"""The uncached forward pass on the CUDA kernels, and the argument validators.

Drop-in for the reference's `ipe.forward` (src/ipe/forward.py):
- `check_dtype`, `check_token_ids`: the same checks and ValueError messages (`:32-63`);
- `forward_full(loaded, token_ids, *, dtype, logit_positions=None, backend="math")`: fp32 logits
  [B, n, V] (bf16 logits widened), computed by the prefill kernels with a cache sized to the
  prompt (`:155-170`);
- `final_hidden` / `lm_logits`: the final-normed states and the tied LM head (`:133-152`);
- `decoder_layer`: one layer with the reference's signature (`:86-115`, ipe_b200.layer).

The CUDA path computes in bf16 (weight-streaming and tcgen05 kernels) or in fp32 (the
reference-precision kernels of ipe_b200.fp32, for the plumbing configuration). fp64 (the
reference's oracle) is rejected with a ValueError: the fp64 oracle is a CPU program and is not part
of this package.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from ipe_b200.config import check_supported
from ipe_b200.layer import decoder_layer  # noqa: F401  (src/ipe/forward.py:86-115, the engine's per-layer hook)
from ipe_b200.model import PackedModel, PrefillBuffers, packed_model, run_prefill_layers
from ipe_b200 import fp32 as _fp32
from ipe_b200 import ops
from ipe_b200 import _native as nat

INTEGER_DTYPES = (torch.int64, torch.int32, torch.int16, torch.int8, torch.uint8)
BACKENDS = ("math", "sdpa")
RUN_DTYPES = (torch.bfloat16, torch.float32)


def check_dtype(loaded, dtype: torch.dtype, allowed: Sequence[torch.dtype]) -> None:
    """The reference's dtype admission (src/ipe/forward.py:32-43), then the CUDA path's limits."""
    if dtype not in allowed:
        raise ValueError(f"dtype {dtype!r}: expected one of {list(allowed)}")
    stored = loaded.weights.embed_tokens
    if stored.dtype.itemsize > dtype.itemsize:
        raise ValueError(f"dtype {dtype!r}: weights are stored in the wider {stored.dtype!r}")
    if stored.device.type == "cuda" and dtype == torch.float32 and torch.backends.cuda.matmul.fp32_precision == "tf32":
        raise ValueError("dtype float32 on cuda: TF32 matmul is enabled; set torch.backends.cuda.matmul.fp32_precision = 'ieee'")
    if dtype not in RUN_DTYPES:
        raise ValueError(f"dtype {dtype!r}: the CUDA path computes in bfloat16 or float32")
    if stored.device.type != "cuda":
        raise ValueError(f"device {stored.device}: the CUDA path needs the weights on a CUDA device")
    if dtype == torch.bfloat16 and stored.dtype != torch.bfloat16:
        raise ValueError(f"weights stored as {stored.dtype}: the bfloat16 path streams bfloat16 weights")
    check_supported(loaded.config)


def _within(values: torch.Tensor, upper: int) -> bool:
    """Whether every integer in `values` lies in [0, upper), compared in int64 (a bound compared in
    a narrower dtype would wrap). Syncs for GPU tensors."""
    wide = values.to(torch.int64)
    return bool(wide.min() >= 0) and bool(wide.max() < upper)


def check_token_ids(config, token_ids: object, capacity: int) -> tuple[int, int]:
    """Integer IDs [B, T] in the vocabulary, 1 <= T <= capacity; (B, T). Syncs for GPU IDs
    (the admission and messages of src/ipe/forward.py:46-63)."""
    if not isinstance(token_ids, torch.Tensor):
        raise ValueError(f"token_ids: expected a tensor, got {type(token_ids).__name__}")
    shape = list(token_ids.shape)
    checks = (
        (token_ids.dtype in INTEGER_DTYPES, lambda: f"expected one of {list(INTEGER_DTYPES)}, got {token_ids.dtype}"),
        (len(shape) == 2 and shape[0] >= 1, lambda: f"expected shape [B, T] with B >= 1, got {shape}"),
        (len(shape) == 2 and 1 <= shape[-1] <= capacity, lambda: f"length {shape[-1]} is outside 1 to {capacity}"),
    )
    for ok, message in checks:
        if not ok:
            raise ValueError(f"token_ids: {message()}")
    if not _within(token_ids, config.vocab_size):
        raise ValueError(f"token_ids: IDs must lie in [0, {config.vocab_size})")
    return shape[0], shape[1]


def check_backend(backend: object) -> None:
    if backend not in BACKENDS:
        raise ValueError(f"backend {backend!r}: expected one of {list(BACKENDS)}")


def _check_logit_positions(logit_positions: object, length: int) -> torch.Tensor:
    """The requested positions as int64 [n], n >= 1, each in [0, length) (src/ipe/forward.py:71-83)."""
    try:
        rows = torch.as_tensor(logit_positions)
    except (TypeError, ValueError, RuntimeError) as error:
        raise ValueError(f"logit_positions: {error}") from error
    if rows.dtype not in INTEGER_DTYPES:
        raise ValueError(f"logit_positions: expected integers, got {rows.dtype}")
    if rows.dim() != 1 or rows.numel() == 0:
        raise ValueError("logit_positions: expected a non-empty 1-D sequence")
    if not _within(rows, length):
        raise ValueError(f"logit_positions: positions must lie in [0, {length})")
    return rows.to(torch.int64)


def _uncached_hidden(model: PackedModel, token_ids: torch.Tensor) -> torch.Tensor:
    """Final-normed bf16 states [B*T, H] through the prefill kernels with a prompt-sized cache."""
    c = model.config
    batch, length = token_ids.shape
    cache_shape = (c.num_hidden_layers, batch, c.num_key_value_heads, length, c.head_dim)
    k = torch.empty(cache_shape, dtype=torch.bfloat16, device=model.device)
    v = torch.empty(cache_shape, dtype=torch.bfloat16, device=model.device)
    buffers = PrefillBuffers(model, batch * length, batch, length)
    cos, sin = model.prefill_rotary(length)
    ids = token_ids.to(device=model.device, dtype=torch.int64).reshape(-1).contiguous()
    x = buffers.x[: batch * length]
    ops.embed(ids, model.embed, x)
    run_prefill_layers(model, buffers, k, v, batch, length, length, cos, sin)
    hidden = torch.empty_like(x)
    ops.rms_norm_out(x, model.final_norm, c.rms_norm_eps, hidden)
    return hidden


def final_hidden(loaded, token_ids: torch.Tensor, *, dtype: torch.dtype, backend: str = "math") -> torch.Tensor:
    """Final-normed hidden states [B, T, H] (src/ipe/forward.py:133-142)."""
    check_dtype(loaded, dtype, (torch.bfloat16, torch.float32, torch.float64))
    check_backend(backend)
    batch, length = check_token_ids(loaded.config, token_ids, loaded.config.max_position_embeddings)
    if dtype == torch.float32:
        return _fp32.uncached_hidden(_fp32.fp32_model(loaded), token_ids).view(batch, length, -1)
    return _uncached_hidden(packed_model(loaded), token_ids).view(batch, length, -1)


def lm_logits(loaded, hidden: torch.Tensor) -> torch.Tensor:
    """Logits [..., V] in hidden.dtype for final-normed states [..., H] (src/ipe/forward.py:145-152)."""
    if not isinstance(hidden, torch.Tensor) or hidden.dim() < 1 or hidden.shape[-1] != loaded.config.hidden_size:
        raise ValueError(f"hidden: expected a tensor [..., {loaded.config.hidden_size}]")
    if hidden.device != loaded.weights.lm_head.device:
        raise ValueError(f"hidden: on {hidden.device}, weights on {loaded.weights.lm_head.device}")
    check_dtype(loaded, hidden.dtype, (torch.bfloat16, torch.float32, torch.float64))
    rows = hidden.reshape(-1, hidden.shape[-1]).contiguous()
    logits = torch.empty((rows.shape[0], loaded.config.vocab_size), dtype=torch.float32, device=hidden.device)
    if hidden.dtype == torch.float32:
        _fp32.lm_logits(_fp32.fp32_model(loaded), rows, logits, torch.cuda.current_stream().cuda_stream)
        return logits.view(*hidden.shape[:-1], -1)
    ops.gemm(rows, packed_model(loaded).embed, logits, nat.EPI_LOGITS)
    return logits.to(hidden.dtype).view(*hidden.shape[:-1], -1)


def forward_full(loaded, token_ids: torch.Tensor, *, dtype: torch.dtype,
                 logit_positions: Sequence[int] | torch.Tensor | None = None, backend: str = "math") -> torch.Tensor:
    """fp32 logits [B, n, V] at logit_positions (all positions when None), uncached
    (src/ipe/forward.py:155-170). `backend` is accepted for API compatibility; one CUDA path runs."""
    check_dtype(loaded, dtype, (torch.bfloat16, torch.float32))
    check_backend(backend)
    batch, length = check_token_ids(loaded.config, token_ids, loaded.config.max_position_embeddings)
    rows = None if logit_positions is None else _check_logit_positions(logit_positions, length)
    if dtype == torch.float32:
        model32 = _fp32.fp32_model(loaded)
        hidden = _fp32.uncached_hidden(model32, token_ids).view(batch, length, -1)
        if rows is not None:
            hidden = hidden[:, rows.to(hidden.device)]
        selected = hidden.reshape(-1, hidden.shape[-1]).contiguous()
        logits = torch.empty((selected.shape[0], loaded.config.vocab_size), dtype=torch.float32, device=model32.device)
        _fp32.lm_logits(model32, selected, logits, torch.cuda.current_stream().cuda_stream)
        return logits.view(batch, -1, loaded.config.vocab_size)
    model = packed_model(loaded)
    hidden = _uncached_hidden(model, token_ids).view(batch, length, -1)
    if rows is not None:
        hidden = hidden[:, rows.to(hidden.device)]
    selected = hidden.reshape(-1, hidden.shape[-1]).contiguous()
    logits = torch.empty((selected.shape[0], loaded.config.vocab_size), dtype=torch.float32, device=model.device)
    ops.gemm(selected, model.embed, logits, nat.EPI_LOGITS)
    return logits.view(batch, -1, loaded.config.vocab_size)
