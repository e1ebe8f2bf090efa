"""CPU restatement of the reference Qwen3 forward pass and cached engine. TEST INFRASTRUCTURE ONLY.

Every function follows the reference's operation order and rounding points at bf16/fp32, so its
results are bitwise comparable with the reference on the same machine; at fp64 every step is fp64
(the reference's oracle, `src/ipe/forward.py:133-152`). The model argument is any object with
`.config` (the ten Qwen3Config fields) and `.weights` (embed_tokens, layers[i].<LayerWeights
fields>, norm, lm_head), which is what `ipe_b200.weights.LoadedCheckpoint` and the reference's
own `LoadedCheckpoint` both provide.

Used only by tests/, `__graft_entry__.smoke()` and bench.py's CPU baseline.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

RUN_DTYPES = (torch.bfloat16, torch.float32)
BACKENDS = ("math", "sdpa")


def statistics_dtype(dtype: torch.dtype) -> torch.dtype:
    """fp32 statistics for bf16/fp32 runs, fp64 for the oracle (`src/ipe/ops.py:18-20`)."""
    return torch.float64 if dtype == torch.float64 else torch.float32


# ----------------------------------------------------------------------------------- operators

def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """weight * cast(x * rsqrt(mean(x^2) + eps)); two roundings at bf16 (`src/ipe/ops.py:23-33`)."""
    wide = x.to(statistics_dtype(x.dtype))
    mean_square = wide.pow(2).mean(-1, keepdim=True)
    return weight * (wide * torch.rsqrt(mean_square + eps)).to(x.dtype)


def qk_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Per-head RMSNorm of queries or keys over head_dim (`src/ipe/ops.py:36-38`)."""
    return rms_norm(x, weight, eps)


def rotary_tables(positions: torch.Tensor, head_dim: int, theta: float,
                  dtype: torch.dtype) -> tuple[torch.Tensor, torch.Tensor]:
    """Split-half cos/sin [T, D] from fp32 (fp64 for the oracle) angles (`src/ipe/ops.py:41-53`)."""
    wide = statistics_dtype(dtype)
    exponent = torch.arange(0, head_dim, 2, dtype=wide) / head_dim
    inverse_frequency = 1.0 / (theta ** exponent)
    angle = positions.to(wide)[:, None] * inverse_frequency[None, :]
    angle = torch.cat((angle, angle), dim=-1)
    return angle.cos().to(dtype), angle.sin().to(dtype)


def apply_rotary(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x*cos + rotate_half(x)*sin in x.dtype, three roundings (`src/ipe/ops.py:56-63`)."""
    half = x.shape[-1] // 2
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return (x * cos) + (rotated * sin)


def _expand_groups(t: torch.Tensor, groups: int) -> torch.Tensor:
    """[B, Hkv, S, D] -> [B, Hkv*groups, S, D], materialised (`src/ipe/ops.py:66-75`)."""
    if groups == 1:
        return t
    b, h, s, d = t.shape
    return t[:, :, None].expand(b, h, groups, s, d).reshape(b, h * groups, s, d)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool,
              backend: str) -> torch.Tensor:
    """GQA attention, scale D^-0.5; `math` or `sdpa` (`src/ipe/ops.py:78-101`)."""
    groups = q.shape[1] // k.shape[1]
    scale = q.shape[-1] ** -0.5
    if backend == "sdpa":
        return F.scaled_dot_product_attention(q, k, v, is_causal=causal and q.shape[2] > 1,
                                              scale=scale, enable_gqa=groups > 1)
    k = _expand_groups(k, groups)
    v = _expand_groups(v, groups)
    scores = torch.matmul(q, k.transpose(2, 3)) * scale
    if causal:
        t = q.shape[2]
        mask = torch.full((t, t), torch.finfo(q.dtype).min, dtype=q.dtype, device=q.device).triu(1)
        scores = scores + mask
    probabilities = F.softmax(scores, dim=-1, dtype=statistics_dtype(q.dtype)).to(q.dtype)
    return torch.matmul(probabilities, v)


def swiglu(x: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor) -> torch.Tensor:
    """down(silu(gate x) * up x) (`src/ipe/ops.py:104-106`)."""
    return F.linear(F.silu(F.linear(x, gate)) * F.linear(x, up), down)


# ------------------------------------------------------------------------------- decoder layer

def decoder_layer(x, layer, rope, config, *, backend, cache=None, start=0):
    """One pre-norm layer at positions start..start+T-1 (`src/ipe/forward.py:86-115`).

    cache is (K, V) [B, Hkv, capacity, D]; a prompt (start 0) attends causally to itself, a
    decode step (T 1) to positions 0..start.
    """
    dtype, eps = x.dtype, config.rms_norm_eps
    b, t, _ = x.shape
    per_head = (b, t, -1, config.head_dim)
    h = rms_norm(x, layer.input_layernorm.to(dtype), eps)
    q = qk_norm(F.linear(h, layer.q_proj.to(dtype)).view(per_head), layer.q_norm.to(dtype), eps)
    k = qk_norm(F.linear(h, layer.k_proj.to(dtype)).view(per_head), layer.k_norm.to(dtype), eps)
    v = F.linear(h, layer.v_proj.to(dtype)).view(per_head).transpose(1, 2)
    cos, sin = rope
    q = apply_rotary(q.transpose(1, 2), cos, sin)
    k = apply_rotary(k.transpose(1, 2), cos, sin)
    if cache is not None:
        end = start + t
        cache[0][:, :, start:end] = k
        cache[1][:, :, start:end] = v
        if start > 0:
            k, v = cache[0][:, :, :end], cache[1][:, :, :end]
    attended = attention(q, k, v, causal=start == 0, backend=backend)
    x = x + F.linear(attended.transpose(1, 2).reshape(b, t, -1), layer.o_proj.to(dtype))
    h = rms_norm(x, layer.post_attention_layernorm.to(dtype), eps)
    return x + swiglu(h, layer.gate_proj.to(dtype), layer.up_proj.to(dtype), layer.down_proj.to(dtype))


# ---------------------------------------------------------------------------- uncached forward

def final_hidden(model, token_ids: torch.Tensor, *, dtype: torch.dtype, backend: str = "math") -> torch.Tensor:
    """Final-normed hidden states [B, T, H] in dtype; fp64 gives the oracle (`src/ipe/forward.py:118-142`)."""
    config, weights = model.config, model.weights
    device = weights.embed_tokens.device
    cos, sin = rotary_tables(torch.arange(token_ids.shape[1]), config.head_dim, config.rope_theta, dtype)
    rope = (cos.to(device), sin.to(device))
    x = F.embedding(token_ids.to(device=device, dtype=torch.int64), weights.embed_tokens).to(dtype)
    for layer in weights.layers:
        x = decoder_layer(x, layer, rope, config, backend=backend)
    return rms_norm(x, weights.norm.to(dtype), config.rms_norm_eps)


def lm_logits(model, hidden: torch.Tensor) -> torch.Tensor:
    """Tied LM head in hidden.dtype (`src/ipe/forward.py:145-152`)."""
    return F.linear(hidden, model.weights.lm_head.to(hidden.dtype))


def forward_full(model, token_ids: torch.Tensor, *, dtype: torch.dtype, logit_positions=None,
                 backend: str = "math") -> torch.Tensor:
    """fp32 logits [B, n, V] at the given positions, uncached (`src/ipe/forward.py:155-170`)."""
    hidden = final_hidden(model, token_ids, dtype=dtype, backend=backend)
    if logit_positions is not None:
        hidden = hidden[:, torch.as_tensor(logit_positions, dtype=torch.int64)]
    return lm_logits(model, hidden).float()


def oracle_logits(model, token_ids: torch.Tensor, positions) -> torch.Tensor:
    """fp64 oracle logits [B, n, V]: `lm_logits(final_hidden(fp64))`, the reference's oracle as used
    by `tests/needs_torch/test_engine.py:93` (`src/ipe/forward.py:133-152`)."""
    hidden = final_hidden(model, token_ids, dtype=torch.float64)[:, torch.as_tensor(positions)]
    return lm_logits(model, hidden)


# ------------------------------------------------------------------------------ cached engine

def sample(logits: torch.Tensor, temperature: float, generator=None):
    """Greedy (lowest ID on ties) or Gumbel-max; untempered logprobs (`src/ipe/engine.py:28-41`)."""
    if temperature == 0:
        tokens = logits.argmax(dim=-1)
    else:
        uniform = torch.rand(logits.shape, generator=generator, dtype=torch.float32, device=logits.device)
        tokens = (logits / temperature - torch.log(-torch.log(uniform))).argmax(dim=-1)
    logprobs = F.log_softmax(logits, dim=-1).gather(-1, tokens[:, None]).squeeze(-1)
    return tokens, logprobs


class CachedEngine:
    """The reference engine's cached prefill/decode/generate (`src/ipe/engine.py:44-148`).

    Argument validation is left to the product under test; this class only computes.
    """

    def __init__(self, model, *, batch: int, capacity: int, dtype: torch.dtype, backend: str = "sdpa"):
        c = model.config
        device = model.weights.embed_tokens.device
        self.model, self.dtype, self.backend, self.capacity = model, dtype, backend, capacity
        shape = (c.num_hidden_layers, batch, c.num_key_value_heads, capacity, c.head_dim)
        self._k = torch.full(shape, float("nan"), dtype=dtype, device=device)
        self._v = torch.full(shape, float("nan"), dtype=dtype, device=device)
        # one position per call, as the reference builds its decode rows (`src/ipe/engine.py:63-67`)
        rows = [rotary_tables(torch.tensor([p]), c.head_dim, c.rope_theta, dtype) for p in range(capacity)]
        self._cos = torch.cat([r[0] for r in rows]).to(device)
        self._sin = torch.cat([r[1] for r in rows]).to(device)
        self.batch = 0
        self.length = 0

    def _step(self, token_ids, rope, start):
        c, w = self.model.config, self.model.weights
        b = token_ids.shape[0]
        x = F.embedding(token_ids.to(device=self._k.device, dtype=torch.int64), w.embed_tokens).to(self.dtype)
        for i, layer in enumerate(w.layers):
            x = decoder_layer(x, layer, rope, c, backend=self.backend, cache=(self._k[i, :b], self._v[i, :b]),
                              start=start)
        hidden = rms_norm(x[:, -1], w.norm.to(self.dtype), c.rms_norm_eps)
        return F.linear(hidden, w.lm_head.to(self.dtype)).float()

    def prefill(self, token_ids):
        c = self.model.config
        b, t = token_ids.shape
        self.batch = self.length = 0
        cos, sin = rotary_tables(torch.arange(t), c.head_dim, c.rope_theta, self.dtype)
        logits = self._step(token_ids, (cos.to(self._k.device), sin.to(self._k.device)), 0)
        self.batch, self.length = b, t
        return logits

    def decode(self, tokens):
        p = self.length
        logits = self._step(tokens[:, None], (self._cos[p:p + 1], self._sin[p:p + 1]), p)
        self.length += 1
        return logits

    def generate(self, token_ids, max_new_tokens, *, temperature=0.0, seed=0):
        generator = torch.Generator(self._k.device).manual_seed(seed) if temperature > 0 else None
        logits = self.prefill(token_ids)
        tokens = torch.empty((self.batch, max_new_tokens), dtype=torch.int64)
        logprobs = torch.empty((self.batch, max_new_tokens), dtype=torch.float32)
        for step in range(max_new_tokens):
            tokens[:, step], logprobs[:, step] = sample(logits, temperature, generator)
            if step + 1 < max_new_tokens:
                logits = self.decode(tokens[:, step])
        return tokens, logprobs


def teacher_forced(engine, token_ids: torch.Tensor, prompt: int) -> torch.Tensor:
    """fp32 logits [B, T-prompt+1, V] for positions prompt-1..T-1 fed the given tokens
    (`tests/needs_torch/test_engine.py:31-35`). Works for any engine with prefill/decode."""
    logits = [engine.prefill(token_ids[:, :prompt])]
    logits += [engine.decode(token_ids[:, p]) for p in range(prompt, token_ids.shape[1])]
    return torch.stack(logits, dim=1)
