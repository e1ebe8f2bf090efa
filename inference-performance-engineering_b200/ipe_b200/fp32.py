"""The fp32 path: the dense Qwen3 engine and uncached forward at dtype=torch.float32, the precision
of the reference's plumbing configuration (src/ipe/forward.py:32-43 admits it with TF32 off).

Every operator runs on the reference-precision kernels of csrc/fp32.cu (fp32 FMA, no tensor
cores, no bf16 rounding points) one launch at a time on the current stream: embedding, RMSNorm
(ipe_rmsnorm, fp32), the QKV / o_proj / gate-up / down_proj / LM-head GEMMs with the residual and
SiLU*up epilogues, q/k norm + RoPE + cache append, and causal attention. Weights are packed once
in fp32 (widened when stored as bf16, as the reference casts them to the run dtype). The rotary
tables are fp32 rows from the reference's formula: one call over the prompt for prefill, one
call per position for decode rows (src/ipe/engine.py:63-67, :78).
"""

from __future__ import annotations

import torch

from ipe_b200 import _native as nat
from ipe_b200 import layer as layer_hook
from ipe_b200.config import check_supported

F32 = 1  # ipe_rmsnorm dtype code


def rotary_rows_f32(positions: torch.Tensor, head_dim: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """fp32 cos/sin [T, D] (src/ipe/ops.py:41-53 at dtype float32)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    angle = positions.to(torch.float32)[:, None] * inv[None, :]
    angle = torch.cat((angle, angle), dim=-1)
    return angle.cos(), angle.sin()


class Fp32Layer:
    __slots__ = ("in_norm", "post_norm", "q_norm", "k_norm", "w_qkv", "w_o", "w_gate_up", "w_down")

    def __init__(self, layer, config):
        f = lambda t: t.to(torch.float32).contiguous()  # noqa: E731
        self.in_norm, self.post_norm = f(layer.input_layernorm), f(layer.post_attention_layernorm)
        self.q_norm, self.k_norm = f(layer.q_norm), f(layer.k_norm)
        self.w_qkv = torch.cat((f(layer.q_proj), f(layer.k_proj), f(layer.v_proj)), dim=0).contiguous()
        self.w_o, self.w_down = f(layer.o_proj), f(layer.down_proj)
        i, h, g = config.intermediate_size, config.hidden_size, nat.GATE_UP_GROUP
        gate, up = f(layer.gate_proj).view(i // g, g, h), f(layer.up_proj).view(i // g, g, h)
        self.w_gate_up = torch.stack((gate, up), dim=1).reshape(2 * i, h).contiguous()


class Fp32Model:
    """fp32 packed weights of a loaded model and its rotary tables."""

    def __init__(self, loaded):
        c, w = loaded.config, loaded.weights
        check_supported(c)
        self.loaded, self.config, self.device = loaded, c, w.embed_tokens.device
        with torch.no_grad():
            self.embed = w.embed_tokens.to(torch.float32).contiguous()
            self.lm_head = self.embed if w.lm_head is w.embed_tokens else w.lm_head.to(torch.float32).contiguous()
            self.final_norm = w.norm.to(torch.float32).contiguous()
            self.layers = [Fp32Layer(layer, c) for layer in w.layers]
        self.q_rows = c.num_attention_heads * c.head_dim
        self.qkv_rows = self.q_rows + 2 * c.num_key_value_heads * c.head_dim
        layer_hook.register(self, torch.float32)
        self._decode: tuple[torch.Tensor, torch.Tensor] | None = None
        self._prefill: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    def decode_rotary(self, capacity: int) -> tuple[torch.Tensor, torch.Tensor]:
        if self._decode is None or self._decode[0].shape[0] < capacity:
            c = self.config
            rows = [rotary_rows_f32(torch.tensor([p]), c.head_dim, c.rope_theta) for p in range(capacity)]
            self._decode = (torch.cat([r[0] for r in rows]).to(self.device).contiguous(),
                            torch.cat([r[1] for r in rows]).to(self.device).contiguous())
        return self._decode[0][:capacity], self._decode[1][:capacity]

    def prefill_rotary(self, length: int) -> tuple[torch.Tensor, torch.Tensor]:
        if length not in self._prefill:
            if len(self._prefill) > 8:
                self._prefill.clear()
            c = self.config
            cos, sin = rotary_rows_f32(torch.arange(length), c.head_dim, c.rope_theta)
            self._prefill[length] = (cos.to(self.device).contiguous(), sin.to(self.device).contiguous())
        return self._prefill[length]


_CACHE: list[tuple[object, Fp32Model]] = []


def fp32_model(loaded) -> Fp32Model:
    """The fp32 packing of `loaded`, reused while the same LoadedCheckpoint object is in use."""
    for key, model in _CACHE:
        if key is loaded:
            return model
    model = Fp32Model(loaded)
    _CACHE.clear()
    _CACHE.append((loaded, model))
    return model


class Fp32Buffers:
    """Activations of `batch` rows of `tokens` tokens (allocated once per shape)."""

    def __init__(self, model: Fp32Model, batch: int, tokens: int):
        c, dev, f = model.config, model.device, torch.float32
        rows = batch * tokens
        self.batch, self.tokens = batch, tokens
        self.ids = torch.empty(rows, dtype=torch.int64, device=dev)
        self.x = torch.empty((rows, c.hidden_size), dtype=f, device=dev)
        self.h = torch.empty_like(self.x)
        self.qkv = torch.empty((rows, model.qkv_rows), dtype=f, device=dev)
        self.q = torch.empty((batch, c.num_attention_heads, tokens, c.head_dim), dtype=f, device=dev)
        self.attn = torch.empty((rows, model.q_rows), dtype=f, device=dev)
        self.act = torch.empty((rows, c.intermediate_size), dtype=f, device=dev)
        self.last = torch.empty((batch, c.hidden_size), dtype=f, device=dev)
        self.logits = torch.empty((batch, c.vocab_size), dtype=f, device=dev)


def layer_ops(c, layer: Fp32Layer, q_rows: int, qkv_rows: int, x: torch.Tensor, h: torch.Tensor, qkv: torch.Tensor,
              q: torch.Tensor, attn: torch.Tensor, act: torch.Tensor, k_layer: torch.Tensor, v_layer: torch.Tensor,
              batch: int, tokens: int, start: int, capacity: int, cos: torch.Tensor, sin: torch.Tensor,
              stream: int) -> None:
    """One decoder layer (src/ipe/forward.py:86-115) for batch rows of `tokens` tokens at positions
    start.., x [batch*tokens, H] updated in place; cos / sin tables indexed by position."""
    lib = nat.load()
    rows, hd, i = batch * tokens, c.hidden_size, c.intermediate_size
    hq, hkv, eps = c.num_attention_heads, c.num_key_value_heads, c.rms_norm_eps
    xp, hp = x.data_ptr(), h.data_ptr()
    nat.check(lib.ipe_rmsnorm(xp, layer.in_norm.data_ptr(), hp, rows, hd, eps, F32, stream), "ipe_rmsnorm")
    nat.check(lib.ipe_gemm_f32(hp, layer.w_qkv.data_ptr(), qkv.data_ptr(), rows, qkv_rows, hd, nat.EPI_STORE, None,
                               stream), "ipe_gemm_f32 qkv")
    nat.check(lib.ipe_qk_norm_rope_append_f32(qkv.data_ptr(), batch, tokens, hq, hkv, layer.q_norm.data_ptr(),
                                              layer.k_norm.data_ptr(), cos.data_ptr(), sin.data_ptr(), start,
                                              q.data_ptr(), k_layer.data_ptr(), v_layer.data_ptr(), capacity, eps,
                                              stream), "ipe_qk_norm_rope_append_f32")
    nat.check(lib.ipe_attention_f32(q.data_ptr(), k_layer.data_ptr(), v_layer.data_ptr(), attn.data_ptr(), batch, hq,
                                    hkv, tokens, capacity, start, stream), "ipe_attention_f32")
    nat.check(lib.ipe_gemm_f32(attn.data_ptr(), layer.w_o.data_ptr(), xp, rows, hd, q_rows, nat.EPI_RESIDUAL, xp,
                               stream), "ipe_gemm_f32 o_proj")
    nat.check(lib.ipe_rmsnorm(xp, layer.post_norm.data_ptr(), hp, rows, hd, eps, F32, stream), "ipe_rmsnorm")
    nat.check(lib.ipe_gemm_f32(hp, layer.w_gate_up.data_ptr(), act.data_ptr(), rows, 2 * i, hd, nat.EPI_SILU_MUL,
                               None, stream), "ipe_gemm_f32 gate_up")
    nat.check(lib.ipe_gemm_f32(act.data_ptr(), layer.w_down.data_ptr(), xp, rows, hd, i, nat.EPI_RESIDUAL, xp, stream),
              "ipe_gemm_f32 down_proj")


def run_layers(model: Fp32Model, buf: Fp32Buffers, k: torch.Tensor, v: torch.Tensor, start: int, capacity: int,
               cos: torch.Tensor, sin: torch.Tensor, stream: int) -> None:
    """Embedding of buf.ids and every decoder layer for buf.batch rows of buf.tokens tokens at
    positions start.. ; the residual stream ends in buf.x. k / v: the fp32 caches [layers, batch
    rows, KV heads, capacity, 128]."""
    c, lib = model.config, nat.load()
    rows = buf.batch * buf.tokens
    nat.check(lib.ipe_embed_f32(buf.ids.data_ptr(), rows, model.embed.data_ptr(), c.vocab_size, c.hidden_size,
                                buf.x.data_ptr(), stream), "ipe_embed_f32")
    for index, layer in enumerate(model.layers):
        layer_ops(c, layer, model.q_rows, model.qkv_rows, buf.x, buf.h, buf.qkv, buf.q, buf.attn, buf.act, k[index],
                  v[index], buf.batch, buf.tokens, start, capacity, cos, sin, stream)


def final_norm(model: Fp32Model, x: torch.Tensor, out: torch.Tensor, stream: int) -> torch.Tensor:
    c = model.config
    nat.check(nat.load().ipe_rmsnorm(x.data_ptr(), model.final_norm.data_ptr(), out.data_ptr(), x.shape[0],
                                     c.hidden_size, c.rms_norm_eps, F32, stream), "ipe_rmsnorm")
    return out


def lm_logits(model: Fp32Model, hidden: torch.Tensor, out: torch.Tensor, stream: int) -> torch.Tensor:
    """out [n, V] = hidden [n, H] (final-normed) @ lm_head^T in fp32 (src/ipe/forward.py:145-152)."""
    c = model.config
    nat.check(nat.load().ipe_gemm_f32(hidden.data_ptr(), model.lm_head.data_ptr(), out.data_ptr(), hidden.shape[0],
                                      c.vocab_size, c.hidden_size, nat.EPI_LOGITS, None, stream), "ipe_gemm_f32 lm_head")
    return out


def step_logits(model: Fp32Model, buf: Fp32Buffers, stream: int) -> torch.Tensor:
    """Final norm of each row's last token and the LM head: fp32 [batch, V] in buf.logits."""
    rows = buf.x.view(buf.batch, buf.tokens, -1)[:, -1].contiguous() if buf.tokens > 1 else buf.x
    final_norm(model, rows, buf.last, stream)
    return lm_logits(model, buf.last, buf.logits, stream)


def uncached_hidden(model: Fp32Model, token_ids: torch.Tensor) -> torch.Tensor:
    """Final-normed fp32 states [B*T, H] through a prompt-sized cache (src/ipe/forward.py:118-142)."""
    c = model.config
    batch, length = token_ids.shape
    shape = (c.num_hidden_layers, batch, c.num_key_value_heads, length, c.head_dim)
    k = torch.empty(shape, dtype=torch.float32, device=model.device)
    v = torch.empty_like(k)
    buf = Fp32Buffers(model, batch, length)
    buf.ids.copy_(token_ids.to(device=model.device, dtype=torch.int64).reshape(-1))
    cos, sin = model.prefill_rotary(length)
    stream = torch.cuda.current_stream().cuda_stream
    run_layers(model, buf, k, v, 0, length, cos, sin, stream)
    return final_norm(model, buf.x, torch.empty_like(buf.x), stream)
