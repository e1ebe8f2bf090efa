"""Device-side layout of a loaded Qwen3 model, and the per-layer launch sequences.

`PackedModel` turns the reference-layout weights ([out, in] per projection, src/ipe/weights.py)
into the layout the kernels stream, once per loaded model:

- w_qkv [Q + 2*KV, H]: q_proj | k_proj | v_proj rows, so one pass computes all three;
- w_gate_up [2*I, H]: gate and up rows interleaved in groups of 64 (IPE_GATE_UP_GROUP), so one
  CTA (decode) or one 128-column tile (prefill) holds matching gate and up rows for SiLU * up;
- o_proj, down_proj, the norms and the tied embedding are used in place.

It also builds the bf16 rotary tables the way the reference engine does on the host
(src/ipe/engine.py:63-67 per position for decode rows; src/ipe/engine.py:78 one call over the
prompt for prefill).

`prefill_ops` / `prefill_layer` issue one decoder layer over a prompt (src/ipe/forward.py:86-115)
as a chain of C-ABI launches on the current stream; nothing here computes on the CPU.
"""

from __future__ import annotations

import torch

from ipe_b200 import _native as nat
from ipe_b200 import layer as layer_hook
from ipe_b200.config import check_supported


def rotary_rows(positions: torch.Tensor, head_dim: int, theta: float) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 cos/sin [T, D] for int64 positions: fp32 angles from inv_freq = 1/theta^(2j/D), split
    halves (the formula of src/ipe/ops.py:41-53, evaluated on the host as the reference does)."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    angle = positions.to(torch.float32)[:, None] * inv[None, :]
    angle = torch.cat((angle, angle), dim=-1)
    return angle.cos().to(torch.bfloat16), angle.sin().to(torch.bfloat16)


def decode_tiles(w: torch.Tensor, w_up: torch.Tensor | None = None) -> torch.Tensor:
    """The decode-tile layout the weight-streaming kernels read (see include/ipe_b200.h), built on
    the GPU by ipe_decode_tiles from a row-major [rows, in] matrix (or a gate/up pair)."""
    lib = nat.load()
    rows, k = w.shape
    tiles = torch.empty(int(lib.ipe_decode_tiles_bytes(rows, k, 1 if w_up is not None else 0)), dtype=torch.uint8,
                        device=w.device)
    nat.check(lib.ipe_decode_tiles(w.data_ptr(), None if w_up is None else w_up.data_ptr(), tiles.data_ptr(), rows, k,
                                   torch.cuda.current_stream(w.device).cuda_stream), "ipe_decode_tiles")
    return tiles


class PackedLayer:
    __slots__ = ("in_norm", "post_norm", "q_norm", "k_norm", "w_qkv", "w_o", "w_gate_up", "w_down", "t_qkv", "t_o",
                 "t_gate_up", "t_down", "ptr")

    def __init__(self, layer, config):
        self.in_norm = layer.input_layernorm.contiguous()
        self.post_norm = layer.post_attention_layernorm.contiguous()
        self.q_norm = layer.q_norm.contiguous()
        self.k_norm = layer.k_norm.contiguous()
        self.w_qkv = torch.cat((layer.q_proj, layer.k_proj, layer.v_proj), dim=0).contiguous()
        self.w_o = layer.o_proj.contiguous()
        i, h, g = config.intermediate_size, config.hidden_size, nat.GATE_UP_GROUP
        gate = layer.gate_proj.reshape(i // g, g, h)
        up = layer.up_proj.reshape(i // g, g, h)
        self.w_gate_up = torch.stack((gate, up), dim=1).reshape(2 * i, h).contiguous()
        self.w_down = layer.down_proj.contiguous()
        # decode: the same weights in the tile layout the streaming kernels copy in contiguous 8 KB pieces
        self.t_qkv = decode_tiles(self.w_qkv)
        self.t_o = decode_tiles(self.w_o)
        self.t_gate_up = decode_tiles(layer.gate_proj.contiguous(), layer.up_proj.contiguous())
        self.t_down = decode_tiles(self.w_down)
        self.ptr = {name: getattr(self, name).data_ptr() for name in
                    ("in_norm", "post_norm", "q_norm", "k_norm", "w_qkv", "w_o", "w_gate_up", "w_down", "t_qkv",
                     "t_o", "t_gate_up", "t_down")}


class PackedModel:
    def __init__(self, loaded):
        c, w = loaded.config, loaded.weights
        check_supported(c)
        self.loaded = loaded
        self.config = c
        self.device = w.embed_tokens.device
        self.embed = w.embed_tokens.contiguous()
        self.lm_head = w.lm_head.contiguous()
        self.final_norm = w.norm.contiguous()
        with torch.no_grad():
            self.layers = [PackedLayer(layer, c) for layer in w.layers]
            self.t_lm_head = decode_tiles(self.lm_head)
        self.q_rows = c.num_attention_heads * c.head_dim
        self.kv_rows = c.num_key_value_heads * c.head_dim
        self.qkv_rows = self.q_rows + 2 * self.kv_rows
        layer_hook.register(self, torch.bfloat16)
        self._decode_cos: torch.Tensor | None = None
        self._decode_sin: torch.Tensor | None = None
        self._prefill_tables: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    def decode_rotary(self, capacity: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Per-position rows [capacity, D], each from its own one-position call."""
        have = 0 if self._decode_cos is None else self._decode_cos.shape[0]
        if have < capacity:
            c = self.config
            rows = [rotary_rows(torch.tensor([p]), c.head_dim, c.rope_theta) for p in range(have, capacity)]
            cos = torch.cat([r[0] for r in rows]).to(self.device)
            sin = torch.cat([r[1] for r in rows]).to(self.device)
            if self._decode_cos is not None:
                cos, sin = torch.cat((self._decode_cos, cos)), torch.cat((self._decode_sin, sin))
            self._decode_cos, self._decode_sin = cos.contiguous(), sin.contiguous()
        return self._decode_cos[:capacity], self._decode_sin[:capacity]

    def prefill_rotary(self, length: int) -> tuple[torch.Tensor, torch.Tensor]:
        """One call over positions 0..length-1, as the reference's prefill and uncached forward."""
        if length not in self._prefill_tables:
            if len(self._prefill_tables) > 8:
                self._prefill_tables.clear()
            c = self.config
            cos, sin = rotary_rows(torch.arange(length), c.head_dim, c.rope_theta)
            self._prefill_tables[length] = (cos.to(self.device).contiguous(), sin.to(self.device).contiguous())
        return self._prefill_tables[length]


_CACHE: list[tuple[object, PackedModel]] = []


def packed_model(loaded) -> PackedModel:
    """The packed layout of `loaded`, reused while the same LoadedCheckpoint object is in use."""
    for key, model in _CACHE:
        if key is loaded:
            return model
    model = PackedModel(loaded)
    _CACHE.clear()
    _CACHE.append((loaded, model))
    return model


def release_packed_models() -> None:
    _CACHE.clear()


class PrefillBuffers:
    """Activation buffers for a prompt of batch x length tokens (allocated per prompt size)."""

    def __init__(self, model: PackedModel, tokens: int, batch: int, length: int):
        c, dev, bf = model.config, model.device, torch.bfloat16
        self.tokens = tokens
        self.x = torch.empty((tokens, c.hidden_size), dtype=bf, device=dev)
        self.h = torch.empty((tokens, c.hidden_size), dtype=bf, device=dev)
        self.qkv = torch.empty((tokens, model.qkv_rows), dtype=bf, device=dev)
        self.q = torch.empty((batch, c.num_attention_heads, length, c.head_dim), dtype=bf, device=dev)
        self.attn = torch.empty((tokens, model.q_rows), dtype=bf, device=dev)
        self.act = torch.empty((tokens, c.intermediate_size), dtype=bf, device=dev)


def prefill_ops(c, p: dict[str, int], q_rows: int, qkv_rows: int, x: torch.Tensor, h: torch.Tensor, qkv: torch.Tensor,
                q: torch.Tensor, attn: torch.Tensor, act: torch.Tensor, k_layer: torch.Tensor, v_layer: torch.Tensor,
                batch: int, length: int, capacity: int, cos: torch.Tensor, sin: torch.Tensor, stream: int) -> None:
    """One decoder layer over a prompt at positions 0..length-1 (src/ipe/forward.py:86-115, start 0):
    p holds the packed layer's device pointers; x [batch*length, H] is updated in place."""
    lib = nat.load()
    m = batch * length
    hp, xp = h.data_ptr(), x.data_ptr()
    eps = c.rms_norm_eps
    nat.check(lib.ipe_rmsnorm(xp, p["in_norm"], hp, m, c.hidden_size, eps, 0, stream), "ipe_rmsnorm")
    nat.check(lib.ipe_gemm(hp, p["w_qkv"], qkv.data_ptr(), m, qkv_rows, c.hidden_size, nat.EPI_STORE, 0, stream),
              "ipe_gemm qkv")
    nat.check(lib.ipe_qk_norm_rope_append(qkv.data_ptr(), batch, length, c.num_attention_heads,
                                          c.num_key_value_heads, p["q_norm"], p["k_norm"], cos.data_ptr(),
                                          sin.data_ptr(), 0, None, q.data_ptr(), k_layer.data_ptr(),
                                          v_layer.data_ptr(), capacity, eps, stream), "ipe_qk_norm_rope_append")
    nat.check(lib.ipe_prefill_attention(q.data_ptr(), k_layer.data_ptr(), v_layer.data_ptr(), attn.data_ptr(),
                                        batch, c.num_attention_heads, c.num_key_value_heads, length, capacity, stream),
              "ipe_prefill_attention")
    nat.check(lib.ipe_gemm(attn.data_ptr(), p["w_o"], xp, m, c.hidden_size, q_rows, nat.EPI_RESIDUAL, xp, stream),
              "ipe_gemm o_proj")
    nat.check(lib.ipe_rmsnorm(xp, p["post_norm"], hp, m, c.hidden_size, eps, 0, stream), "ipe_rmsnorm")
    nat.check(lib.ipe_gemm(hp, p["w_gate_up"], act.data_ptr(), m, 2 * c.intermediate_size, c.hidden_size,
                           nat.EPI_SILU_MUL, 0, stream), "ipe_gemm gate_up")
    nat.check(lib.ipe_gemm(act.data_ptr(), p["w_down"], xp, m, c.hidden_size, c.intermediate_size,
                           nat.EPI_RESIDUAL, xp, stream), "ipe_gemm down_proj")


def prefill_layer(model: PackedModel, index: int, buf: PrefillBuffers, k_layer: torch.Tensor, v_layer: torch.Tensor,
                  batch: int, length: int, capacity: int, cos: torch.Tensor, sin: torch.Tensor, stream: int) -> None:
    """Layer `index` of the packed model over a prompt (prefill_ops on the engine's buffers)."""
    prefill_ops(model.config, model.layers[index].ptr, model.q_rows, model.qkv_rows, buf.x, buf.h, buf.qkv, buf.q,
                buf.attn, buf.act, k_layer, v_layer, batch, length, capacity, cos, sin, stream)


def run_prefill_layers(model: PackedModel, buf: PrefillBuffers, k: torch.Tensor, v: torch.Tensor, batch: int,
                       length: int, capacity: int, cos: torch.Tensor, sin: torch.Tensor) -> None:
    stream = torch.cuda.current_stream().cuda_stream
    for index in range(len(model.layers)):
        prefill_layer(model, index, buf, k[index], v[index], batch, length, capacity, cos, sin, stream)


class DecodeBuffers:
    """Fixed buffers of one decode step for up to `batch` rows; allocated once per engine."""

    def __init__(self, model: PackedModel, batch: int, capacity: int):
        c, dev, bf = model.config, model.device, torch.bfloat16
        self.x = torch.empty((batch, c.hidden_size), dtype=bf, device=dev)
        self.qkv = torch.empty((batch, model.qkv_rows), dtype=bf, device=dev)
        self.attn = torch.empty((batch, model.q_rows), dtype=bf, device=dev)
        self.act = torch.empty((batch, c.intermediate_size), dtype=bf, device=dev)
        self.logits = torch.empty((batch, c.vocab_size), dtype=torch.float32, device=dev)
        parts = int(nat.load().ipe_lm_head_parts(c.vocab_size))
        self.parts = parts
        self.partials = torch.empty((parts, batch, nat.PARTIAL_WORDS), dtype=torch.float32, device=dev)
        lib = nat.load()
        self.state = torch.zeros(nat.STATE_WORDS, dtype=torch.int64, device=dev)
        self.tokens = torch.zeros(batch, dtype=torch.int64, device=dev)
        # generation history: row b, sampled token s at [b, s] (fixed buffers, so captured steps replay)
        self.history_tokens = torch.zeros((batch, capacity), dtype=torch.int64, device=dev)
        self.history_logprobs = torch.zeros((batch, capacity), dtype=torch.float32, device=dev)
        step_ws = int(lib.ipe_decode_step_workspace(batch, c.num_attention_heads, c.num_key_value_heads, capacity))
        # grid barrier, attention arrival counters and partial records of the one-kernel decode step
        self.step_workspace = torch.zeros(step_ws, dtype=torch.uint8, device=dev)


def layer_descs(model: PackedModel, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """The device array of ipe_layer_desc for a cache pair k / v [layers, batch, kv_heads, capacity, 128]."""
    import ctypes

    descs = (nat.LayerDesc * len(model.layers))()
    for i, layer in enumerate(model.layers):
        p = layer.ptr
        fields = (p["in_norm"], p["post_norm"], p["q_norm"], p["k_norm"], p["t_qkv"], p["t_o"], p["t_gate_up"],
                  p["t_down"], k[i].data_ptr(), v[i].data_ptr())
        if any(f % 16 for f in fields):
            raise ValueError(f"layer {i}: the decode step needs 16-byte aligned operands")
        descs[i] = nat.LayerDesc(*fields)
    raw = torch.frombuffer(bytearray(ctypes.string_at(ctypes.addressof(descs), ctypes.sizeof(descs))),
                           dtype=torch.uint8)
    return raw.to(model.device)


def step_desc(model: PackedModel, buf: DecodeBuffers, descs: torch.Tensor, batch: int, capacity: int,
              cos: torch.Tensor, sin: torch.Tensor, sample: bool):
    """ipe_decode_step_desc of one decode step over the engine's fixed buffers."""
    c = model.config
    d = nat.StepDesc()
    d.layers, d.hidden, d.intermediate = c.num_hidden_layers, c.hidden_size, c.intermediate_size
    d.q_heads, d.kv_heads, d.vocab, d.capacity, d.batch = (c.num_attention_heads, c.num_key_value_heads,
                                                           c.vocab_size, capacity, batch)
    d.eps = c.rms_norm_eps
    d.vocab_total, d.tp_world = c.vocab_size, 1
    d.layer_descs = descs.data_ptr()
    d.embed, d.lm_head_tiles, d.final_norm = model.embed.data_ptr(), model.t_lm_head.data_ptr(), model.final_norm.data_ptr()
    d.cos_table, d.sin_table = cos.data_ptr(), sin.data_ptr()
    d.state, d.tokens = buf.state.data_ptr(), buf.tokens.data_ptr()
    d.x, d.qkv, d.attn, d.act = buf.x.data_ptr(), buf.qkv.data_ptr(), buf.attn.data_ptr(), buf.act.data_ptr()
    d.logits, d.partials = buf.logits.data_ptr(), buf.partials.data_ptr()
    d.workspace, d.workspace_bytes = buf.step_workspace.data_ptr(), buf.step_workspace.numel()
    if sample:
        d.history_tokens, d.history_logprobs = buf.history_tokens.data_ptr(), buf.history_logprobs.data_ptr()
        d.history_stride = buf.history_tokens.shape[1]
    return d
