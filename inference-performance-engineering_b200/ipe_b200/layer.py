"""One decoder layer with the reference's signature, on the per-operator CUDA kernels.

`decoder_layer(x, layer, rope, config, *, backend, cache=None, start=0)` is the function the
reference's engine calls once per layer (src/ipe/forward.py:86-115), with the same arguments,
return value and ValueError: x [B, T, H] (bf16 or fp32, on the GPU) at positions start..start+T-1,
`layer` the reference-layout LayerWeights, rope the (cos, sin) rows [T, 128] of those positions,
cache the layer's (K, V) [B, KV heads, capacity, 128] that receive this step's keys and values.
A prompt (start 0) attends causally to its own keys, a decode step (T = 1) to positions 0..start.

The engine's own steps do not call it: a decode step is one kernel replayed from a CUDA graph and
a prefill the fused per-layer launch chain. While `ipe_b200.engine.decoder_layer` is this function
the engine uses those; once a caller replaces the module global (to wrap, count or fail a layer,
as the reference's fault-injection tests do), the engine calls the replacement for every layer of
every step instead, and the replacement can call this function to do the layer's work. Each call
issues the kernels of one layer on the current stream:
- bf16, start 0: RMSNorm, tcgen05 QKV GEMM, q/k norm + RoPE + cache append, tcgen05 causal
  attention, o_proj / gate-up / down GEMMs with their residual and SiLU*up epilogues;
- bf16, decode: the weight-streaming RMSNorm+QKV, fused q/k norm + RoPE + append + split-KV
  attention, o_proj + residual, RMSNorm + gate/up + SiLU*up, down_proj + residual;
- fp32: the reference-precision kernels of ipe_b200.fp32.
The rope rows are used as given (a caller may pass rows of other positions). Buffers are cached
per shape; results are fresh tensors.
"""

from __future__ import annotations

import weakref

import torch

from ipe_b200 import _native as nat

_BF16, _F32 = torch.bfloat16, torch.float32

# Packed models (model.PackedModel, fp32.Fp32Model) register themselves here, weakly; a layer of a
# registered model is found by identity. A layer packed here for a caller without one is kept
# (with its source) in a short list.
_MODELS: list[tuple[weakref.ref, torch.dtype]] = []
_OWNED: list[tuple[object, object, torch.dtype]] = []


def register(model, dtype: torch.dtype) -> None:
    """Record a packed model (its `loaded` and `layers` attributes) for layer lookups."""
    _MODELS[:] = [(ref, dt) for ref, dt in _MODELS if ref() is not None]
    _MODELS.append((weakref.ref(model), dtype))


def _packed_layer(layer, config, dtype):
    for ref, dt in _MODELS:
        model = ref()
        if model is None or dt != dtype:
            continue
        for index, source in enumerate(model.loaded.weights.layers):
            if source is layer:
                return model.layers[index]
    for source, packed, dt in _OWNED:
        if source is layer and dt == dtype:
            return packed
    with torch.no_grad():
        if dtype == _F32:
            from ipe_b200.fp32 import Fp32Layer
            packed = Fp32Layer(layer, config)
        else:
            from ipe_b200.model import PackedLayer
            packed = PackedLayer(layer, config)
    _OWNED.append((layer, packed, dtype))
    del _OWNED[:-4]
    return packed


_BUFFERS: dict[tuple, dict[str, torch.Tensor]] = {}


def _buffers(key: tuple, make) -> dict[str, torch.Tensor]:
    buf = _BUFFERS.get(key)
    if buf is None:
        if len(_BUFFERS) > 16:
            _BUFFERS.clear()
        buf = _BUFFERS[key] = make()
    return buf


def decoder_layer(x: torch.Tensor, layer, rope: tuple[torch.Tensor, torch.Tensor], config, *, backend: str,
                  cache: tuple[torch.Tensor, torch.Tensor] | None = None, start: int = 0) -> torch.Tensor:
    """x + attention + SwiGLU of one pre-norm layer for x [B, T, H] (src/ipe/forward.py:86-115)."""
    from ipe_b200.forward import check_backend

    check_backend(backend)
    if start > 0 and x.shape[1] > 1:
        raise ValueError("decoder_layer: a step after position 0 takes one token; chunked prefill is not supported")
    if not isinstance(x, torch.Tensor) or x.dim() != 3 or x.shape[2] != config.hidden_size:
        raise ValueError(f"x: expected [B, T, {config.hidden_size}]")
    if x.dtype not in (_BF16, _F32) or x.device.type != "cuda":
        raise ValueError(f"x: the CUDA path takes bfloat16 or float32 CUDA tensors, got {x.dtype} on {x.device}")
    batch, length, hidden = x.shape
    kv, d = config.num_key_value_heads, config.head_dim
    if cache is None:
        if start != 0:
            raise ValueError("decoder_layer: a decode step needs the cache")
        shape = (batch, kv, length, d)
        cache = (torch.empty(shape, dtype=x.dtype, device=x.device), torch.empty(shape, dtype=x.dtype, device=x.device))
    k, v = cache
    capacity = k.shape[2]
    if (k.shape[0] < batch or k.shape[1:] != (kv, capacity, d) or v.shape != k.shape or k.dtype != x.dtype
            or not (k.is_contiguous() and v.is_contiguous())):
        raise ValueError("cache: expected contiguous (K, V) [B, KV heads, capacity, head_dim] of x's dtype")
    if start < 0 or start + length > capacity:
        raise ValueError(f"positions {start}..{start + length - 1} outside the cache's {capacity}")
    cos, sin = (t.to(device=x.device, dtype=x.dtype).contiguous() for t in rope)
    if cos.shape != (length, d) or sin.shape != (length, d):
        raise ValueError(f"rope: expected (cos, sin) [{length}, {d}]")
    # the kernels index the rotary table by position: place the given rows at start..start+T-1
    table = _buffers(("rope", x.dtype, capacity, x.device), lambda: {
        "cos": torch.zeros((capacity, d), dtype=x.dtype, device=x.device),
        "sin": torch.zeros((capacity, d), dtype=x.dtype, device=x.device)})
    table["cos"][start:start + length] = cos
    table["sin"][start:start + length] = sin
    packed = _packed_layer(layer, config, x.dtype)
    stream = torch.cuda.current_stream().cuda_stream
    if x.dtype == _F32:
        return _layer_f32(x, packed, config, k, v, start, capacity, table, stream)
    if start == 0:
        return _prefill_bf16(x, packed, config, k, v, capacity, table, stream)
    return _decode_bf16(x, packed, config, k, v, start, capacity, table, stream)


def _prefill_bf16(x, p, c, k, v, capacity, table, stream) -> torch.Tensor:
    from ipe_b200.model import prefill_ops

    batch, length, hidden = x.shape
    rows = batch * length
    q_rows, qkv_rows = c.num_attention_heads * c.head_dim, (c.num_attention_heads + 2 * c.num_key_value_heads) * c.head_dim
    buf = _buffers(("prefill", batch, length, x.device), lambda: {
        "x": torch.empty((rows, hidden), dtype=_BF16, device=x.device),
        "h": torch.empty((rows, hidden), dtype=_BF16, device=x.device),
        "qkv": torch.empty((rows, qkv_rows), dtype=_BF16, device=x.device),
        "q": torch.empty((batch, c.num_attention_heads, length, c.head_dim), dtype=_BF16, device=x.device),
        "attn": torch.empty((rows, q_rows), dtype=_BF16, device=x.device),
        "act": torch.empty((rows, c.intermediate_size), dtype=_BF16, device=x.device)})
    buf["x"].copy_(x.reshape(rows, hidden))
    prefill_ops(c, p.ptr, q_rows, qkv_rows, buf["x"], buf["h"], buf["qkv"], buf["q"], buf["attn"], buf["act"], k, v,
                batch, length, capacity, table["cos"], table["sin"], stream)
    return buf["x"].view(batch, length, hidden).clone()


def _decode_bf16(x, p, c, k, v, start, capacity, table, stream) -> torch.Tensor:
    lib = nat.load()
    batch, _, hidden = x.shape
    hq, hkv, eps = c.num_attention_heads, c.num_key_value_heads, c.rms_norm_eps
    q_rows, qkv_rows = hq * c.head_dim, (hq + 2 * hkv) * c.head_dim

    def make():
        linear = max(int(lib.ipe_decode_linear_workspace(batch, r, kk)) for r, kk in (
            (qkv_rows, hidden), (hidden, q_rows), (2 * c.intermediate_size, hidden), (hidden, c.intermediate_size)))
        return {"x": torch.empty((batch, hidden), dtype=_BF16, device=x.device),
                "qkv": torch.empty((batch, qkv_rows), dtype=_BF16, device=x.device),
                "attn": torch.empty((batch, q_rows), dtype=_BF16, device=x.device),
                "act": torch.empty((batch, c.intermediate_size), dtype=_BF16, device=x.device),
                "lws": torch.zeros(max(linear, 256), dtype=torch.uint8, device=x.device),
                "aws": torch.zeros(int(lib.ipe_decode_attention_qkv_workspace(batch, hq, hkv, capacity)),
                                   dtype=torch.uint8, device=x.device)}

    buf = _buffers(("decode", batch, capacity, x.device), make)
    buf["x"].copy_(x.reshape(batch, hidden))
    xp, lws, lwn = buf["x"].data_ptr(), buf["lws"].data_ptr(), buf["lws"].numel()
    ptr = p.ptr
    nat.check(lib.ipe_rmsnorm_qkv(xp, ptr["in_norm"], ptr["t_qkv"], buf["qkv"].data_ptr(), batch, hidden, qkv_rows,
                                  eps, lws, lwn, stream), "ipe_rmsnorm_qkv")
    nat.check(lib.ipe_decode_attention_qkv(buf["qkv"].data_ptr(), ptr["q_norm"], ptr["k_norm"],
                                           table["cos"].data_ptr(), table["sin"].data_ptr(), start, None,
                                           k.data_ptr(), v.data_ptr(), buf["attn"].data_ptr(), batch, hq, hkv,
                                           capacity, eps, buf["aws"].data_ptr(), buf["aws"].numel(), stream),
              "ipe_decode_attention_qkv")
    nat.check(lib.ipe_linear_residual(buf["attn"].data_ptr(), ptr["t_o"], xp, batch, q_rows, hidden, lws, lwn, stream),
              "ipe_linear_residual o_proj")
    nat.check(lib.ipe_rmsnorm_gate_up_silu(xp, ptr["post_norm"], ptr["t_gate_up"], buf["act"].data_ptr(), batch,
                                           hidden, c.intermediate_size, eps, lws, lwn, stream),
              "ipe_rmsnorm_gate_up_silu")
    nat.check(lib.ipe_linear_residual(buf["act"].data_ptr(), ptr["t_down"], xp, batch, c.intermediate_size, hidden,
                                      lws, lwn, stream), "ipe_linear_residual down_proj")
    return buf["x"].view(batch, 1, hidden).clone()


def _layer_f32(x, p, c, k, v, start, capacity, table, stream) -> torch.Tensor:
    from ipe_b200.fp32 import layer_ops

    batch, length, hidden = x.shape
    rows = batch * length
    q_rows, qkv_rows = c.num_attention_heads * c.head_dim, (c.num_attention_heads + 2 * c.num_key_value_heads) * c.head_dim
    buf = _buffers(("f32", batch, length, x.device), lambda: {
        "x": torch.empty((rows, hidden), dtype=_F32, device=x.device),
        "h": torch.empty((rows, hidden), dtype=_F32, device=x.device),
        "qkv": torch.empty((rows, qkv_rows), dtype=_F32, device=x.device),
        "q": torch.empty((batch, c.num_attention_heads, length, c.head_dim), dtype=_F32, device=x.device),
        "attn": torch.empty((rows, q_rows), dtype=_F32, device=x.device),
        "act": torch.empty((rows, c.intermediate_size), dtype=_F32, device=x.device)})
    buf["x"].copy_(x.reshape(rows, hidden))
    layer_ops(c, p, q_rows, qkv_rows, buf["x"], buf["h"], buf["qkv"], buf["q"], buf["attn"], buf["act"], k, v, batch,
              length, start, capacity, table["cos"], table["sin"], stream)
    return buf["x"].view(batch, length, hidden).clone()
