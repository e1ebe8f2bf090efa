"""Torch-facing operators over the C-ABI kernels.

Every function here takes CUDA tensors, checks dtype / shape / device / contiguity, and calls
exactly one entry point of libipe_b200.so on the current stream (no copies, no CPU path). The
same functions are registered as torch custom ops in the `ipe_b200` namespace
(`torch.ops.ipe_b200.<name>`), with out-tensors, so they compose with torch code and CUDA-graph
capture. The engine calls the plain functions, which skip the dispatcher.

Operators and the reference code each replaces (src/ipe/...):
  rms_norm                ops.py:23-33
  embed                   forward.py:125, engine.py:106
  rmsnorm_qkv             forward.py:100-103
  qk_norm_rope_append     forward.py:101-109, ops.py:36-63
  decode_attention        ops.py:78-101 (decode step)
  prefill_attention       ops.py:78-101 (prompt, causal)
  linear_residual         forward.py:113, :115
  rmsnorm_gate_up_silu    forward.py:114-115, ops.py:104-106
  lm_head_sample          engine.py:110-111, engine.py:28-41
  sample_logits           engine.py:28-41 (logits the caller holds)
  decode_tiles            (no counterpart) the decode-side weight layout the decode linears read
  gemm                    the prefill F.linear calls of forward.py:100-115 and forward.py:145-152
"""

from __future__ import annotations

import torch

from ipe_b200 import _native as nat


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
            raise ValueError("ipe_b200 operators take CUDA tensors")
        if not t.is_contiguous():
            raise ValueError("ipe_b200 operators take contiguous tensors")


def _bf16(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t.dtype != torch.bfloat16:
            raise ValueError(f"expected bfloat16, got {t.dtype}")


# ------------------------------------------------------------------------------------ functions

def rms_norm_out(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor) -> torch.Tensor:
    _cuda(x, weight, out)
    if x.dtype not in (torch.bfloat16, torch.float32) or weight.dtype != x.dtype or out.dtype != x.dtype:
        raise ValueError("rms_norm: x, weight and out must share dtype bfloat16 or float32")
    width = x.shape[-1]
    if weight.shape != (width,) or out.shape != x.shape:
        raise ValueError("rms_norm: shape mismatch")
    nat.call("ipe_rmsnorm", x.data_ptr(), weight.data_ptr(), out.data_ptr(), x.numel() // max(width, 1), width,
             float(eps), 0 if x.dtype == torch.bfloat16 else 1, _stream())
    return out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm with fp32 statistics and the reference's two roundings (src/ipe/ops.py:23-33)."""
    return rms_norm_out(x, weight, eps, torch.empty_like(x))


def embed(ids: torch.Tensor, table: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    _cuda(ids, table, out)
    _bf16(table, out)
    if ids.dtype != torch.int64:
        raise ValueError("embed: ids must be int64")
    nat.call("ipe_embed", ids.data_ptr(), ids.numel(), table.data_ptr(), table.shape[0], table.shape[1],
             out.data_ptr(), _stream())
    return out


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, epilogue: int = nat.EPI_STORE,
         residual: torch.Tensor | None = None, m: int | None = None) -> torch.Tensor:
    """out = epilogue(a[:m] @ b^T) on tcgen05 tensor cores; a [M, K], b [N, K] bf16."""
    _cuda(a, b, out)
    _bf16(a, b)
    rows = a.shape[0] if m is None else m
    n, k = b.shape
    if a.shape[1] != k:
        raise ValueError(f"gemm: a has {a.shape[1]} columns, b has {k}")
    expected_cols = n // 2 if epilogue == nat.EPI_SILU_MUL else n
    if out.shape[-1] != expected_cols or out.numel() < rows * expected_cols:
        raise ValueError("gemm: output shape")
    if epilogue == nat.EPI_LOGITS:
        if out.dtype != torch.float32:
            raise ValueError("gemm: logits epilogue writes float32")
    else:
        _bf16(out)
    res = 0
    if epilogue == nat.EPI_RESIDUAL:
        if residual is None:
            raise ValueError("gemm: residual epilogue needs a residual")
        _cuda(residual)
        _bf16(residual)
        res = residual.data_ptr()
    nat.call("ipe_gemm", a.data_ptr(), b.data_ptr(), out.data_ptr(), rows, n, k, int(epilogue), res, _stream())
    return out


def sample_logits(logits: torch.Tensor, temperature: float, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Tokens [B] int64 and untempered log-probabilities [B] fp32 from logits [B, V] fp32."""
    _cuda(logits)
    if logits.dtype != torch.float32 or logits.dim() != 2:
        raise ValueError("sample: logits must be float32 [B, V]")
    rows, vocab = logits.shape
    tokens = torch.empty(rows, dtype=torch.int64, device=logits.device)
    logprobs = torch.empty(rows, dtype=torch.float32, device=logits.device)
    nat.call("ipe_sample_logits", logits.data_ptr(), rows, vocab, float(temperature), int(seed) & (2**64 - 1),
             tokens.data_ptr(), logprobs.data_ptr(), _stream())
    return tokens, logprobs


# Zero-filled scratch of the kernels that split work across CTAs (their counters end every call at
# zero), one buffer per device and size. Calls share it, so they must stay on one stream, as the
# reference's engine does (src/ipe/engine.py:6).
_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def _workspace(device: torch.device, size: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(), int(size))
    ws = _workspaces.get(key)
    if ws is None:
        ws = _workspaces[key] = torch.zeros(max(int(size), 256), dtype=torch.uint8, device=device)
    return ws


def decode_tiles(w: torch.Tensor, w_up: torch.Tensor | None = None) -> torch.Tensor:
    """The decode-tile layout of a weight [rows, in] (or of the gate/up pair) as a uint8 tensor:
    the weight operand of rmsnorm_qkv, linear_residual, rmsnorm_gate_up_silu and lm_head_sample."""
    _cuda(w)
    _bf16(w)
    rows, k = w.shape
    if w_up is not None:
        _cuda(w_up)
        _bf16(w_up)
        if w_up.shape != w.shape:
            raise ValueError("decode_tiles: gate and up shapes differ")
    size = int(nat.load().ipe_decode_tiles_bytes(rows, k, 1 if w_up is not None else 0))
    tiles = torch.empty(size, dtype=torch.uint8, device=w.device)
    nat.call("ipe_decode_tiles", w.data_ptr(), w_up.data_ptr() if w_up is not None else None, tiles.data_ptr(), rows,
             k, _stream())
    return tiles


def _linear_ws(x: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    return _workspace(x.device, int(nat.load().ipe_decode_linear_workspace(x.shape[0], rows, k)))


def rmsnorm_qkv(x: torch.Tensor, norm_weight: torch.Tensor, w_qkv_tiles: torch.Tensor, eps: float,
                out: torch.Tensor) -> torch.Tensor:
    """out [B, rows] = rms_norm(x [B, H]) @ W_qkv^T (src/ipe/forward.py:100-103), one row per token."""
    _cuda(x, norm_weight, w_qkv_tiles, out)
    _bf16(x, norm_weight, out)
    batch, hidden = x.shape
    rows = out.shape[1]
    if out.shape[0] != batch or norm_weight.shape != (hidden,):
        raise ValueError("rmsnorm_qkv: shape mismatch")
    ws = _linear_ws(x, rows, hidden)
    nat.call("ipe_rmsnorm_qkv", x.data_ptr(), norm_weight.data_ptr(), w_qkv_tiles.data_ptr(), out.data_ptr(), batch,
             hidden, rows, float(eps), ws.data_ptr(), ws.numel(), _stream())
    return out


def linear_residual(a: torch.Tensor, w_tiles: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """x [B, N] = bf16(x + bf16(a [B, K] @ W^T)) in place (src/ipe/forward.py:113, :115)."""
    _cuda(a, w_tiles, x)
    _bf16(a, x)
    batch, k = a.shape
    if x.shape[0] != batch:
        raise ValueError("linear_residual: batch mismatch")
    ws = _linear_ws(a, x.shape[1], k)
    nat.call("ipe_linear_residual", a.data_ptr(), w_tiles.data_ptr(), x.data_ptr(), batch, k, x.shape[1],
             ws.data_ptr(), ws.numel(), _stream())
    return x


def rmsnorm_gate_up_silu(x: torch.Tensor, norm_weight: torch.Tensor, w_gate_up_tiles: torch.Tensor, eps: float,
                         out: torch.Tensor) -> torch.Tensor:
    """out [B, I] = silu(rms_norm(x) @ gate^T) * (rms_norm(x) @ up^T) with the reference's roundings
    (src/ipe/forward.py:114-115, src/ipe/ops.py:104-106)."""
    _cuda(x, norm_weight, w_gate_up_tiles, out)
    _bf16(x, norm_weight, out)
    batch, hidden = x.shape
    inter = out.shape[1]
    if out.shape[0] != batch or norm_weight.shape != (hidden,):
        raise ValueError("rmsnorm_gate_up_silu: shape mismatch")
    ws = _linear_ws(x, 2 * inter, hidden)
    nat.call("ipe_rmsnorm_gate_up_silu", x.data_ptr(), norm_weight.data_ptr(), w_gate_up_tiles.data_ptr(),
             out.data_ptr(), batch, hidden, inter, float(eps), ws.data_ptr(), ws.numel(), _stream())
    return out


def qk_norm_rope_append(qkv: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor, cos: torch.Tensor,
                        sin: torch.Tensor, start: int, eps: float, q_out: torch.Tensor, k_cache: torch.Tensor,
                        v_cache: torch.Tensor) -> torch.Tensor:
    """q/k RMSNorm per head, RoPE at positions start.., and the K/V cache append
    (src/ipe/forward.py:101-109, src/ipe/ops.py:36-63). qkv [B*T, (Hq+2Hkv)*128] bf16; q_out
    [B, Hq, T, 128]; caches [B, Hkv, capacity, 128]; cos/sin [>= start+T, 128]."""
    _cuda(qkv, q_norm, k_norm, cos, sin, q_out, k_cache, v_cache)
    _bf16(qkv, q_norm, k_norm, cos, sin, q_out, k_cache, v_cache)
    batch, q_heads, tokens, d = q_out.shape
    _, kv_heads, capacity, _ = k_cache.shape
    if d != 128 or qkv.shape != (batch * tokens, (q_heads + 2 * kv_heads) * 128) or v_cache.shape != k_cache.shape:
        raise ValueError("qk_norm_rope_append: shape mismatch")
    nat.call("ipe_qk_norm_rope_append", qkv.data_ptr(), batch, tokens, q_heads, kv_heads, q_norm.data_ptr(),
             k_norm.data_ptr(), cos.data_ptr(), sin.data_ptr(), int(start), None, q_out.data_ptr(),
             k_cache.data_ptr(), v_cache.data_ptr(), capacity, float(eps), _stream())
    return q_out


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, length: int,
                     out: torch.Tensor) -> torch.Tensor:
    """out [B, Hq*128] = softmax(q k^T / sqrt(128)) v over keys 0..length-1 of the caches, GQA, one
    query token per row (src/ipe/ops.py:78-101, decode). q [B, Hq, 128]."""
    _cuda(q, k_cache, v_cache, out)
    _bf16(q, k_cache, v_cache, out)
    batch, q_heads, _ = q.shape
    _, kv_heads, capacity, _ = k_cache.shape
    ws = _workspace(q.device, decode_attention_workspace(batch, q_heads, capacity))
    nat.call("ipe_decode_attention", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), batch,
             q_heads, kv_heads, capacity, int(length), None, ws.data_ptr(), ws.numel(), _stream())
    return out


def prefill_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """Causal attention of the prompt's queries q [B, Hq, T, 128] over cache positions 0..T-1:
    out [B, T, Hq*128] (src/ipe/ops.py:78-101, prefill)."""
    _cuda(q, k_cache, v_cache, out)
    _bf16(q, k_cache, v_cache, out)
    batch, q_heads, tokens, _ = q.shape
    _, kv_heads, capacity, _ = k_cache.shape
    nat.call("ipe_prefill_attention", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), batch,
             q_heads, kv_heads, tokens, capacity, _stream())
    return out


def lm_head_sample(x: torch.Tensor, norm_weight: torch.Tensor, lm_tiles: torch.Tensor, eps: float,
                   temperature: float, seed: int, logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Final RMSNorm of x [B, H], tied LM head into fp32 logits [B, V] (bf16-rounded, as
    src/ipe/engine.py:110-111), then the sampler of src/ipe/engine.py:28-41 in one more kernel:
    tokens [B] int64 and untempered log-probabilities [B] fp32."""
    _cuda(x, norm_weight, lm_tiles, logits)
    _bf16(x, norm_weight)
    if logits.dtype != torch.float32:
        raise ValueError("lm_head_sample: logits must be float32")
    batch, hidden = x.shape
    vocab = logits.shape[1]
    parts = lm_head_parts(vocab)
    partials = torch.empty((parts, batch, nat.PARTIAL_WORDS), dtype=torch.float32, device=x.device)
    tokens = torch.empty(batch, dtype=torch.int64, device=x.device)
    logprobs = torch.empty(batch, dtype=torch.float32, device=x.device)
    seed = int(seed) & (2**64 - 1)
    nat.call("ipe_lm_head", x.data_ptr(), hidden, norm_weight.data_ptr(), lm_tiles.data_ptr(), logits.data_ptr(),
             partials.data_ptr(), batch, hidden, vocab, float(eps), float(temperature), seed, None, _stream())
    nat.call("ipe_sample", partials.data_ptr(), logits.data_ptr(), batch, vocab, float(temperature), None,
             tokens.data_ptr(), logprobs.data_ptr(), 1, None, _stream())
    return tokens, logprobs


def decode_attention_workspace(batch: int, q_heads: int, capacity: int) -> int:
    return int(nat.load().ipe_decode_attention_workspace(batch, q_heads, capacity))


def lm_head_parts(vocab: int) -> int:
    return int(nat.load().ipe_lm_head_parts(vocab))


# --------------------------------------------------------------------------- torch custom ops

_lib = torch.library.Library("ipe_b200", "DEF")
_lib.define("rms_norm(Tensor x, Tensor weight, float eps, Tensor(a!) out) -> ()")
_lib.define("gemm(Tensor a, Tensor b, Tensor(a!) out, int epilogue, Tensor? residual) -> ()")
_lib.define("embed(Tensor ids, Tensor table, Tensor(a!) out) -> ()")
_lib.define("sample_logits(Tensor logits, float temperature, int seed) -> (Tensor, Tensor)")
_lib.define("decode_tiles(Tensor w, Tensor? w_up) -> Tensor")
_lib.define("rmsnorm_qkv(Tensor x, Tensor norm_weight, Tensor w_qkv_tiles, float eps, Tensor(a!) out) -> ()")
_lib.define("linear_residual(Tensor a, Tensor w_tiles, Tensor(a!) x) -> ()")
_lib.define("rmsnorm_gate_up_silu(Tensor x, Tensor norm_weight, Tensor w_gate_up_tiles, float eps, Tensor(a!) out) -> ()")
_lib.define("qk_norm_rope_append(Tensor qkv, Tensor q_norm, Tensor k_norm, Tensor cos, Tensor sin, int start, "
            "float eps, Tensor(a!) q_out, Tensor(b!) k_cache, Tensor(c!) v_cache) -> ()")
_lib.define("decode_attention(Tensor q, Tensor k_cache, Tensor v_cache, int length, Tensor(a!) out) -> ()")
_lib.define("prefill_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor(a!) out) -> ()")
_lib.define("lm_head_sample(Tensor x, Tensor norm_weight, Tensor lm_tiles, float eps, float temperature, int seed, "
            "Tensor(a!) logits) -> (Tensor, Tensor)")


def _op_rms_norm(x, weight, eps, out):
    rms_norm_out(x, weight, eps, out)


def _op_gemm(a, b, out, epilogue, residual):
    gemm(a, b, out, epilogue, residual)


def _op_embed(ids, table, out):
    embed(ids, table, out)


_lib.impl("rms_norm", _op_rms_norm, "CUDA")
_lib.impl("gemm", _op_gemm, "CUDA")
_lib.impl("embed", _op_embed, "CUDA")
_lib.impl("sample_logits", sample_logits, "CUDA")
_lib.impl("decode_tiles", decode_tiles, "CUDA")
_lib.impl("lm_head_sample", lm_head_sample, "CUDA")


def _returns_none(fn):
    """The out-variant op implementations return nothing (their schemas end in `-> ()`)."""

    def op(*args):
        fn(*args)

    return op


for _name, _fn in (("rmsnorm_qkv", rmsnorm_qkv), ("linear_residual", linear_residual),
                   ("rmsnorm_gate_up_silu", rmsnorm_gate_up_silu), ("qk_norm_rope_append", qk_norm_rope_append),
                   ("decode_attention", decode_attention), ("prefill_attention", prefill_attention)):
    _lib.impl(_name, _returns_none(_fn), "CUDA")
