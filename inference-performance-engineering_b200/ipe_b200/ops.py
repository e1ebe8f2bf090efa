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
  lm_head / sample        engine.py:110-111, engine.py:28-41
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
