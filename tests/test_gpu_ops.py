"""The torch custom ops (`torch.ops.ipe_b200.*`) of the decode and attention kernels, each called
through the dispatcher and checked against a PyTorch fp32 computation of the same operator."""

import pytest
import torch

import ipe_b200.ops  # noqa: F401  (registers the ops)
from ipe_b200 import _native as nat
from oracle import qwen3 as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"
REL = 2.0 ** -7
OPS = torch.ops.ipe_b200


def rand(shape, seed, scale=1.0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype).to(DEV)


def close(actual, expected, rel, abs_):
    a, e = actual.float(), expected.float()
    return int(((a - e).abs() > rel * e.abs() + abs_).sum())


def rms(x, w, eps):
    """The reference's RMSNorm roundings: bf16(w * bf16(x * rsqrt(mean(x^2) + eps)))."""
    xf = x.float()
    h = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).bfloat16()
    return (w.float() * h.float()).bfloat16()


@pytest.mark.parametrize("batch", [1, 3, 16])
def test_rmsnorm_qkv_op(batch):
    hidden, rows, eps = 1024, 1536, 1e-6
    x, w = rand((batch, hidden), 1), (1 + 0.1 * rand((hidden,), 2, dtype=torch.float32)).bfloat16()
    weight = rand((rows, hidden), 3, hidden ** -0.5)
    out = torch.empty((batch, rows), dtype=torch.bfloat16, device=DEV)
    OPS.rmsnorm_qkv(x, w, OPS.decode_tiles(weight, None), eps, out)
    ref = rms(x, w, eps).float() @ weight.float().T
    assert close(out, ref, 2 * REL, 2e-3) == 0


@pytest.mark.parametrize("batch", [1, 5])
def test_linear_residual_op(batch):
    k, n = 2048, 1024
    a, weight = rand((batch, k), 4), rand((n, k), 5, k ** -0.5)
    x = rand((batch, n), 6)
    before = x.clone()
    OPS.linear_residual(a, OPS.decode_tiles(weight, None), x)
    acc = a.float() @ weight.float().T
    ref = before.float() + acc.bfloat16().float()
    assert ((x.float() - ref).abs() <= 2 * REL * (acc.abs() + before.float().abs()) + 1e-3).all()


def test_rmsnorm_gate_up_silu_op():
    batch, hidden, inter, eps = 2, 1024, 768, 1e-6
    x, w = rand((batch, hidden), 7), (1 + 0.1 * rand((hidden,), 8, dtype=torch.float32)).bfloat16()
    gate, up = rand((inter, hidden), 9, hidden ** -0.5), rand((inter, hidden), 10, hidden ** -0.5)
    out = torch.empty((batch, inter), dtype=torch.bfloat16, device=DEV)
    OPS.rmsnorm_gate_up_silu(x, w, OPS.decode_tiles(gate, up), eps, out)
    h = rms(x, w, eps).float()
    g, u = (h @ gate.float().T).bfloat16().float(), (h @ up.float().T).bfloat16().float()
    ref = torch.nn.functional.silu(g).bfloat16().float() * u
    assert close(out, ref, 3 * REL, 2e-3) == 0


def test_qk_norm_rope_append_op():
    batch, hq, hkv, tokens, cap, start, eps = 2, 8, 2, 5, 16, 3, 1e-6
    qkv = rand((batch * tokens, (hq + 2 * hkv) * 128), 11)
    qn, kn = rand((128,), 12), rand((128,), 13)
    cos, sin = (t.to(DEV) for t in oq.rotary_tables(torch.arange(cap), 128, 1e6, torch.bfloat16))
    q = torch.empty((batch, hq, tokens, 128), dtype=torch.bfloat16, device=DEV)
    k = torch.zeros((batch, hkv, cap, 128), dtype=torch.bfloat16, device=DEV)
    v = torch.zeros_like(k)
    OPS.qk_norm_rope_append(qkv, qn, kn, cos, sin, start, eps, q, k, v)
    split = qkv.view(batch, tokens, hq + 2 * hkv, 128)
    rows = slice(start, start + tokens)
    q_ref = oq.apply_rotary(oq.qk_norm(split[:, :, :hq], qn, eps).transpose(1, 2), cos[rows], sin[rows])
    k_ref = oq.apply_rotary(oq.qk_norm(split[:, :, hq:hq + hkv], kn, eps).transpose(1, 2), cos[rows], sin[rows])
    assert close(q, q_ref, REL, 1e-6) == 0 and close(k[:, :, rows], k_ref, REL, 1e-6) == 0
    assert torch.equal(v[:, :, rows], split[:, :, hq + hkv:].transpose(1, 2))


def attention_ref(q, k, v, causal):
    groups = q.shape[1] // k.shape[1]
    k, v = k.float().repeat_interleave(groups, 1), v.float().repeat_interleave(groups, 1)
    s = (q.float() @ k.transpose(-1, -2)) * 128 ** -0.5
    if causal:
        t = q.shape[2]
        s = s.masked_fill(torch.ones(t, t, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    return torch.softmax(s, -1) @ v


@pytest.mark.parametrize(("batch", "length"), [(1, 1), (2, 77), (4, 600)])
def test_decode_attention_op(batch, length):
    hq, hkv, cap = 16, 8, 640
    q = rand((batch, hq, 128), 14)
    k, v = rand((batch, hkv, cap, 128), 15), rand((batch, hkv, cap, 128), 16)
    out = torch.empty((batch, hq * 128), dtype=torch.bfloat16, device=DEV)
    for _ in range(2):  # the second call reuses the workspace the first left at zero
        OPS.decode_attention(q, k, v, length, out)
    ref = attention_ref(q[:, :, None], k[:, :, :length], v[:, :, :length], False).reshape(batch, hq * 128)
    assert close(out, ref, 2 * REL, 2e-3) == 0
    assert nat.device_error() == 0


def test_prefill_attention_op():
    batch, hq, hkv, tokens, cap = 2, 8, 4, 100, 128
    q = rand((batch, hq, tokens, 128), 17)
    k, v = rand((batch, hkv, cap, 128), 18), rand((batch, hkv, cap, 128), 19)
    out = torch.empty((batch, tokens, hq * 128), dtype=torch.bfloat16, device=DEV)
    OPS.prefill_attention(q, k, v, out)
    ref = attention_ref(q, k[:, :, :tokens], v[:, :, :tokens], True).transpose(1, 2).reshape(batch, tokens, hq * 128)
    assert close(out, ref, 3 * REL, 4e-3) == 0


def test_lm_head_sample_op_greedy_and_logprobs():
    batch, hidden, vocab, eps = 3, 1024, 4096, 1e-6
    x, w = rand((batch, hidden), 20), (1 + 0.1 * rand((hidden,), 21, dtype=torch.float32)).bfloat16()
    table = rand((vocab, hidden), 22, hidden ** -0.5)
    logits = torch.empty((batch, vocab), dtype=torch.float32, device=DEV)
    tokens, logprobs = OPS.lm_head_sample(x, w, OPS.decode_tiles(table, None), eps, 0.0, 0, logits)
    ref = (rms(x, w, eps).float() @ table.float().T).bfloat16().float()
    assert close(logits, ref, 2 * REL, 1e-3) == 0
    assert torch.equal(tokens, logits.argmax(-1))
    expected = torch.log_softmax(logits.double(), -1).gather(-1, tokens[:, None]).squeeze(-1)
    assert torch.allclose(logprobs.double(), expected, atol=1e-4, rtol=0)
