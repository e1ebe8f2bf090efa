"""Each CUDA kernel through the C-ABI against a plain PyTorch fp32 computation of the same op.

Tolerances are stated per test: bf16 outputs may differ from the correctly rounded fp32 value by
the rounding of a differently ordered fp32 sum, i.e. about one bf16 ulp (2^-8 relative to the
value, 2^-7 to be safe) plus a small absolute term for values near zero.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from ipe_b200 import _native as nat
from ipe_b200 import ops
from oracle import qwen3 as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16_REL = 2.0 ** -7


def bf16_close(actual, expected, rel=BF16_REL, abs_=1e-4):
    a, e = actual.float(), expected.float()
    bad = (a - e).abs() > rel * e.abs() + abs_
    return int(bad.sum()), float((a - e).abs().max())


def stream():
    return torch.cuda.current_stream().cuda_stream


def no_device_error():
    assert nat.device_error(reset=True) == 0


def tiles(w, w_up=None):
    """Decode tiles of a weight (or a gate/up pair) through the C-ABI tile builder."""
    from ipe_b200.model import decode_tiles

    return decode_tiles(w.contiguous(), None if w_up is None else w_up.contiguous())


def linear_workspace(batch, rows, k):
    """A zero-filled split-K workspace for the decode linear kernels (they keep it zeroed)."""
    n = int(nat.load().ipe_decode_linear_workspace(batch, rows, k))
    return torch.zeros(max(n, 16), dtype=torch.uint8, device=DEV)


# ----------------------------------------------------------------------------------- rms_norm

def contract_inputs(width, dtype, seed=0):
    """Rows of N(0, s^2) for s from 1e-4 to 100, outlier rows and a zero row (the reference's
    operator contract inputs, tests/needs_torch/test_rms_norm.py:30-42)."""
    g = torch.Generator().manual_seed(seed)
    scales = torch.tensor([1e-4, 1e-3, 3e-3, 1e-2, 0.1, 1.0, 1.0, 1.0, 10.0, 100.0], dtype=torch.float64)
    x = torch.randn((len(scales) * 4, width), generator=g, dtype=torch.float64) * scales.repeat(4)[:, None]
    x[-4:-1, 0] *= 300
    x[-2, width // 2] *= 50
    x[-1] = 0
    w = 1 + 0.2 * torch.randn(width, generator=g, dtype=torch.float64)
    w[:: max(width // 8, 1)] *= 20
    return x.to(dtype), w.to(dtype)


def contract_violations(actual, x, w, eps, dtype, width):
    """Elements outside the contract (tests/needs_torch/test_rms_norm.py:50-59): bf16 within 1.5
    ulp of the exact value; fp32 within (n/2 + 5) * 2^-24 relative; zero rows exactly zero."""
    xd, wd = x.double(), w.double()
    exact = wd * xd / torch.sqrt(xd.pow(2).mean(-1, keepdim=True) + eps)
    actual = actual.double()
    if dtype == torch.bfloat16:
        _, exponent = np.frexp(exact.abs().numpy())
        bound = torch.from_numpy(1.5 * np.ldexp(1.0, exponent - 8))
    else:
        bound = (width / 2 + 5) * 2.0 ** -24 * exact.abs()
    return int(((actual - exact).abs() > bound).sum()) + int((actual[exact == 0] != 0).sum())


@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float32))
@pytest.mark.parametrize("width", (8, 128, 1000, 2048))
def test_rms_norm_meets_the_exact_value_contract(dtype, width):
    x, w = contract_inputs(width, dtype)
    out = ops.rms_norm(x.to(DEV), w.to(DEV), 1e-6).cpu()
    assert contract_violations(out, x, w, 1e-6, dtype, width) == 0


def test_rms_norm_is_a_registered_torch_op():
    x, w = contract_inputs(128, torch.bfloat16)
    out = torch.empty_like(x, device=DEV)
    torch.ops.ipe_b200.rms_norm(x.to(DEV), w.to(DEV), 1e-6, out)
    assert contract_violations(out.cpu(), x, w, 1e-6, torch.bfloat16, 128) == 0


# --------------------------------------------------------------------------------------- GEMM

def rand(shape, seed, scale=1.0, dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * scale).to(dtype).to(DEV)


GEMM_SHAPES = [(1, 128, 64), (100, 256, 128), (128, 384, 192), (512, 4096, 2048), (300, 2048, 6144),
               (1000, 12288, 2048), (4096, 2048, 2048), (2, 151936, 1024)]


@pytest.mark.parametrize(("m", "n", "k"), GEMM_SHAPES)
def test_gemm_store_matches_fp32(m, n, k):
    a, b = rand((m, k), 1), rand((n, k), 2, 1 / k ** 0.5)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=DEV)
    ops.gemm(a, b, out, nat.EPI_STORE)
    ref = a.float() @ b.float().T
    assert bf16_close(out, ref) [0] == 0
    no_device_error()


@pytest.mark.parametrize(("m", "n", "k"), [(77, 256, 512), (512, 2048, 6144), (1024, 2048, 2048)])
def test_gemm_residual_matches_fp32(m, n, k):
    a, b, r = rand((m, k), 3), rand((n, k), 4, 1 / k ** 0.5), rand((m, n), 5)
    out = r.clone()
    ops.gemm(a, b, out, nat.EPI_RESIDUAL, residual=out)
    acc = a.float() @ b.float().T
    ref = r.float() + acc.bfloat16().float()
    # a one-ulp flip of the rounded product plus the half-ulp rounding of the sum, relative to the
    # operands rather than the (possibly cancelling) result
    bound = 2 * BF16_REL * (acc.abs() + r.float().abs()) + 1e-3
    assert int(((out.float() - ref).abs() > bound).sum()) == 0


@pytest.mark.parametrize(("m", "inter", "k"), [(64, 128, 256), (333, 512, 256), (512, 6144, 2048)])
def test_gemm_silu_mul_matches_fp32(m, inter, k):
    a = rand((m, k), 6)
    gate, up = rand((inter, k), 7, 1 / k ** 0.5), rand((inter, k), 8, 1 / k ** 0.5)
    g = nat.GATE_UP_GROUP
    packed = torch.stack((gate.view(inter // g, g, k), up.view(inter // g, g, k)), 1).reshape(2 * inter, k).contiguous()
    out = torch.empty((m, inter), dtype=torch.bfloat16, device=DEV)
    ops.gemm(a, packed, out, nat.EPI_SILU_MUL)
    gv = (a.float() @ gate.float().T).bfloat16()
    uv = (a.float() @ up.float().T).bfloat16()
    ref = (F.silu(gv) * uv).float()
    assert bf16_close(out, ref, rel=3 * BF16_REL, abs_=2e-3)[0] == 0


def test_gemm_logits_are_bf16_values_widened():
    a, b = rand((37, 1024), 9), rand((2048, 1024), 10, 0.03)
    out = torch.empty((37, 2048), dtype=torch.float32, device=DEV)
    ops.gemm(a, b, out, nat.EPI_LOGITS)
    assert torch.equal(out, out.bfloat16().float())
    assert bf16_close(out, a.float() @ b.float().T)[0] == 0


# ------------------------------------------------------------------------------ decode GEMVs

def rmsnorm_ref(x, w, eps):
    return oq.rms_norm(x, w, eps)


@pytest.mark.parametrize("batch", (1, 3, 8, 16))
@pytest.mark.parametrize(("hidden", "rows"), [(2048, 4096), (1024, 4096), (256, 1024)])
def test_rmsnorm_qkv_matches_fp32(batch, hidden, rows):
    x, w = rand((batch, hidden), 11), (1 + 0.1 * rand((hidden,), 12, dtype=torch.float32)).bfloat16()
    wq = rand((rows, hidden), 13, 0.02)
    out = torch.empty((batch, rows), dtype=torch.bfloat16, device=DEV)
    ws = linear_workspace(batch, rows, hidden)
    tq = tiles(wq)
    for _ in range(2):  # the second call reuses the workspace its first call left zeroed
        nat.call("ipe_rmsnorm_qkv", x.data_ptr(), w.data_ptr(), tq.data_ptr(), out.data_ptr(), batch, hidden, rows,
                 1e-6, ws.data_ptr(), ws.numel(), stream())
    assert int(ws[: 4 * ((rows + 31) // 32)].count_nonzero()) == 0  # arrival counters back at zero
    ref = rmsnorm_ref(x, w, 1e-6).float() @ wq.float().T
    assert bf16_close(out, ref, rel=2 * BF16_REL, abs_=1e-3)[0] == 0
    no_device_error()


def test_decode_linear_layers_can_share_one_workspace():
    """Qwen3-1.7B shapes, one workspace for all four decode linear layers in turn, twice: every
    call must match the same call on a fresh workspace bit for bit."""
    batch, hidden, inter = 2, 2048, 6144
    x = rand((batch, hidden), 50)
    nw = (1 + 0.1 * rand((hidden,), 51, dtype=torch.float32)).bfloat16()
    wq, wo = tiles(rand((4096, hidden), 52, 0.02)), tiles(rand((hidden, 2048), 53, 0.02))
    wgu = tiles(rand((inter, hidden), 54, 0.02), rand((inter, hidden), 55, 0.02))
    wd = tiles(rand((hidden, inter), 56, 0.02))
    need = max(int(nat.load().ipe_decode_linear_workspace(batch, r, k))
               for r, k in ((4096, hidden), (hidden, 2048), (2 * inter, hidden), (hidden, inter)))
    shared = torch.zeros(need, dtype=torch.uint8, device=DEV)

    def run(ws):
        qkv = torch.empty((batch, 4096), dtype=torch.bfloat16, device=DEV)
        act = torch.empty((batch, inter), dtype=torch.bfloat16, device=DEV)
        y = x.clone()
        p = (ws.data_ptr(), ws.numel(), stream())
        nat.call("ipe_rmsnorm_qkv", y.data_ptr(), nw.data_ptr(), wq.data_ptr(), qkv.data_ptr(), batch, hidden, 4096,
                 1e-6, *p)
        nat.call("ipe_linear_residual", qkv.data_ptr(), wo.data_ptr(), y.data_ptr(), batch, 2048, hidden, *p)
        nat.call("ipe_rmsnorm_gate_up_silu", y.data_ptr(), nw.data_ptr(), wgu.data_ptr(), act.data_ptr(), batch, hidden,
                 inter, 1e-6, *p)
        nat.call("ipe_linear_residual", act.data_ptr(), wd.data_ptr(), y.data_ptr(), batch, inter, hidden, *p)
        return qkv, act, y

    fresh = [run(torch.zeros(need, dtype=torch.uint8, device=DEV)) for _ in range(1)][0]
    for _ in range(2):
        for a, b in zip(run(shared), fresh):
            assert torch.equal(a, b)


@pytest.mark.parametrize("batch", (1, 4, 16))
@pytest.mark.parametrize(("k", "n"), [(2048, 2048), (6144, 2048), (3072, 1024), (512, 256)])
def test_linear_residual_matches_fp32(batch, k, n):
    a, w, x = rand((batch, k), 14), rand((n, k), 15, 1 / k ** 0.5), rand((batch, n), 16)
    out = x.clone()
    ws = linear_workspace(batch, n, k)
    tw = tiles(w)
    nat.call("ipe_linear_residual", a.data_ptr(), tw.data_ptr(), out.data_ptr(), batch, k, n, ws.data_ptr(), ws.numel(),
             stream())
    acc = a.float() @ w.float().T
    ref = x.float() + acc.bfloat16().float()
    bound = 2 * BF16_REL * (acc.abs() + x.float().abs()) + 1e-3
    assert int(((out.float() - ref).abs() > bound).sum()) == 0


@pytest.mark.parametrize("batch", (1, 5, 16))
@pytest.mark.parametrize(("hidden", "inter"), [(2048, 6144), (1024, 3072), (256, 512)])
def test_rmsnorm_gate_up_silu_matches_fp32(batch, hidden, inter):
    x, w = rand((batch, hidden), 17), (1 + 0.1 * rand((hidden,), 18, dtype=torch.float32)).bfloat16()
    gate, up = rand((inter, hidden), 19, 0.03), rand((inter, hidden), 20, 0.03)
    g = nat.GATE_UP_GROUP
    packed = torch.stack((gate.view(inter // g, g, hidden), up.view(inter // g, g, hidden)), 1)
    packed = packed.reshape(2 * inter, hidden).contiguous()
    out = torch.empty((batch, inter), dtype=torch.bfloat16, device=DEV)
    ws = linear_workspace(batch, 2 * inter, hidden)
    tgu = tiles(gate, up)
    nat.call("ipe_rmsnorm_gate_up_silu", x.data_ptr(), w.data_ptr(), tgu.data_ptr(), out.data_ptr(), batch, hidden,
             inter, 1e-6, ws.data_ptr(), ws.numel(), stream())
    h = rmsnorm_ref(x, w, 1e-6).float()
    ref = (F.silu((h @ gate.float().T).bfloat16()) * (h @ up.float().T).bfloat16()).float()
    assert bf16_close(out, ref, rel=3 * BF16_REL, abs_=2e-3)[0] == 0


@pytest.mark.parametrize("batch", (1, 2, 16))
@pytest.mark.parametrize(("hidden", "vocab"), [(2048, 151936), (256, 2048), (128, 1024)])
def test_lm_head_logits_and_greedy_sample(batch, hidden, vocab):
    x, w = rand((batch, hidden), 21), (1 + 0.1 * rand((hidden,), 22, dtype=torch.float32)).bfloat16()
    emb = rand((vocab, hidden), 23, 0.02)
    parts = ops.lm_head_parts(vocab)
    logits = torch.empty((batch, vocab), dtype=torch.float32, device=DEV)
    partials = torch.empty((parts, batch, nat.PARTIAL_WORDS), dtype=torch.float32, device=DEV)
    nat.call("ipe_lm_head", x.data_ptr(), hidden, w.data_ptr(), tiles(emb).data_ptr(), logits.data_ptr(),
             partials.data_ptr(), batch, hidden, vocab, 1e-6, 0.0, 0, None, stream())
    ref = rmsnorm_ref(x, w, 1e-6).float() @ emb.float().T
    assert torch.equal(logits, logits.bfloat16().float())
    assert bf16_close(logits, ref, rel=2 * BF16_REL, abs_=1e-3)[0] == 0
    tokens = torch.empty((batch, 1), dtype=torch.int64, device=DEV)
    logprobs = torch.empty((batch, 1), dtype=torch.float32, device=DEV)
    nxt = torch.empty(batch, dtype=torch.int64, device=DEV)
    nat.call("ipe_sample", partials.data_ptr(), logits.data_ptr(), batch, vocab, 0.0, None, tokens.data_ptr(),
             logprobs.data_ptr(), 1, nxt.data_ptr(), stream())
    assert torch.equal(tokens[:, 0], logits.argmax(-1)) and torch.equal(nxt, tokens[:, 0])
    expected = torch.log_softmax(logits.double(), -1).gather(-1, tokens).float()
    assert torch.allclose(logprobs, expected, rtol=0, atol=2e-5)


# ---------------------------------------------------------------- q/k norm + RoPE + cache append

@pytest.mark.parametrize(("batch", "tokens", "start"), [(1, 1, 0), (2, 1, 37), (3, 1, 100), (2, 77, 0)])
def test_qk_norm_rope_append_matches_the_oracle_ops(batch, tokens, start):
    hq, hkv, d, cap, eps = 16, 8, 128, 256, 1e-6
    qkv = rand((batch * tokens, (hq + 2 * hkv) * d), 24)
    qn, kn = (1 + 0.1 * rand((d,), 25, dtype=torch.float32)).bfloat16(), (1 + 0.1 * rand((d,), 26, dtype=torch.float32)).bfloat16()
    cos, sin = oq.rotary_tables(torch.arange(cap), d, 1e6, torch.bfloat16)
    cos, sin = cos.to(DEV), sin.to(DEV)
    q = torch.empty((batch, hq, tokens, d), dtype=torch.bfloat16, device=DEV)
    k = torch.full((batch, hkv, cap, d), float("nan"), dtype=torch.bfloat16, device=DEV)
    v = k.clone()
    nat.call("ipe_qk_norm_rope_append", qkv.data_ptr(), batch, tokens, hq, hkv, qn.data_ptr(), kn.data_ptr(),
             cos.data_ptr(), sin.data_ptr(), start, None, q.data_ptr(), k.data_ptr(), v.data_ptr(), cap, eps,
             stream())
    split = qkv.view(batch, tokens, hq + 2 * hkv, d)
    rows = slice(start, start + tokens)
    q_ref = oq.apply_rotary(oq.qk_norm(split[:, :, :hq], qn, eps).transpose(1, 2), cos[rows], sin[rows])
    k_ref = oq.apply_rotary(oq.qk_norm(split[:, :, hq:hq + hkv], kn, eps).transpose(1, 2), cos[rows], sin[rows])
    v_ref = split[:, :, hq + hkv:].transpose(1, 2)
    assert bf16_close(q, q_ref, rel=BF16_REL, abs_=1e-6)[0] == 0
    assert bf16_close(k[:, :, rows], k_ref, rel=BF16_REL, abs_=1e-6)[0] == 0
    assert torch.equal(v[:, :, rows], v_ref)
    untouched = torch.ones(cap, dtype=torch.bool)
    untouched[rows] = False
    assert torch.isnan(k[:, :, untouched].float()).all() and torch.isnan(v[:, :, untouched].float()).all()


# --------------------------------------------------------------------------------- attention

def attention_ref(q, k, v, causal):
    """fp32 attention with GQA (query head j reads KV head j // groups)."""
    groups = q.shape[1] // k.shape[1]
    k = k.float().repeat_interleave(groups, 1)
    v = v.float().repeat_interleave(groups, 1)
    s = (q.float() @ k.transpose(-1, -2)) * 128 ** -0.5
    if causal:
        t = q.shape[2]
        s = s.masked_fill(torch.ones(t, t, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    return torch.softmax(s, -1) @ v


@pytest.mark.parametrize(("batch", "hq", "hkv", "length", "cap"),
                         [(1, 16, 8, 1, 64), (1, 16, 8, 31, 64), (2, 16, 8, 32, 64), (1, 16, 8, 33, 64),
                          (3, 16, 8, 1000, 1024), (1, 8, 8, 77, 128), (2, 16, 4, 300, 320), (1, 32, 4, 129, 256),
                          (1, 16, 8, 4097, 4352)])
def test_decode_attention_matches_fp32(batch, hq, hkv, length, cap):
    q = rand((batch, hq, 1, 128), 27)
    k = torch.full((batch, hkv, cap, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    v = k.clone()
    k[:, :, :length] = rand((batch, hkv, length, 128), 28)
    v[:, :, :length] = rand((batch, hkv, length, 128), 29)
    out = torch.empty((batch, hq * 128), dtype=torch.bfloat16, device=DEV)
    ws = torch.empty(ops.decode_attention_workspace(batch, hq, cap), dtype=torch.uint8, device=DEV)
    nat.call("ipe_decode_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), batch, hq, hkv, cap,
             length, None, ws.data_ptr(), ws.numel(), stream())
    ref = attention_ref(q, k[:, :, :length], v[:, :, :length], False).reshape(batch, hq * 128)
    assert bf16_close(out, ref, rel=2 * BF16_REL, abs_=2e-3)[0] == 0


def test_decode_attention_reads_its_length_from_the_device_state():
    batch, hq, hkv, cap, pos = 2, 16, 8, 256, 150
    q = rand((batch, hq, 1, 128), 30)
    k, v = rand((batch, hkv, cap, 128), 31), rand((batch, hkv, cap, 128), 32)
    state = torch.zeros(nat.STATE_WORDS, dtype=torch.int64, device=DEV)
    state[nat.STATE_POS] = pos
    out = torch.empty((batch, hq * 128), dtype=torch.bfloat16, device=DEV)
    ws = torch.empty(ops.decode_attention_workspace(batch, hq, cap), dtype=torch.uint8, device=DEV)
    nat.call("ipe_decode_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), batch, hq, hkv, cap, 0,
             state.data_ptr(), ws.data_ptr(), ws.numel(), stream())
    ref = attention_ref(q, k[:, :, :pos + 1], v[:, :, :pos + 1], False).reshape(batch, hq * 128)
    assert bf16_close(out, ref, rel=2 * BF16_REL, abs_=2e-3)[0] == 0


@pytest.mark.parametrize(("batch", "hq", "hkv", "pos", "cap"),
                         [(1, 16, 8, 0, 64), (1, 16, 8, 31, 64), (2, 16, 8, 32, 64), (3, 16, 8, 700, 1024),
                          (1, 16, 4, 99, 128), (2, 8, 8, 4099, 4352), (1, 32, 4, 40, 64)])
def test_fused_decode_attention_matches_the_unfused_ops(batch, hq, hkv, pos, cap):
    """q/k norm + RoPE + append + attention from the QKV output, against the oracle operators and
    an fp32 attention; run twice so the second call sees the counters the first left at zero."""
    eps = 1e-6
    qkv = rand((batch, (hq + 2 * hkv) * 128), 40)
    qn = (1 + 0.1 * rand((128,), 41, dtype=torch.float32)).bfloat16()
    kn = (1 + 0.1 * rand((128,), 42, dtype=torch.float32)).bfloat16()
    cos, sin = oq.rotary_tables(torch.arange(cap), 128, 1e6, torch.bfloat16)
    cos, sin = cos.to(DEV), sin.to(DEV)
    k = torch.full((batch, hkv, cap, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    v = k.clone()
    k[:, :, :pos] = rand((batch, hkv, pos, 128), 43) if pos else k[:, :, :0]
    v[:, :, :pos] = rand((batch, hkv, pos, 128), 44) if pos else v[:, :, :0]
    ws = torch.zeros(int(nat.load().ipe_decode_attention_qkv_workspace(batch, hq, hkv, cap)), dtype=torch.uint8,
                     device=DEV)
    outs = []
    for _ in range(2):
        out = torch.empty((batch, hq * 128), dtype=torch.bfloat16, device=DEV)
        nat.call("ipe_decode_attention_qkv", qkv.data_ptr(), qn.data_ptr(), kn.data_ptr(), cos.data_ptr(),
                 sin.data_ptr(), pos, None, k.data_ptr(), v.data_ptr(), out.data_ptr(), batch, hq, hkv, cap, eps,
                 ws.data_ptr(), ws.numel(), stream())
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    split = qkv.view(batch, 1, hq + 2 * hkv, 128)
    rows = slice(pos, pos + 1)
    q_ref = oq.apply_rotary(oq.qk_norm(split[:, :, :hq], qn, eps).transpose(1, 2), cos[rows], sin[rows])
    k_ref = oq.apply_rotary(oq.qk_norm(split[:, :, hq:hq + hkv], kn, eps).transpose(1, 2), cos[rows], sin[rows])
    assert bf16_close(k[:, :, rows], k_ref, rel=BF16_REL, abs_=1e-6)[0] == 0
    assert torch.equal(v[:, :, rows], split[:, :, hq + hkv:].transpose(1, 2))
    ref = attention_ref(q_ref, k[:, :, :pos + 1], v[:, :, :pos + 1], False).reshape(batch, hq * 128)
    assert bf16_close(outs[0], ref, rel=2 * BF16_REL, abs_=2e-3)[0] == 0
    counters = ws[: 4 * batch * hkv].view(torch.int32)
    assert int(counters.count_nonzero()) == 0


@pytest.mark.parametrize(("batch", "hq", "hkv", "tokens", "cap"),
                         [(1, 16, 8, 1, 8), (2, 16, 8, 17, 32), (1, 16, 8, 64, 64), (1, 16, 8, 65, 80),
                          (2, 4, 1, 200, 256), (1, 16, 8, 513, 1024), (1, 8, 8, 1024, 1024),
                          (1, 16, 8, 4096, 4352), (3, 8, 2, 300, 320)])
def test_prefill_attention_matches_fp32(batch, hq, hkv, tokens, cap):
    q = rand((batch, hq, tokens, 128), 33)
    k = torch.full((batch, hkv, cap, 128), float("nan"), dtype=torch.bfloat16, device=DEV)
    v = k.clone()
    k[:, :, :tokens] = rand((batch, hkv, tokens, 128), 34)
    v[:, :, :tokens] = rand((batch, hkv, tokens, 128), 35)
    out = torch.empty((batch, tokens, hq * 128), dtype=torch.bfloat16, device=DEV)
    nat.call("ipe_prefill_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), batch, hq, hkv, tokens,
             cap, stream())
    ref = attention_ref(q, k[:, :, :tokens], v[:, :, :tokens], True).transpose(1, 2).reshape(batch, tokens, hq * 128)
    assert bf16_close(out, ref, rel=3 * BF16_REL, abs_=4e-3)[0] == 0


def test_a_query_never_reads_a_later_key():
    """Changing keys and values after position 25 leaves queries 0..24 bit-identical."""
    batch, hq, hkv, tokens = 1, 4, 2, 40
    q = rand((batch, hq, tokens, 128), 36)
    k, v = rand((batch, hkv, tokens, 128), 37), rand((batch, hkv, tokens, 128), 38)
    outs = []
    for kk, vv in ((k, v), (torch.cat((k[:, :, :25], k[:, :, 25:] + 3), 2), torch.cat((v[:, :, :25], -v[:, :, 25:]), 2))):
        out = torch.empty((batch, tokens, hq * 128), dtype=torch.bfloat16, device=DEV)
        nat.call("ipe_prefill_attention", q.data_ptr(), kk.contiguous().data_ptr(), vv.contiguous().data_ptr(),
                 out.data_ptr(), batch, hq, hkv, tokens, tokens, stream())
        torch.cuda.synchronize()
        outs.append(out)
    assert torch.equal(outs[0][:, :25], outs[1][:, :25])
    assert not torch.equal(outs[0][:, 25], outs[1][:, 25])


# ---------------------------------------------------------------------------------- sampling

def test_greedy_breaks_ties_to_the_lowest_id_and_reports_log_probabilities():
    logits = torch.tensor([[0.0, 3.0, 3.0, 1.0], [5.0, 5.0, 5.0, 5.0]], device=DEV)
    tokens, logprobs = ops.sample_logits(logits, 0.0, 0)
    assert tokens.tolist() == [1, 0]
    assert torch.allclose(logprobs, torch.log_softmax(logits, -1)[[0, 1], [1, 0]], atol=1e-6)


@pytest.mark.parametrize("temperature", (0.6, 1.0))
def test_temperature_sampling_follows_the_tempered_distribution(temperature):
    """Chi-square over 100,000 draws, alpha 0.01 (tests/needs_torch/test_engine.py:284-296)."""
    from scipy.stats import chi2

    logits = torch.linspace(-6.0, 4.0, 50, device=DEV).expand(100_000, 50).contiguous()
    draws, _ = ops.sample_logits(logits, temperature, 20261016)
    observed = torch.bincount(draws.cpu(), minlength=50).double()
    expected = torch.softmax(torch.linspace(-6.0, 4.0, 50).double() / temperature, 0) * 100_000
    small = expected < 5
    observed = torch.cat((observed[~small], observed[small].sum()[None]))
    expected = torch.cat((expected[~small], expected[small].sum()[None]))
    statistic = ((observed - expected) ** 2 / expected).sum().item()
    assert statistic < chi2.ppf(0.99, len(expected) - 1)


def test_the_same_seed_gives_the_same_draws():
    logits = torch.randn((4, 100), generator=torch.Generator().manual_seed(11)).to(DEV)
    draws = [ops.sample_logits(logits, 1.0, seed)[0] for seed in (7, 7, 8)]
    assert torch.equal(draws[0], draws[1]) and not torch.equal(draws[0], draws[2])


def test_out_of_range_token_ids_set_the_device_error_instead_of_faulting():
    table = rand((100, 64), 39)
    out = torch.empty((2, 64), dtype=torch.bfloat16, device=DEV)
    nat.device_error(reset=True)
    ops.embed(torch.tensor([5, 100], device=DEV), table, out)
    assert nat.device_error(reset=True) == 1
    assert torch.equal(out[0], table[5]) and (out[1] == 0).all()
