"""The accuracy rule, restated in oracle/accuracy.py, separates seeded bugs from legitimate
reorderings the way the reference's rule does (tests/needs_torch/test_engine.py:130-188).

Candidates are the oracle's cached engine with one defect planted (on the CPU, in the oracle);
references are the oracle's uncached bf16/fp32 variants; every error is measured against the fp64 oracle.
"""

import dataclasses

import pytest
import torch

from cases import build
from oracle import accuracy
from oracle import qwen3 as oq

PROMPT, LENGTH = 16, 56


@pytest.fixture(scope="module")
def rule_inputs():
    loaded = build("mqa")
    ids = torch.randint(0, loaded.config.vocab_size, (2, LENGTH), generator=torch.Generator().manual_seed(2))
    positions = list(range(PROMPT - 1, LENGTH))
    oracle = oq.oracle_logits(loaded, ids, positions)
    references = {dtype: [accuracy.errors(oracle, oq.forward_full(loaded, ids, dtype=dtype, backend=b,
                                                                   logit_positions=positions)) for b in oq.BACKENDS]
                  for dtype in oq.RUN_DTYPES}
    return loaded, ids, oracle, references


def rule_failures(rule_inputs, dtype, loaded=None):
    default, ids, oracle, references = rule_inputs
    engine = oq.CachedEngine(loaded or default, batch=2, capacity=LENGTH + 1, dtype=dtype)
    return accuracy.failures(accuracy.errors(oracle, oq.teacher_forced(engine, ids, PROMPT)), references[dtype])


def _late_rope(start_filter):
    real = oq.decoder_layer

    def layer(x, w, rope, config, *, backend, cache=None, start=0):
        if start > 0 and start_filter(start):
            rope = tuple(t[1:] for t in oq.rotary_tables(torch.arange(start, start + 2), config.head_dim,
                                                         config.rope_theta, x.dtype))
        return real(x, w, rope, config, backend=backend, cache=cache, start=start)
    return layer


def interleaved_rotary(x, cos, sin):
    half = x.shape[-1] // 2
    c, s = cos[..., :half].repeat_interleave(2, -1), sin[..., :half].repeat_interleave(2, -1)
    rotated = torch.stack((-x[..., 1::2], x[..., 0::2]), dim=-1).flatten(-2)
    return x * c + rotated * s


def bf16_rms_norm(x, weight, eps):
    h = x.bfloat16()
    return (weight.bfloat16() * (h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps))).to(x.dtype)


def divided_rms_norm(x, weight, eps):
    h = x.float() if x.dtype != torch.float64 else x
    return weight * (h / torch.sqrt(h.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype)


def plant(monkeypatch, defect):
    attention, rotary = oq.attention, oq.rotary_tables
    if defect == "interleaved rotary":
        monkeypatch.setattr(oq, "apply_rotary", interleaved_rotary)
    elif defect == "decode rotated one position late":
        monkeypatch.setattr(oq, "decoder_layer", _late_rope(lambda start: True))
    elif defect == "first decode step rotated one position late":
        monkeypatch.setattr(oq, "decoder_layer", _late_rope(lambda start: start == PROMPT))
    elif defect == "no QK-norm":
        monkeypatch.setattr(oq, "qk_norm", lambda x, w, eps: x)
    elif defect == "RMSNorm in bf16":
        monkeypatch.setattr(oq, "rms_norm", bf16_rms_norm)
    elif defect == "decode misses its own key":
        monkeypatch.setattr(oq, "attention", lambda q, k, v, *, causal, backend: attention(
            q, k if causal else k[:, :, :-1], v if causal else v[:, :, :-1], causal=causal, backend=backend))
    elif defect == "decode reads one position past its end":
        def past(t):
            b, h, n, d = t.shape
            return t.as_strided((b, h, n + 1, d), t.stride(), t.storage_offset())
        monkeypatch.setattr(oq, "attention", lambda q, k, v, *, causal, backend: attention(
            q, k if causal else past(k), v if causal else past(v), causal=causal, backend=backend))
    elif defect == "uniform rotary offset":
        monkeypatch.setattr(oq, "rotary_tables", lambda positions, *args: rotary(positions + 1, *args))
    elif defect == "RMSNorm divides by the root":
        monkeypatch.setattr(oq, "rms_norm", divided_rms_norm)


BUGS = ("interleaved rotary", "decode rotated one position late", "first decode step rotated one position late",
        "no QK-norm", "RMSNorm in bf16", "decode misses its own key", "decode reads one position past its end",
        "epsilon 1e-5")
REORDERINGS = ("uniform rotary offset", "RMSNorm divides by the root")


def test_the_unmodified_oracle_engine_passes(rule_inputs):
    for dtype in oq.RUN_DTYPES:
        assert rule_failures(rule_inputs, dtype) == []


@pytest.mark.parametrize("bug", BUGS)
def test_the_rule_fails_seeded_bugs_at_fp32(rule_inputs, monkeypatch, bug):
    loaded = rule_inputs[0]
    if bug == "epsilon 1e-5":
        loaded = dataclasses.replace(loaded, config=dataclasses.replace(loaded.config, rms_norm_eps=1e-5))
    plant(monkeypatch, bug)
    assert rule_failures(rule_inputs, torch.float32, loaded) != []


@pytest.mark.parametrize("dtype", oq.RUN_DTYPES)
@pytest.mark.parametrize("variant", REORDERINGS)
def test_the_rule_accepts_legitimate_reorderings(rule_inputs, monkeypatch, dtype, variant):
    plant(monkeypatch, variant)
    assert rule_failures(rule_inputs, dtype) == []
