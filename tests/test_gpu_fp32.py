"""The fp32 path (dtype=torch.float32, the reference's plumbing precision) against the
reference's own fp32 results in the golden fixtures and the fp64 oracle.

The envelope is the reference's accuracy rule (tests/needs_torch/accuracy.py:31-45) with the
reference's fp32 uncached forwards (math, sdpa) as references, and the 1.5x bar: the cached
engine's error at most 1.5x the reference fp32 engine's on the same inputs."""

import pytest
import torch

from cases import build, to_device
from ipe_b200 import _native as nat
from ipe_b200.engine import Engine
from ipe_b200.forward import forward_full
from oracle import accuracy
from oracle import qwen3 as oq

pytestmark = pytest.mark.gpu
F32 = torch.float32


@pytest.fixture(scope="module")
def models():
    cache = {}

    def get(name):
        if name not in cache:
            cpu = build(name)
            cache[name] = (cpu, to_device(cpu, "cuda"))
        return cache[name]

    return get


def fp32_refs(g):
    oracle = g["oracle"]
    return oracle, [accuracy.errors(oracle, g[f"forward_float32_{b}"]) for b in ("math", "sdpa")]


@pytest.mark.parametrize("name", ("small", "mqa"))
def test_fp32_cached_decoding_meets_the_rule_and_the_reference_engine_bar(golden, models, name):
    _, gpu = models(name)
    g = golden(name)
    ids, prompt = g["token_ids"], g["prompt"]
    engine = Engine(gpu, batch=ids.shape[0], capacity=ids.shape[1] + 1, dtype=F32)
    assert engine.dtype == F32 and engine._k.dtype == F32
    logits = oq.teacher_forced(engine, ids, prompt).cpu()
    oracle, refs = fp32_refs(g)
    mine = accuracy.errors(oracle, logits)
    assert accuracy.failures(mine, refs) == [], (mine.summary(), [r.summary() for r in refs])
    theirs = accuracy.errors(oracle, g["engine_float32_sdpa"]).summary()
    for key, value in mine.summary().items():
        assert value <= 1.5 * theirs[key] + 1e-9, (key, mine.summary(), theirs)
    assert nat.device_error() == 0


@pytest.mark.parametrize("name", ("small", "mqa"))
def test_fp32_forward_full_meets_the_rule(golden, models, name):
    _, gpu = models(name)
    g = golden(name)
    ids, positions = g["token_ids"], g["positions"].tolist()
    logits = forward_full(gpu, ids, dtype=F32, logit_positions=positions).cpu()
    oracle, refs = fp32_refs(g)
    assert accuracy.failures(accuracy.errors(oracle, logits), refs) == []
    # and close to the reference's own fp32 forward, far inside the bf16 scale
    assert (logits - g["forward_float32_math"]).abs().max() < 1e-3


def test_fp32_greedy_generation_equals_the_reference_except_at_near_ties(golden, models):
    cpu, gpu = models("small")
    g = golden("small")
    prompt = g["token_ids"][:, :g["prompt"]]
    out = Engine(gpu, batch=prompt.shape[0], capacity=prompt.shape[1] + 12, dtype=F32).generate(prompt, 12)
    expected = g["generate_float32_tokens"]
    if not torch.equal(out.tokens, expected):
        # a different choice is only allowed where the oracle's top two are within fp32 noise
        first = int((out.tokens != expected).any(0).nonzero()[0])
        seq = torch.cat((prompt, expected[:, :first]), 1)
        oracle = oq.oracle_logits(cpu, seq, [seq.shape[1] - 1])[:, 0]
        top2 = oracle.topk(2, -1).values
        assert ((top2[:, 0] - top2[:, 1]) < 1e-3).any()
    assert torch.allclose(out.logprobs[:, :1], g["generate_float32_logprobs"][:, :1], atol=1e-4)


def test_fp32_plumbing_model_top16_matches_the_reference(golden, models):
    """The 0.6B-width model (H=1024, I=3072, 2 layers) at fp32: the top-16 logits of each checked
    position are the reference fp32 forward's, within fp32 rounding."""
    _, gpu = models("qwen3-0.6b-2layer")
    g = golden("qwen3-0.6b-2layer")
    ids, positions = g["token_ids"], g["positions"].tolist()
    logits = forward_full(gpu, ids, dtype=F32, logit_positions=positions).cpu()[0]
    ref = g["forward_float32_math"]
    values = logits.gather(-1, ref["top_ids"])
    assert (values - ref["top_values"]).abs().max() < 1e-3
    assert torch.allclose(logits.double().sum(-1), ref["sum"].double(), rtol=1e-4, atol=1e-2)
