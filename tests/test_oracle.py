"""The oracle (a CPU restatement of the reference) against golden vectors made by the reference.

tests/golden/*.pt were written by tests/golden/make_golden.py running the reference package
itself. These checks pin `oracle/qwen3.py` to it: the fp64 oracle logits to 1e-9, the bf16 / fp32
uncached and cached paths to the reference's own bits on the machine that made the vectors (a
small tolerance elsewhere, since CPU BLAS kernels differ across machines), greedy generation, and
the rotary tables bit for bit.
"""

import pytest
import torch

from cases import CASES, build
from oracle import qwen3 as oq

FULL = ("small", "mqa")
SUMMARY = ("qwen3-0.6b-2layer", "qwen3-1.7b-2layer")


def close(actual, expected, dtype_name):
    if torch.equal(actual, expected):
        return True
    tol = {"bfloat16": 2 ** -6, "float32": 1e-5}[dtype_name]
    return bool(((actual.double() - expected.double()).abs() <= tol * (1 + expected.double().abs())).all())


@pytest.fixture(scope="module")
def models():
    return {}


def model_of(models, name):
    if name not in models:
        models[name] = build(name)
    return models[name]


@pytest.mark.parametrize("name", FULL + SUMMARY)
def test_models_are_rebuilt_identically(golden, models, name):
    g = golden(name)
    assert torch.equal(model_of(models, name).weights.embed_tokens.double().sum(), g["embed_checksum"])


@pytest.mark.parametrize("name", FULL)
def test_fp64_oracle_matches_the_reference(golden, models, name):
    g = golden(name)
    loaded = model_of(models, name)
    oracle = oq.oracle_logits(loaded, g["token_ids"], g["positions"])
    assert oracle.dtype == torch.float64
    assert torch.allclose(oracle, g["oracle"], rtol=0, atol=1e-9)


@pytest.mark.parametrize("name", FULL)
@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float32))
@pytest.mark.parametrize("backend", ("math", "sdpa"))
def test_uncached_forward_matches_the_reference(golden, models, name, dtype, backend):
    g = golden(name)
    loaded = model_of(models, name)
    logits = oq.forward_full(loaded, g["token_ids"], dtype=dtype, backend=backend, logit_positions=g["positions"])
    assert close(logits, g[f"forward_{str(dtype)[6:]}_{backend}"], str(dtype)[6:])


@pytest.mark.parametrize("name", FULL)
@pytest.mark.parametrize("dtype", (torch.bfloat16, torch.float32))
def test_cached_engine_matches_the_reference(golden, models, name, dtype):
    g = golden(name)
    loaded = model_of(models, name)
    ids, prompt = g["token_ids"], g["prompt"]
    engine = oq.CachedEngine(loaded, batch=ids.shape[0], capacity=ids.shape[1] + 1, dtype=dtype)
    logits = oq.teacher_forced(engine, ids, prompt)
    assert close(logits, g[f"engine_{str(dtype)[6:]}_sdpa"], str(dtype)[6:])
    tokens, logprobs = engine.generate(ids[:, :prompt], 12)
    assert torch.equal(tokens, g[f"generate_{str(dtype)[6:]}_tokens"])
    assert torch.allclose(logprobs, g[f"generate_{str(dtype)[6:]}_logprobs"], rtol=0, atol=1e-4)


@pytest.mark.parametrize("name", FULL)
def test_rotary_tables_match_the_reference_bitwise(golden, name):
    g = golden(name)
    config = CASES[name][0]
    cos, sin = oq.rotary_tables(torch.arange(g["rotary_cos_bf16"].shape[0]), config.head_dim, config.rope_theta,
                                torch.bfloat16)
    assert torch.equal(cos, g["rotary_cos_bf16"]) and torch.equal(sin, g["rotary_sin_bf16"])


def summary(logits):
    flat = logits.reshape(-1, logits.shape[-1]).double()
    values, ids = flat.topk(16, dim=-1)
    return ids, values, flat.sum(-1)


@pytest.mark.parametrize("name", SUMMARY)
def test_full_vocabulary_models_match_the_reference_summaries(golden, models, name):
    """Two-layer Qwen3-0.6B / 1.7B-width models with the 151,936-entry vocabulary: fp64 oracle and
    bf16 uncached logits against the reference's top-16 and row sums."""
    g = golden(name)
    loaded = model_of(models, name)
    ids, positions = g["token_ids"], g["positions"]
    oracle_ids, oracle_values, oracle_sum = summary(oq.oracle_logits(loaded, ids, positions))
    assert torch.equal(oracle_ids, g["oracle"]["top_ids"])
    assert torch.allclose(oracle_values, g["oracle"]["top_values"], rtol=0, atol=1e-9)
    assert torch.allclose(oracle_sum, g["oracle"]["sum"], rtol=0, atol=1e-6)
    bf16 = oq.forward_full(loaded, ids, dtype=torch.bfloat16, backend="sdpa", logit_positions=positions)
    _, values, _ = summary(bf16)
    assert torch.allclose(values, g["forward_bfloat16_sdpa"]["top_values"], rtol=0, atol=2 ** -5)
