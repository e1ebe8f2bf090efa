"""The CUDA engine end to end against the oracle and the reference's golden vectors.

Models are the golden-vector models (tests/cases.py) moved to the GPU, and a full 28-layer
Qwen3-1.7B-architecture random-init model for the bar of at most 1.5x the reference bf16 engine's
errors. Every logit is checked against the fp64 oracle on the CPU; the acceptance envelope is the reference's accuracy rule with the oracle's
bf16 uncached variants (math, sdpa) as the references (tests/needs_torch/accuracy.py:31-45).
"""

import dataclasses

import pytest
import torch

from cases import build, to_device
from ipe_b200 import _native as nat
from ipe_b200.config import QWEN3_1_7B
from ipe_b200.engine import Engine, sample
from ipe_b200 import engine as engine_module
from ipe_b200.forward import forward_full
from ipe_b200.synthetic import random_model
from oracle import accuracy
from oracle import qwen3 as oq

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
NEAR_TIE = 1e-2  # the oracle's top-2 gap below which greedy choices may differ


def off_choices(choice, oracle):
    """Positions where `choice` differs from the oracle's argmax although the oracle's top-2 gap is
    at least NEAR_TIE (a disagreement the near-tie exception does not cover)."""
    top2 = oracle.topk(2, -1).values
    gap = top2[..., 0] - top2[..., 1]
    return int(((choice != oracle.argmax(-1)) & (gap >= NEAR_TIE)).sum())


def reference_off_choices(cpu_model, ids, prompt, oracle):
    """off_choices of the restated reference bf16 engine (sdpa and math attention), teacher-forced
    on the same tokens: how often the reference's own variants leave the oracle outside near ties."""
    counts = []
    for backend in oq.BACKENDS:
        engine = oq.CachedEngine(cpu_model, batch=ids.shape[0], capacity=ids.shape[1] + 1, dtype=BF16, backend=backend)
        counts.append(off_choices(oq.teacher_forced(engine, ids, prompt).argmax(-1), oracle))
    return counts


@pytest.fixture(scope="module")
def models():
    cache = {}

    def get(name):
        if name not in cache:
            cpu = build(name)
            cache[name] = (cpu, to_device(cpu, "cuda"))
        return cache[name]

    return get


def teacher_forced(engine, ids, prompt):
    return oq.teacher_forced(engine, ids, prompt).cpu()


def rule_check(cpu_model, ids, logits, prompt):
    """Accuracy-rule failures of `logits` (positions prompt-1..T-1) and the summaries."""
    positions = list(range(prompt - 1, ids.shape[1]))
    oracle = oq.oracle_logits(cpu_model, ids, positions)
    refs = [accuracy.errors(oracle, oq.forward_full(cpu_model, ids, dtype=BF16, backend=b, logit_positions=positions))
            for b in oq.BACKENDS]
    mine = accuracy.errors(oracle, logits)
    return accuracy.failures(mine, refs), mine.summary(), [r.summary() for r in refs], oracle


@pytest.mark.parametrize("name", ("small", "mqa"))
def test_cached_decoding_meets_the_accuracy_rule(golden, models, name):
    cpu, gpu = models(name)
    g = golden(name)
    ids, prompt = g["token_ids"], g["prompt"]
    engine = Engine(gpu, batch=ids.shape[0], capacity=ids.shape[1] + 1)
    logits = teacher_forced(engine, ids, prompt)
    failures, mine, refs, _ = rule_check(cpu, ids, logits, prompt)
    assert failures == [], (mine, refs)
    # and the reference engine's own bf16 logits (golden) are within the same envelope of ours
    assert (logits - g["engine_bfloat16_sdpa"]).abs().max() < 4 * max(r["max_abs"] for r in refs)
    assert nat.device_error() == 0


@pytest.mark.parametrize("name", ("small", "mqa"))
def test_uncached_forward_meets_the_accuracy_rule(golden, models, name):
    cpu, gpu = models(name)
    g = golden(name)
    ids, positions = g["token_ids"], g["positions"].tolist()
    logits = forward_full(gpu, ids, dtype=BF16, logit_positions=positions).cpu()
    failures, mine, refs, _ = rule_check(cpu, ids, logits, positions[0] + 1)
    assert failures == [], (mine, refs)


def test_prefill_equals_the_uncached_last_position(models):
    cpu, gpu = models("small")
    ids = torch.randint(0, 2048, (2, 37), generator=torch.Generator().manual_seed(3))
    engine = Engine(gpu, batch=2, capacity=64)
    a = engine.prefill(ids)
    b = forward_full(gpu, ids, dtype=BF16, logit_positions=[36])[:, 0]
    # same kernels up to the LM head, whose GEMV and GEMM sum in different orders: one bf16 ulp
    assert ((a - b).abs() <= 2 ** -7 * b.abs() + 1e-3).all()


def test_greedy_generation_follows_the_oracle_except_at_near_ties(models):
    cpu, gpu = models("small")
    prompt = torch.randint(0, 2048, (2, 12), generator=torch.Generator().manual_seed(9))
    engine = Engine(gpu, batch=2, capacity=40)
    out = engine.generate(prompt, 20)
    assert out.tokens.shape == (2, 20) and out.lengths.tolist() == [20, 20]
    seq = torch.cat((prompt, out.tokens[:, :-1]), 1)
    oracle = oq.oracle_logits(cpu, seq, list(range(11, seq.shape[1])))
    # our greedy choices equal the oracle's except at near ties, or no more often than the
    # reference's own bf16 engine departs from it on the same tokens
    ours = off_choices(out.tokens, oracle)
    assert ours <= max(reference_off_choices(cpu, seq, 12, oracle)), ours


def test_generation_is_reproducible_and_logprobs_match_the_logits(models):
    _, gpu = models("small")
    prompt = torch.randint(0, 2048, (2, 8), generator=torch.Generator().manual_seed(6))
    engine = Engine(gpu, batch=2, capacity=40)
    first = engine.generate(prompt, 24, temperature=30.0, seed=7)
    again = engine.generate(prompt, 24, temperature=30.0, seed=7)
    other = engine.generate(prompt, 24, temperature=30.0, seed=8)
    assert torch.equal(again.tokens, first.tokens) and not torch.equal(other.tokens, first.tokens)
    assert len(first.tokens.unique()) > 4
    logits = teacher_forced(engine, torch.cat((prompt, first.tokens[:, :-1]), 1), 8)
    expected = torch.log_softmax(logits.double(), -1).gather(-1, first.tokens[..., None]).squeeze(-1)
    assert torch.allclose(first.logprobs.double(), expected, rtol=0, atol=1e-4)


def test_temperature_draws_follow_the_tempered_distribution_of_the_step(models):
    """Many seeds, one step: the first sampled token's frequencies follow softmax(l / T)."""
    _, gpu = models("mqa")
    prompt = torch.randint(0, 512, (1, 6), generator=torch.Generator().manual_seed(1))
    engine = Engine(gpu, batch=1, capacity=8)
    logits = engine.prefill(prompt)[0].double().cpu()
    probs = torch.softmax(logits / 2.0, -1)
    counts = torch.zeros(512, dtype=torch.float64)
    for seed in range(600):
        counts[engine.generate(prompt, 1, temperature=2.0, seed=seed).tokens[0, 0]] += 1
    top = probs.argmax()
    assert abs(counts[top] / 600 - probs[top]) < 5 * (probs[top] * (1 - probs[top]) / 600) ** 0.5 + 0.01


def test_stop_ids_set_lengths_and_end_generation(models):
    _, gpu = models("small")
    engine = Engine(gpu, batch=2, capacity=40)
    prompt = torch.randint(0, 2048, (2, 8), generator=torch.Generator().manual_seed(10))
    free = engine.generate(prompt, 30, temperature=30.0, seed=3).tokens
    stops = (free[0, 3].item(), free[1, 5].item())
    lengths = [int(torch.isin(row, torch.tensor(stops)).nonzero()[0]) + 1 for row in free]
    stopped = engine.generate(prompt, 30, temperature=30.0, seed=3, stop_ids=stops)
    assert stopped.lengths.tolist() == lengths
    assert torch.equal(stopped.tokens, free[:, :max(lengths)])


# ------------------------------------------------------------------------- the cache contract

def test_decode_validates_state_and_inputs(models):
    _, gpu = models("small")
    engine = Engine(gpu, batch=2, capacity=6)
    with pytest.raises(ValueError, match="prefill first"):
        engine.decode(torch.tensor([1, 2]))
    engine.prefill(torch.randint(0, 2048, (2, 5)))
    for bad in (torch.tensor([1]), torch.tensor([1.0, 2.0]), torch.tensor([1, 2048]), [1, 2]):
        with pytest.raises(ValueError):
            engine.decode(bad)
    assert engine.length == 5
    engine.decode(torch.tensor([1, 2]))
    with pytest.raises(ValueError, match="all 6 positions"):
        engine.decode(torch.tensor([1, 2]))
    assert engine.length == 6


def test_an_invalid_prefill_leaves_the_current_batch(models):
    _, gpu = models("small")
    engine = Engine(gpu, batch=2, capacity=6)
    engine.prefill(torch.randint(0, 2048, (2, 4)))
    for bad in (torch.randint(0, 2048, (3, 4)), torch.randint(0, 2048, (1, 7)), torch.zeros(1, 0, dtype=torch.int64),
                torch.tensor([[1, 2048]])):
        with pytest.raises(ValueError):
            engine.prefill(bad)
    assert (engine.batch, engine.length) == (2, 4)
    engine.decode(torch.tensor([1, 2]))


@pytest.mark.parametrize("arguments", [{"batch": 0, "capacity": 4}, {"batch": 1, "capacity": 0},
                                       {"batch": 1, "capacity": 8193}, {"batch": 1, "capacity": 4, "backend": "flash"},
                                       {"batch": 1, "capacity": 4, "dtype": torch.float64},
                                       {"batch": 17, "capacity": 4}])
def test_construction_validates_its_arguments(models, arguments):
    _, gpu = models("small")
    with pytest.raises(ValueError):
        Engine(gpu, **arguments)


def test_a_new_batch_never_reads_the_previous_one(models):
    _, gpu = models("small")
    long_ids = torch.randint(0, 2048, (2, 30), generator=torch.Generator().manual_seed(3))
    short_ids = torch.randint(0, 2048, (1, 12), generator=torch.Generator().manual_seed(4))
    fresh = teacher_forced(Engine(gpu, batch=2, capacity=30), short_ids, 4)
    engine = Engine(gpu, batch=2, capacity=30)
    teacher_forced(engine, long_ids, 3)
    engine.prefill(short_ids[:, :4])
    engine._k[:, :, :, 4:] = float("nan")
    engine._v[:, :, :, 4:] = float("nan")
    engine._k[:, 1:] = engine._v[:, 1:] = float("nan")
    logits = torch.stack([engine.decode(short_ids[:, p]) for p in range(4, 12)], 1).cpu()
    assert torch.equal(logits, fresh[:, 1:])


def test_a_failed_step_keeps_the_committed_prefix(models, monkeypatch):
    _, gpu = models("small")
    ids = torch.randint(0, 2048, (2, 12), generator=torch.Generator().manual_seed(5))
    expected = teacher_forced(Engine(gpu, batch=2, capacity=12), ids, 6)
    engine = Engine(gpu, batch=2, capacity=12)
    logits = [engine.prefill(ids[:, :6]).cpu()]
    real, calls = engine_module.decoder_layer, []

    def fail_in_layer_1(*args, **kwargs):
        calls.append(None)
        if len(calls) == 2:
            raise RuntimeError("injected")
        return real(*args, **kwargs)

    monkeypatch.setattr(engine_module, "decoder_layer", fail_in_layer_1)
    with pytest.raises(RuntimeError, match="injected"):
        engine.decode(ids[:, 6])
    monkeypatch.undo()
    assert engine.length == 6
    logits += [engine.decode(ids[:, p]).cpu() for p in range(6, 12)]
    assert torch.equal(torch.stack(logits, 1), expected)


def test_capacity_holds_prompt_plus_new_tokens_minus_one(models):
    _, gpu = models("small")
    engine = Engine(gpu, batch=1, capacity=8)
    assert engine.generate(torch.randint(0, 2048, (1, 5)), 4).tokens.shape == (1, 4)
    assert engine.length == 8
    with pytest.raises(ValueError, match="exceeds capacity"):
        engine.generate(torch.randint(0, 2048, (1, 5)), 5)
    assert engine.generate(torch.randint(0, 2048, (1, 1)), 1).tokens.shape == (1, 1)


def test_decode_steps_never_synchronize_or_grow_the_allocator(models):
    _, gpu = models("small")
    engine = Engine(gpu, batch=1, capacity=64)
    tokens = sample(engine.prefill(torch.randint(0, 2048, (1, 16))), 0.0)[0]
    for _ in range(2):  # the first decode runs eagerly, the second captures the step graph
        tokens = sample(engine.decode(tokens), 0.0)[0]
    torch.cuda.synchronize()
    reserved = torch.cuda.memory_reserved()
    torch.cuda.set_sync_debug_mode("error")
    try:
        for _ in range(32):
            tokens = sample(engine.decode(tokens), 0.0)[0]
    finally:
        torch.cuda.set_sync_debug_mode(0)
    torch.cuda.synchronize()
    assert torch.cuda.memory_reserved() == reserved


def test_tempered_sample_with_a_cuda_generator_never_synchronizes():
    logits = torch.randn((3, 4096), generator=torch.Generator().manual_seed(2)).cuda()
    first = torch.Generator(device="cuda").manual_seed(11)
    again = torch.Generator(device="cuda").manual_seed(11)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        a1, a2 = sample(logits, 0.8, first)[0], sample(logits, 0.8, first)[0]
        b1 = sample(logits, 0.8, again)[0]
    finally:
        torch.cuda.set_sync_debug_mode(0)
    # the same generator seed gives the same draws; a generator moves on after each draw
    assert torch.equal(a1, b1)
    draws = torch.stack([sample(logits, 0.8, first)[0] for _ in range(6)] + [a1, a2])
    assert len({tuple(r.tolist()) for r in draws}) > 1


@pytest.mark.parametrize(("name", "batch", "length", "prompt"), [
    ("small", 2, 20, 6),
    ("qwen3-1.7b-2layer", 1, 700, 694),   # one row: 11 attention splits merged, half-tile o/down units
    ("qwen3-1.7b-2layer", 4, 300, 296),   # 4 rows: activations staged in shared memory (o_proj and
                                          # down_proj rows by bulk copies), 4 splits
    ("qwen3-1.7b-2layer", 8, 300, 296),   # 8 rows: the normalised rows (QKV, gate/up, LM head) staged
                                          # in shared memory, o_proj / down_proj reading theirs from L2
    ("qwen3-1.7b-2layer", 16, 300, 296),  # 16 rows: two MMA column tiles, the same split staging,
                                          # one attention split streaming many 32-key sub-chunks
])
def test_one_kernel_step_agrees_with_the_per_operator_kernels(models, monkeypatch, name, batch, length, prompt):
    """The graph-replayed one-kernel decode step against the per-operator kernels run eagerly (a
    replaced layer hook selects them): the same math summed in a different order, so within a few
    bf16 ulps of the logits, and the greedy choices agree."""
    _, gpu = models(name)
    vocab = gpu.config.vocab_size
    ids = torch.randint(0, vocab, (batch, length), generator=torch.Generator().manual_seed(12))
    stepped = teacher_forced(Engine(gpu, batch=batch, capacity=length + 4), ids, prompt)
    assert nat.device_error() == 0
    monkeypatch.setattr(engine_module, "decoder_layer", lambda *a, **k: engine_module._BUILTIN_DECODE(*a, **k))
    per_op = teacher_forced(Engine(gpu, batch=batch, capacity=length + 4), ids, prompt)
    assert ((stepped - per_op).abs() <= 4 * 2 ** -8 * per_op.abs() + 0.05).all()
    assert (stepped.argmax(-1) == per_op.argmax(-1)).float().mean() > 0.9


def test_one_kernel_steps_are_deterministic(models):
    _, gpu = models("mqa")
    ids = torch.randint(0, 512, (1, 30), generator=torch.Generator().manual_seed(13))
    a = teacher_forced(Engine(gpu, batch=1, capacity=32), ids, 5)
    b = teacher_forced(Engine(gpu, batch=1, capacity=32), ids, 5)
    assert torch.equal(a, b)


# --------------------------------------------------------------- Qwen3-1.7B, 28 layers

@pytest.fixture(scope="module")
def qwen17():
    cpu = random_model(QWEN3_1_7B, seed=0, std=0.02)
    return cpu, to_device(cpu, "cuda")


def test_qwen3_1_7b_meets_the_rule_and_the_reference_engine_bar(qwen17):
    """Prompt 64, 16 teacher-forced decode steps: our bf16 error against the fp64 oracle is within
    the accuracy rule and at most 1.5x the reference bf16 engine's on the same inputs."""
    cpu, gpu = qwen17
    ids = torch.randint(0, QWEN3_1_7B.vocab_size, (1, 80), generator=torch.Generator().manual_seed(0))
    prompt = 64
    mine = teacher_forced(Engine(gpu, batch=1, capacity=96), ids, prompt)
    failures, summary, refs, oracle = rule_check(cpu, ids, mine, prompt)
    assert failures == [], (summary, refs)
    ref_engine = oq.CachedEngine(cpu, batch=1, capacity=96, dtype=BF16, backend="sdpa")
    theirs = accuracy.errors(oracle, oq.teacher_forced(ref_engine, ids, prompt)).summary()
    for key in ("median_abs", "max_abs", "mean_kl"):
        assert summary[key] <= 1.5 * theirs[key], (key, summary, theirs)
    # Greedy choices are checked over the 256 steps of the W1 generation
    # (test_gpu_parity_1_7b.py::test_w1_greedy_choices_follow_the_reference_engine_except_near_ties):
    # 17 positions are too few to compare departure counts with the reference engines'.
