"""Parity of the full 28-layer Qwen3-1.7B-architecture model at the benchmark contexts.

Every logit is checked against the reference's fp64 oracle, `lm_logits(final_hidden(float64))`
(src/ipe/forward.py:133-152), run on the GPU in fp64 and anchored to the CPU oracle on a short
prefix (tests/needs_torch/test_gpu.py:72-78). At the W1 context (prompt 512, then teacher-forced
decode steps) and the W3 context (prompt 4096, the tcgen05 prefill, then decode steps) the engine's
fp32 logits must
- pass the reference's accuracy rule (tests/needs_torch/accuracy.py:31-45) against the reference's
  bf16 uncached variants (math and sdpa), and
- have median / max error and mean KL at most 1.5x the reference bf16 cached engine's (the oracle's
  restatement of src/ipe/engine.py, sdpa) on the same inputs.
Greedy choices are compared with the reference bf16 engine's along its own W1 generation.
Weights are the benchmark's random init (N(0, 0.02) matrices, unit norms) drawn on the GPU.
"""

import pytest
import torch

from ipe_b200.config import QWEN3_1_7B
from ipe_b200.engine import Engine
from ipe_b200.synthetic import random_model
from oracle import accuracy
from oracle import qwen3 as oq

pytestmark = pytest.mark.gpu
BF16 = torch.bfloat16
VOCAB = QWEN3_1_7B.vocab_size
NEAR_TIE = 1e-2  # the oracle's top-2 gap below which greedy choices may differ


@pytest.fixture(scope="module")
def qwen17():
    return random_model(QWEN3_1_7B, seed=0, std=0.02, device="cuda", generator_device="cuda")


def prompt_ids(length, seed=0):
    return torch.randint(0, VOCAB, (1, length), generator=torch.Generator().manual_seed(seed))


def cpu_copy(model):
    from cases import to_device
    return to_device(model, "cpu")


def test_the_gpu_oracle_is_the_cpu_oracle(qwen17):
    """The fp64 oracle on the GPU against the same program on the CPU over a short prefix."""
    ids = prompt_ids(24, seed=5)
    gpu = oq.oracle_logits(qwen17, ids, [23]).cpu()
    cpu = oq.oracle_logits(cpu_copy(qwen17), ids, [23])
    assert torch.allclose(gpu, cpu, rtol=0, atol=1e-8), (gpu - cpu).abs().max()


def check_context(model, prompt, steps, capacity):
    ids = prompt_ids(prompt + steps)
    positions = list(range(prompt - 1, prompt + steps))
    mine = oq.teacher_forced(Engine(model, batch=1, capacity=capacity), ids, prompt)
    oracle = oq.oracle_logits(model, ids, positions)
    refs = [accuracy.errors(oracle, oq.forward_full(model, ids, dtype=BF16, backend=b, logit_positions=positions))
            for b in oq.BACKENDS]
    ours = accuracy.errors(oracle, mine)
    assert accuracy.failures(ours, refs) == [], (ours.summary(), [r.summary() for r in refs])
    reference = oq.CachedEngine(model, batch=1, capacity=capacity, dtype=BF16, backend="sdpa")
    theirs = accuracy.errors(oracle, oq.teacher_forced(reference, ids, prompt)).summary()
    summary = ours.summary()
    for key in ("median_abs", "max_abs", "mean_kl"):
        assert summary[key] <= 1.5 * theirs[key], (key, summary, theirs)
    return summary, theirs


def test_w1_context_meets_the_rule_and_the_reference_engine_bar(qwen17):
    """W1: a 512-token prompt, then 16 teacher-forced decode steps (capacity 1024)."""
    summary, theirs = check_context(qwen17, 512, 16, 1024)
    print("W1 ours", summary, "reference engine", theirs)


def test_w3_context_meets_the_rule_and_the_reference_engine_bar(qwen17):
    """W3: a 4096-token prompt through the tcgen05 prefill, then 4 decode steps (capacity 4352)."""
    summary, theirs = check_context(qwen17, 4096, 4, 4352)
    print("W3 ours", summary, "reference engine", theirs)


def test_w1_greedy_choices_follow_the_reference_engine_except_near_ties(qwen17):
    """Along the reference bf16 engine's own W1 generation (sdpa, 256 greedy tokens), this engine's
    greedy choice at every step equals the reference's wherever the oracle's top-2 gap is at least
    1e-2, as often as the reference's own math-backend engine does.

    Any two bf16 engines disagree at steps whose oracle gap is below their logit error (about 0.15
    at this size), so the reference's math and sdpa engines are the yardstick: the test counts the
    steps at which each differs from the sdpa engine's choice with an oracle gap >= 1e-2."""
    prompt, new = 512, 256
    ids = prompt_ids(prompt)
    reference = oq.CachedEngine(qwen17, batch=1, capacity=1024, dtype=BF16, backend="sdpa")
    ref_tokens, _ = reference.generate(ids.cuda(), new)
    seq = torch.cat((ids, ref_tokens[:, :-1]), 1)
    positions = list(range(prompt - 1, prompt + new - 1))
    mine = oq.teacher_forced(Engine(qwen17, batch=1, capacity=1024), seq, prompt).argmax(-1).cpu()
    math = oq.teacher_forced(oq.CachedEngine(qwen17, batch=1, capacity=1024, dtype=BF16, backend="math"), seq,
                             prompt).argmax(-1).cpu()
    oracle = oq.oracle_logits(qwen17, seq, positions)
    top2 = oracle.topk(2, -1).values
    gap = (top2[..., 0] - top2[..., 1]).cpu()
    ref = ref_tokens.cpu()
    ours_off = ((mine != ref) & (gap >= NEAR_TIE)).sum().item()
    math_off = ((math != ref) & (gap >= NEAR_TIE)).sum().item()
    print(f"W1 greedy, {new} steps: ours differ from the reference sdpa engine at {(mine != ref).sum().item()} steps "
          f"({ours_off} with oracle gap >= {NEAR_TIE}); the reference math engine at {(math != ref).sum().item()} "
          f"({math_off}); near ties (gap < {NEAR_TIE}): {(gap < NEAR_TIE).sum().item()}; "
          f"smallest gap where ours differ: {gap[mine != ref].min().item() if (mine != ref).any() else None}")
    assert ours_off <= max(math_off, 1), (ours_off, math_off)
