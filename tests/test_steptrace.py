"""The step-trace reader on a synthetic trace (no GPU): phase kinds, stage / work / barrier sums
and the sampling tail, for the word layout IPE_TRACE_WORDS of include/ipe_b200.h."""

import torch

from ipe_b200 import _native as nat
from ipe_b200.steptrace import detail, exchange_stage_us, format_detail, format_summary, summarize


def test_summary_of_a_synthetic_trace():
    layers, grid = 2, 3
    words = nat.trace_words(layers)
    raw = torch.zeros(grid, words, dtype=torch.int64)
    ends = 5 * layers + 2
    t = 1_000_000  # ns
    for c in range(grid):
        raw[c, 0] = t
    clock = t
    for p in range(1, ends + 1):
        b = 1 + 5 * (p - 1)
        for c in range(grid):
            raw[c, b - 3 if p > 1 else 0] = clock + 1000 if p > 1 else t  # staged 1 us after the phase start
            raw[c, b] = clock + 3000 + 100 * c                             # arrivals 3.0, 3.1, 3.2 us
            raw[c, b + 1] = clock + 3500                                   # release 3.5 us
        clock += 3500
    raw[:, words - 2] = clock + 2000
    raw[0, words - 1] = clock + 2500
    summary = summarize(raw, layers)
    phases = summary["phases"]
    assert list(phases) == ["embed", "qkv", "attn", "o", "gu", "down", "lm"]
    stage, work, barrier = phases["qkv"]
    assert abs(stage - 2 * 1.0) < 1e-9 and abs(work - 2 * 2.2) < 1e-9 and abs(barrier - 2 * 0.3) < 1e-9
    assert phases["attn"][1] == 0.0
    assert abs(summary["sampling_tail_us"] - 0.5) < 1e-9
    assert "sampling tail 0.5 us" in format_summary(summary, 1234.0, "x")


def test_exchange_staging_of_a_synthetic_tensor_parallel_trace():
    # every phase staged 1 us after its start, except the phases that follow an exchange (gate/up,
    # and QKV from the second layer on), staged 4 us after theirs; 3 layers: 3 + 2 of them
    layers, grid = 3, 4
    words = nat.trace_words(layers)
    raw = torch.zeros(grid, words, dtype=torch.int64)
    ends = 5 * layers + 2
    clock = 1_000_000
    raw[:, 0] = clock
    for p in range(1, ends + 1):
        b = 1 + 5 * (p - 1)
        kind = None if p in (1, ends) else ("qkv", "attn", "o", "gu", "down")[(p - 2) % 5]
        after_exchange = kind == "gu" or (kind == "qkv" and p > 2)
        if p > 1:
            raw[:, b - 3] = clock + (4000 if after_exchange else 1000)
        raw[:, b] = raw[:, b + 1] = clock + 5000
        clock += 5000
    assert abs(exchange_stage_us(raw, layers) - 5 * 4.0) < 1e-9


def test_detail_of_a_synthetic_trace():
    # every phase: staged 1 us after its start, first stage 0.5 us later, last stage 2 us after that,
    # arrival 0.25 us after the last stage, release 0.25 us after the arrival
    layers, grid = 2, 2
    words = nat.trace_words(layers)
    raw = torch.zeros(grid, words, dtype=torch.int64)
    ends = 5 * layers + 2
    clock = 1_000_000
    raw[:, 0] = clock
    for p in range(1, ends + 1):
        b = 1 + 5 * (p - 1)
        if p > 1:
            raw[:, b - 3] = clock + 1000
            raw[:, b - 2] = clock + 1500
            raw[:, b - 1] = clock + 3500
        raw[:, b] = clock + 3750
        raw[:, b + 1] = clock + 4000
        clock += 4000
    table = detail(raw, layers)
    span, stage, first, stream, tail, barrier = table["gu"]
    assert abs(span - 2 * 4.0) < 1e-9 and abs(stage - 2 * 1.0) < 1e-9 and abs(first - 2 * 0.5) < 1e-9
    assert abs(stream - 2 * 2.0) < 1e-9 and abs(tail - 2 * 0.25) < 1e-9 and abs(barrier - 2 * 0.25) < 1e-9
    assert "stream" in format_detail(table)
