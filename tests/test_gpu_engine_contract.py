"""The reference's engine-contract cases that go through its per-layer hook, restated against
ipe_b200 on the GPU (the reference's test modules are not importable where these run, so each case
is restated here and cites the reference test it follows).

The reference's tests replace `ipe.engine.decoder_layer` to wrap, fail or mis-rotate a layer
(tests/needs_torch/test_engine.py:130-188, :243-261) and trace what a step does on the device
(:343-366). `ipe_b200.engine.decoder_layer` has the same signature (src/ipe/forward.py:86-88), so
the same wrappers drive this engine: the engine then calls the replacement for every layer of
every step, and the replacement calls the built-in layer (the per-operator CUDA kernels).
"""

import pytest
import torch
from torch.utils._python_dispatch import TorchDispatchMode

from cases import build, to_device
from ipe_b200 import engine as engine_module
from ipe_b200.engine import Engine
from ipe_b200.fp32 import rotary_rows_f32
from ipe_b200.model import rotary_rows
from oracle import accuracy
from oracle import qwen3 as oq

pytestmark = pytest.mark.gpu
BF16, F32 = torch.bfloat16, torch.float32
PROMPT = 6


@pytest.fixture(scope="module")
def small():
    cpu = build("small")
    return cpu, to_device(cpu, "cuda")


def ids_of(batch, length, seed):
    return torch.randint(0, 2048, (batch, length), generator=torch.Generator().manual_seed(seed))


def teacher_forced(engine, ids, prompt):
    return oq.teacher_forced(engine, ids, prompt).cpu()


def late_rope(real, when, dtype):
    """A hook that rotates decode steps one position late when `when(start)` (the reference's
    seeded bugs "decode rotated one position late" and "first decode step rotated one position
    late", tests/needs_torch/test_engine.py:134-149)."""
    def hook(x, layer, rope, config, *, backend, cache=None, start=0):
        if start > 0 and when(start):
            rows = rotary_rows_f32 if dtype == F32 else rotary_rows
            cos, sin = rows(torch.arange(start, start + 2), config.head_dim, config.rope_theta)
            rope = (cos[1:].to(x.device), sin[1:].to(x.device))
        return real(x, layer, rope, config, backend=backend, cache=cache, start=start)
    return hook


@pytest.mark.parametrize("bug", ("decode rotated one position late", "first decode step rotated one position late"))
def test_the_rule_fails_a_hook_that_rotates_late(small, monkeypatch, bug):
    """tests/needs_torch/test_engine.py:161-168 (at fp32, as there) for the two seeded bugs that
    replace the hook."""
    cpu, gpu = small
    dtype = F32
    ids = ids_of(2, 20, 8)
    positions = list(range(PROMPT - 1, ids.shape[1]))
    oracle = oq.oracle_logits(cpu, ids, positions)
    refs = [accuracy.errors(oracle, oq.forward_full(cpu, ids, dtype=dtype, backend=b, logit_positions=positions))
            for b in oq.BACKENDS]
    clean = teacher_forced(Engine(gpu, batch=2, capacity=24, dtype=dtype), ids, PROMPT)
    assert accuracy.failures(accuracy.errors(oracle, clean), refs) == []
    when = (lambda start: True) if bug.startswith("decode") else (lambda start: start == PROMPT)
    monkeypatch.setattr(engine_module, "decoder_layer", late_rope(engine_module.decoder_layer, when, dtype))
    buggy = teacher_forced(Engine(gpu, batch=2, capacity=24, dtype=dtype), ids, PROMPT)
    assert accuracy.failures(accuracy.errors(oracle, buggy), refs) != []


@pytest.mark.parametrize("dtype", (BF16, F32))
def test_a_forwarding_hook_is_called_for_every_layer_of_every_step(small, monkeypatch, dtype):
    """The engine calls the module global once per layer per step with the reference's arguments
    (src/ipe/engine.py:103-111), and a hook that only forwards keeps the accuracy rule."""
    cpu, gpu = small
    real, calls = engine_module.decoder_layer, []

    def counting(x, layer, rope, config, *, backend, cache=None, start=0):
        calls.append((tuple(x.shape), x.dtype, start, tuple(cache[0].shape), tuple(rope[0].shape), backend))
        return real(x, layer, rope, config, backend=backend, cache=cache, start=start)

    monkeypatch.setattr(engine_module, "decoder_layer", counting)
    ids = ids_of(2, 12, 3)
    engine = Engine(gpu, batch=2, capacity=16, dtype=dtype)
    logits = teacher_forced(engine, ids, PROMPT)
    layers, hidden = gpu.config.num_hidden_layers, gpu.config.hidden_size
    cache = (2, gpu.config.num_key_value_heads, 16, 128)
    expected = [((2, PROMPT, hidden), dtype, 0, cache, (PROMPT, 128), "sdpa")] * layers
    for p in range(PROMPT, 12):
        expected += [((2, 1, hidden), dtype, p, cache, (1, 128), "sdpa")] * layers
    assert calls == expected
    positions = list(range(PROMPT - 1, 12))
    oracle = oq.oracle_logits(cpu, ids, positions)
    refs = [accuracy.errors(oracle, oq.forward_full(cpu, ids, dtype=dtype, backend=b, logit_positions=positions))
            for b in oq.BACKENDS]
    assert accuracy.failures(accuracy.errors(oracle, logits), refs) == []
    # generate goes through the hook too (src/ipe/engine.py:137-147 -> decode -> _step)
    calls.clear()
    out = engine.generate(ids[:, :PROMPT], 3)
    assert out.tokens.shape == (2, 3) and len(calls) == 3 * layers


def test_a_failed_fp32_step_keeps_the_committed_prefix(small, monkeypatch):
    """tests/needs_torch/test_engine.py:243-261 at the reference's own dtype (float32): a layer-1
    failure inside decode leaves length at the prefix, and decoding on gives the fresh engine's
    bits."""
    _, gpu = small
    ids = ids_of(2, 12, 5)
    expected = teacher_forced(Engine(gpu, batch=2, capacity=12, dtype=F32), ids, 6)
    engine = Engine(gpu, batch=2, capacity=12, dtype=F32)
    logits = [engine.prefill(ids[:, :6]).cpu()]
    real, calls = engine_module.decoder_layer, []

    def fail_in_layer_1(*args, **kwargs):
        calls.append(None)
        if len(calls) == 2:
            raise RuntimeError("injected")
        return real(*args, **kwargs)

    monkeypatch.setattr(engine_module, "decoder_layer", fail_in_layer_1)
    with pytest.raises(RuntimeError, match="injected"):
        engine.decode(ids[:, 6])  # layer 0 has already written position 6
    monkeypatch.undo()
    assert engine.length == 6
    logits += [engine.decode(ids[:, p]).cpu() for p in range(6, 12)]
    assert torch.equal(torch.stack(logits, 1), expected)


# Operators that read device values to the host (tests/needs_torch/test_engine.py:343-345).
SYNCHRONIZING = {"_local_scalar_dense", "is_nonzero", "equal", "nonzero", "masked_select", "_unique2",
                 "repeat_interleave", "index"}


class Trace(TorchDispatchMode):
    def __init__(self):
        super().__init__()
        self.ops = []

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        self.ops.append(func.overloadpacket.__name__)
        return func(*args, **(kwargs or {}))


@pytest.mark.parametrize("hook", (False, True))
@pytest.mark.parametrize("dtype", (BF16, F32))
def test_a_step_never_reads_device_values(small, monkeypatch, hook, dtype):
    """tests/needs_torch/test_engine.py:358-366: the torch work of a prefill and a decode step
    (`_step`) holds no operator that reads a device value, on the fused path and through a
    replaced hook."""
    _, gpu = small
    if hook:
        real = engine_module.decoder_layer
        monkeypatch.setattr(engine_module, "decoder_layer", lambda *a, **k: real(*a, **k))
    engine = Engine(gpu, batch=2, capacity=16, dtype=dtype)
    engine.prefill(ids_of(2, 8, 0))
    rows = rotary_rows_f32 if dtype == F32 else rotary_rows
    cos, sin = (t.cuda() for t in rows(torch.arange(8), 128, gpu.config.rope_theta))
    with Trace() as trace:
        engine._step(ids_of(2, 8, 0), (cos, sin), 0)
        engine._step(torch.tensor([[1], [2]]), (engine._cos[8:9], engine._sin[8:9]), 8)
    assert SYNCHRONIZING.isdisjoint(trace.ops), sorted(SYNCHRONIZING & set(trace.ops))
