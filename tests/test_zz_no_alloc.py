"""The allocation-free decode attention entry point, for callers that cannot allocate device memory
(a host that hands a plugin only its inputs and outputs, or a loop that must not call cudaMalloc).

`ipe_decode_attention_static_scratch` keeps its split partials in a fixed array inside the library
instead of a caller workspace. Called through the C-ABI, its output must match the workspace entry
point `ipe_decode_attention` within the tolerance the other attention tests use, on two calls in a
row (the second smaller, so the array still holds the first call's partials beyond what it writes),
and both must match an fp32 PyTorch attention of the same bf16 operands. The position can also come
from a device step state, a request just under the 2 MiB limit is accepted, and a device position
outside the cache makes both entry points touch nothing and set device error 2.
This file is collected last and runs alone or after the other tests.
"""

import pytest
import torch

from ipe_b200 import _native as nat

pytestmark = pytest.mark.gpu
BF16_REL = 2.0 ** -7
LIMIT = 2 << 20


def operands(batch, q_heads, kv_heads, capacity, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((batch, q_heads, 1, 128), generator=g).bfloat16().cuda()
    k = torch.randn((batch, kv_heads, capacity, 128), generator=g).bfloat16().cuda()
    v = torch.randn((batch, kv_heads, capacity, 128), generator=g).bfloat16().cuda()
    return q, k, v


def attention_fp32(q, k, v, length):
    """fp32 GQA attention of one query per row over keys 0..length-1 (src/ipe/ops.py:66-101)."""
    group = q.shape[1] // k.shape[1]
    kk = k[:, :, :length].float().repeat_interleave(group, 1)
    vv = v[:, :, :length].float().repeat_interleave(group, 1)
    scores = (q.float() @ kk.transpose(-1, -2)) * 128 ** -0.5
    return (scores.softmax(-1) @ vv).reshape(q.shape[0], -1)


def state_at(position):
    state = torch.zeros(nat.STATE_WORDS, dtype=torch.int64, device="cuda")
    state[nat.STATE_POS] = position
    return state


def run_pair(q, k, v, length, state=None):
    """The workspace entry point and the static-scratch one on the same operands."""
    batch, q_heads, kv_heads, capacity = q.shape[0], q.shape[1], k.shape[1], k.shape[2]
    stream = torch.cuda.current_stream().cuda_stream
    lib = nat.load()
    ws = torch.empty(int(lib.ipe_decode_attention_workspace(batch, q_heads, capacity)), dtype=torch.uint8,
                     device="cuda")
    state_ptr = None if state is None else state.data_ptr()
    expected = torch.full((batch, q_heads * 128), 7.0, dtype=torch.bfloat16, device="cuda")
    nat.call("ipe_decode_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), expected.data_ptr(), batch, q_heads,
             kv_heads, capacity, length, state_ptr, ws.data_ptr(), ws.numel(), stream)
    actual = torch.full_like(expected, 7.0)
    nat.call("ipe_decode_attention_static_scratch", q.data_ptr(), k.data_ptr(), v.data_ptr(), actual.data_ptr(),
             batch, q_heads, kv_heads, capacity, length, state_ptr, stream)
    torch.cuda.synchronize()
    return actual.float(), expected.float()


def close(actual, expected, reference):
    assert int(((actual - expected).abs() > 2 * BF16_REL * expected.abs() + 2e-3).sum()) == 0
    # and both against fp32 attention of the same bf16 operands (one bf16 rounding of the output)
    for out in (actual, expected):
        assert int(((out - reference).abs() > 2 * BF16_REL * reference.abs() + 2e-3).sum()) == 0


def test_static_scratch_matches_the_workspace_entry_point_on_two_calls_in_a_row():
    nat.device_error(reset=True)
    for batch, q_heads, kv_heads, capacity, length, seed in ((2, 16, 8, 640, 600, 1), (1, 16, 8, 128, 40, 2)):
        q, k, v = operands(batch, q_heads, kv_heads, capacity, seed)
        actual, expected = run_pair(q, k, v, length)
        close(actual, expected, attention_fp32(q, k, v, length))
    assert nat.device_error(reset=True) == 0


def test_static_scratch_reads_the_position_from_a_device_state():
    nat.device_error(reset=True)
    q, k, v = operands(2, 16, 8, 512, 3)
    for position in (300, 17):  # two calls in a row through the state, the second shorter
        actual, expected = run_pair(q, k, v, 0, state=state_at(position))
        close(actual, expected, attention_fp32(q, k, v, position + 1))
    assert nat.device_error(reset=True) == 0


def test_a_request_just_under_the_limit_is_accepted():
    lib = nat.load()
    capacity = 8064  # 252 chunks of 32 keys x 16 heads x 130 floats: 2,096,640 bytes
    need = int(lib.ipe_decode_attention_workspace(1, 16, capacity))
    assert LIMIT - 8320 < need <= LIMIT
    assert int(lib.ipe_decode_attention_workspace(1, 16, capacity + 32)) > LIMIT
    q, k, v = operands(1, 16, 8, capacity, 4)
    actual, expected = run_pair(q, k, v, capacity)
    close(actual, expected, attention_fp32(q, k, v, capacity))


def test_a_device_position_outside_the_cache_touches_nothing():
    q, k, v = operands(1, 16, 8, 64, 5)
    for position in (64, -3):
        nat.device_error(reset=True)
        actual, expected = run_pair(q, k, v, 0, state=state_at(position))
        assert nat.device_error(reset=True) == 2
        assert bool((actual == 7.0).all()) and bool((expected == 7.0).all())


def test_sizes_beyond_the_static_scratch_are_rejected_before_launch():
    lib = nat.load()
    status = lib.ipe_decode_attention_static_scratch(16, 16, 16, 16, 16, 16, 8, 4096, 10, None, None)
    assert status == 2
    assert b"2 MiB" in lib.ipe_last_error()
