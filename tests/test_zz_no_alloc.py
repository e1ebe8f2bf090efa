"""The allocation-free decode attention entry point, for callers that cannot allocate device memory
(a host that hands a plugin only its inputs and outputs, or a loop that must not call cudaMalloc).

`ipe_decode_attention_static_scratch` keeps its split partials in a fixed array inside the library
instead of a caller workspace. Called through the C-ABI, its output must match the workspace entry
point `ipe_decode_attention` within the tolerance the other attention tests use, on two calls in a
row (the second smaller, so the array still holds the first call's partials beyond what it writes).
This file is collected last and runs alone or after the other tests.
"""

import pytest
import torch

from ipe_b200 import _native as nat

pytestmark = pytest.mark.gpu
BF16_REL = 2.0 ** -7


def attention_pair(batch, q_heads, kv_heads, capacity, length, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((batch, q_heads, 1, 128), generator=g).bfloat16().cuda()
    k = torch.randn((batch, kv_heads, capacity, 128), generator=g).bfloat16().cuda()
    v = torch.randn((batch, kv_heads, capacity, 128), generator=g).bfloat16().cuda()
    stream = torch.cuda.current_stream().cuda_stream
    lib = nat.load()
    ws = torch.empty(int(lib.ipe_decode_attention_workspace(batch, q_heads, capacity)), dtype=torch.uint8,
                     device="cuda")
    expected = torch.empty((batch, q_heads * 128), dtype=torch.bfloat16, device="cuda")
    nat.call("ipe_decode_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), expected.data_ptr(), batch, q_heads,
             kv_heads, capacity, length, None, ws.data_ptr(), ws.numel(), stream)
    actual = torch.empty_like(expected)
    nat.call("ipe_decode_attention_static_scratch", q.data_ptr(), k.data_ptr(), v.data_ptr(), actual.data_ptr(),
             batch, q_heads, kv_heads, capacity, length, None, stream)
    torch.cuda.synchronize()
    return actual.float(), expected.float()


def test_static_scratch_matches_the_workspace_entry_point_on_two_calls_in_a_row():
    for batch, q_heads, kv_heads, capacity, length, seed in ((2, 16, 8, 640, 600, 1), (1, 16, 8, 128, 40, 2)):
        actual, expected = attention_pair(batch, q_heads, kv_heads, capacity, length, seed)
        bad = (actual - expected).abs() > 2 * BF16_REL * expected.abs() + 2e-3
        assert int(bad.sum()) == 0, (batch, capacity, length)


def test_sizes_beyond_the_static_scratch_are_rejected_before_launch():
    lib = nat.load()
    status = lib.ipe_decode_attention_static_scratch(16, 16, 16, 16, 16, 16, 8, 4096, 10, None, None)
    assert status == 2
    assert b"2 MiB" in lib.ipe_last_error()
