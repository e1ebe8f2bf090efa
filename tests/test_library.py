"""The C-ABI library without a GPU: it loads, exports every function include/ipe_b200.h declares,
and rejects bad arguments on the host before launching anything (no device call is made)."""

import ctypes
import re

import pytest

from conftest import REPO
from ipe_b200 import _native as nat

HEADER = REPO / "include" / "ipe_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(ipe_\w+)\s*\(", text, flags=re.M)))


def test_the_library_is_built_in_tree_and_loads():
    assert nat.LIBRARY.exists(), "run __graft_entry__.build() first"
    lib = nat.load()
    assert lib.ipe_abi_version() == 1


def test_every_declared_function_is_exported_and_bound():
    names = declared_functions()
    assert len(names) >= 18, names
    lib = nat.load()
    for name in names:
        assert hasattr(lib, name), name
        assert name in nat.SIGNATURES, f"{name} has no ctypes signature"


def test_the_binding_declares_nothing_the_header_lacks():
    assert set(nat.SIGNATURES) <= set(declared_functions())


@pytest.mark.parametrize(("name", "args"), [
    ("ipe_rmsnorm", (None, None, None, 4, 8, 1e-6, 0, None)),
    ("ipe_rmsnorm", (16, 16, 16, 4, 0, 1e-6, 0, None)),
    ("ipe_rmsnorm", (16, 16, 16, 4, 8, 1e-6, 7, None)),
    ("ipe_embed", (16, 4, 16, 10, 12, 16, None)),
    ("ipe_gemm", (16, 16, 16, 128, 100, 64, 0, None, None)),
    ("ipe_gemm", (16, 16, 16, 128, 128, 48, 0, None, None)),
    ("ipe_gemm", (16, 16, 16, 128, 128, 64, 1, None, None)),
    ("ipe_gemm", (16, 16, 16, 128, 128, 64, 9, None, None)),
    ("ipe_rmsnorm_qkv", (16, 16, 16, 16, 17, 2048, 4096, 1e-6, 16, 1 << 30, None)),
    ("ipe_rmsnorm_qkv", (16, 16, 16, 16, 1, 2047, 4096, 1e-6, 16, 1 << 30, None)),
    ("ipe_rmsnorm_qkv", (16, 16, 16, 16, 1, 2048, 4096, 1e-6, None, 0, None)),
    ("ipe_linear_residual", (16, 16, 16, 1, 2048, 2048, 16, 16, None)),
    ("ipe_rmsnorm_gate_up_silu", (16, 16, 16, 16, 1, 2048, 100, 1e-6, 16, 1 << 30, None)),
    ("ipe_decode_attention", (16, 16, 16, 16, 1, 16, 8, 64, 65, None, 16, 1 << 20, None)),
    ("ipe_decode_attention", (16, 16, 16, 16, 1, 12, 8, 64, 8, None, 16, 1 << 20, None)),
    ("ipe_decode_attention", (16, 16, 16, 16, 1, 16, 8, 64, 8, None, 16, 0, None)),
    ("ipe_prefill_attention", (16, 16, 16, 16, 1, 16, 8, 65, 64, None)),
    ("ipe_prefill_attention", (16, 16, 16, 17, 1, 16, 8, 8, 64, None)),
    ("ipe_qk_norm_rope_append", (16, 1, 4, 16, 8, 16, 16, 16, 16, 62, None, 16, 16, 16, 64, 1e-6, None)),
    ("ipe_sample", (16, 16, 17, 100, 0.0, None, 16, 16, 1, None, None)),
    ("ipe_sample_logits", (16, 4, 100, -1.0, 0, 16, 16, None)),
    ("ipe_lm_head", (16, 2048, 16, 16, 16, 16, 1, 2048, 1000, 1e-6, -0.5, 0, None, None)),
    ("ipe_state_set", (16, 8, 0, None)),
])
def test_bad_arguments_are_rejected_on_the_host(name, args):
    status = getattr(nat.load(), name)(*args)
    assert status in (1, 2), (name, status)
    assert nat.load().ipe_last_error().decode().startswith(name)


def test_a_failed_call_raises_with_the_library_message():
    with pytest.raises(RuntimeError, match="ipe_gemm"):
        nat.call("ipe_gemm", 16, 16, 16, 128, 100, 64, 0, None, None)


def test_device_error_needs_an_output_pointer():
    assert nat.load().ipe_device_error(0, ctypes.POINTER(ctypes.c_int)()) == 1


def test_the_custom_ops_of_the_boundary_are_registered():
    """torch.ops.ipe_b200 holds the operator set the drop-in boundary names (plus the helpers)."""
    import torch

    import ipe_b200.ops  # noqa: F401

    for name in ("rms_norm", "rmsnorm_qkv", "qk_norm_rope_append", "decode_attention", "prefill_attention",
                 "linear_residual", "rmsnorm_gate_up_silu", "lm_head_sample", "gemm", "embed", "sample_logits",
                 "decode_tiles"):
        assert hasattr(torch.ops.ipe_b200, name), name
