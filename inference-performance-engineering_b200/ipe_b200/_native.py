"""ctypes binding of libipe_b200.so, the C-ABI declared in include/ipe_b200.h.

The library is loaded from `ipe_b200/lib/` (built in-tree by `ipe_b200.build`). There is no
fallback: if the library is missing or fails to load, every call raises `NativeUnavailable`.
A nonzero ipe_status becomes a RuntimeError carrying `ipe_last_error()`; the entry points check
their arguments on the host before launching anything.
"""

from __future__ import annotations

import ctypes
from ctypes import c_float, c_int, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "lib" / "libipe_b200.so"

# enum values of include/ipe_b200.h
EPI_STORE, EPI_RESIDUAL, EPI_SILU_MUL, EPI_LOGITS, EPI_PARTIAL = 0, 1, 2, 3, 4
STATE_POS, STATE_STEP, STATE_SEED, STATE_TEMPERATURE, STATE_WORDS = 0, 1, 2, 3, 8
GATE_UP_GROUP = 64
PARTIAL_WORDS = 8

_P = c_void_p
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "ipe_last_error": (ctypes.c_char_p, []),
    "ipe_abi_version": (c_int, []),
    "ipe_device_error": (c_int, [c_int, ctypes.POINTER(c_int)]),
    "ipe_rmsnorm": (c_int, [_P, _P, _P, c_int64, c_int, c_float, c_int, _P]),
    "ipe_embed": (c_int, [_P, c_int64, _P, c_int64, c_int, _P, _P]),
    "ipe_qk_norm_rope_append": (c_int, [_P, c_int, c_int, c_int, c_int, _P, _P, _P, _P, c_int, _P, _P, _P, _P,
                                        c_int, c_float, _P]),
    "ipe_decode_linear_workspace": (c_size_t, [c_int, c_int, c_int]),
    "ipe_decode_tiles": (c_int, [_P, _P, _P, c_int, c_int, _P]),
    "ipe_decode_tiles_bytes": (c_size_t, [c_int, c_int, c_int]),
    "ipe_rmsnorm_qkv": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_float, _P, c_size_t, _P]),
    "ipe_linear_residual": (c_int, [_P, _P, _P, c_int, c_int, c_int, _P, c_size_t, _P]),
    "ipe_rmsnorm_gate_up_silu": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_float, _P, c_size_t, _P]),
    "ipe_lm_head": (c_int, [_P, c_int64, _P, _P, _P, _P, c_int, c_int, c_int, c_float, c_float, c_uint64, _P, _P]),
    "ipe_lm_head_parts": (c_int, [c_int]),
    "ipe_sample": (c_int, [_P, _P, c_int, c_int, c_float, _P, _P, _P, c_int64, _P, _P]),
    "ipe_sample_logits": (c_int, [_P, c_int64, c_int, c_float, c_uint64, _P, _P, _P]),
    "ipe_decode_attention": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P, _P, c_size_t, _P]),
    "ipe_decode_attention_workspace": (c_size_t, [c_int, c_int, c_int]),
    "ipe_decode_attention_qkv": (c_int, [_P, _P, _P, _P, _P, c_int, _P, _P, _P, _P, c_int, c_int, c_int, c_int,
                                         c_float, _P, c_size_t, _P]),
    "ipe_decode_attention_qkv_workspace": (c_size_t, [c_int, c_int, c_int, c_int]),
    "ipe_decode_attention_static_scratch": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P, _P]),
    "ipe_prefill_attention": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, _P]),
    "ipe_gemm": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, _P, _P]),
    "ipe_decode_step": (c_int, [ctypes.c_void_p, _P]),
    "ipe_decode_step_workspace": (c_size_t, [c_int, c_int, c_int, c_int]),
    "ipe_decode_step_grid": (c_int, []),
    "ipe_decode_step_comm_bytes": (c_size_t, [c_int, c_int, c_int]),
    "ipe_read_to_device": (c_int, [c_int, _P, c_int, _P, _P, _P, _P, c_size_t, c_int, _P]),
    "ipe_gemm_f32": (c_int, [_P, _P, _P, c_int, c_int, c_int, c_int, _P, _P]),
    "ipe_embed_f32": (c_int, [_P, c_int64, _P, c_int64, c_int, _P, _P]),
    "ipe_qk_norm_rope_append_f32": (c_int, [_P, c_int, c_int, c_int, c_int, _P, _P, _P, _P, c_int, _P, _P, _P, c_int,
                                            c_float, _P]),
    "ipe_attention_f32": (c_int, [_P, _P, _P, _P, c_int, c_int, c_int, c_int, c_int, c_int, _P]),
    "ipe_linear_partial": (c_int, [_P, _P, _P, c_int, c_int, c_int, _P, c_size_t, _P]),
    "ipe_add_partial": (c_int, [_P, _P, c_int64, _P]),
    "ipe_lm_head_shard": (c_int, [_P, c_int64, _P, _P, _P, _P, c_int, c_int, c_int, c_int, c_float, c_float, c_uint64,
                                  _P, _P]),
    "ipe_sample_records": (c_int, [_P, c_int, c_int, c_float, _P, _P, _P, c_int64, _P, _P]),
    "ipe_comm_bytes": (c_size_t, [c_size_t]),
    "ipe_comm_slot_offset": (c_size_t, [c_int, c_size_t]),
    "ipe_comm_alloc": (c_int, [c_size_t, ctypes.POINTER(c_void_p)]),
    "ipe_comm_free": (c_int, [_P]),
    "ipe_ipc_handle": (c_int, [_P, _P]),
    "ipe_ipc_open": (c_int, [_P, ctypes.POINTER(c_void_p)]),
    "ipe_ipc_close": (c_int, [_P]),
    "ipe_allreduce_residual": (c_int, [_P, c_int64, _P, c_int, c_int, c_int, c_size_t, _P]),
    "ipe_state_set": (c_int, [_P, c_int, c_int64, _P]),
    "ipe_state_add": (c_int, [_P, c_int, c_int64, _P]),
}


class LayerDesc(ctypes.Structure):
    """ipe_layer_desc of include/ipe_b200.h."""

    _fields_ = [(name, c_void_p) for name in (
        "input_layernorm", "post_attention_layernorm", "q_norm", "k_norm", "qkv_tiles", "o_tiles", "gate_up_tiles",
        "down_tiles", "k_cache", "v_cache")]


class StepDesc(ctypes.Structure):
    """ipe_decode_step_desc of include/ipe_b200.h."""

    _fields_ = [("layers", c_int), ("hidden", c_int), ("intermediate", c_int), ("q_heads", c_int),
                ("kv_heads", c_int), ("vocab", c_int), ("capacity", c_int), ("batch", c_int), ("eps", c_float),
                ("layer_descs", c_void_p), ("embed", c_void_p), ("lm_head_tiles", c_void_p), ("final_norm", c_void_p),
                ("cos_table", c_void_p), ("sin_table", c_void_p), ("state", c_void_p), ("tokens", c_void_p),
                ("x", c_void_p), ("qkv", c_void_p), ("attn", c_void_p), ("act", c_void_p), ("logits", c_void_p),
                ("partials", c_void_p), ("workspace", c_void_p), ("workspace_bytes", c_size_t),
                ("history_tokens", c_void_p), ("history_logprobs", c_void_p), ("history_stride", c_int64),
                ("trace", c_void_p), ("tp_world", c_int), ("tp_rank", c_int), ("tp_peers", c_void_p),
                ("x_alt", c_void_p), ("vocab_offset", c_int), ("vocab_total", c_int), ("wait_limit_ns", c_int64)]


def trace_words(layers: int) -> int:
    """IPE_TRACE_WORDS of include/ipe_b200.h: timestamps per CTA of one traced decode step."""
    return 25 * layers + 13


class NativeUnavailable(RuntimeError):
    """The CUDA library could not be loaded; the package has no other implementation."""


_lib: ctypes.CDLL | None = None
_load_error: str | None = None


def load() -> ctypes.CDLL:
    global _lib, _load_error
    if _lib is not None:
        return _lib
    if _load_error is not None:
        raise NativeUnavailable(_load_error)
    if not LIBRARY.exists():
        _load_error = f"{LIBRARY} is missing: build it with `python -m ipe_b200.build` (needs nvcc)"
        raise NativeUnavailable(_load_error)
    try:
        lib = ctypes.CDLL(str(LIBRARY))
    except OSError as error:
        _load_error = f"cannot load {LIBRARY}: {error}"
        raise NativeUnavailable(_load_error) from error
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def check(status: int, name: str) -> None:
    if status != 0:
        message = load().ipe_last_error().decode(errors="replace")
        raise RuntimeError(f"{name} failed (status {status}): {message}")


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args), name)


def device_error(reset: bool = True) -> int:
    """The first device-side error code since the last reset (synchronises the device)."""
    code = c_int(0)
    call("ipe_device_error", 1 if reset else 0, ctypes.byref(code))
    return code.value
