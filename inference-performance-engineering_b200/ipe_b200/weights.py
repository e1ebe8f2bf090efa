"""The weight interface the hot path consumes.

Field names, order and layout ([out, in]) follow the reference's dataclasses
(`src/ipe/weights.py:38-75`): a `LoadedCheckpoint` built by the reference's loader can be passed
to this package unchanged, and the reverse. `lm_head is embed_tokens` whenever the head is tied.
`load_checkpoint` reads a Transformers-style safetensors checkpoint directory, streaming the
payloads straight to the GPU; `ipe_b200.synthetic` builds the random-init models the benchmarks
use.
"""

import ctypes
from dataclasses import dataclass

import torch

from ipe_b200.config import Qwen3Config

DTYPES = (torch.bfloat16, torch.float32, torch.float64)

LAYER_FIELDS = ("input_layernorm", "q_proj", "k_proj", "v_proj", "q_norm", "k_norm", "o_proj",
                "post_attention_layernorm", "gate_proj", "up_proj", "down_proj")


@dataclass(frozen=True, slots=True)
class LayerWeights:
    input_layernorm: torch.Tensor
    q_proj: torch.Tensor
    k_proj: torch.Tensor
    v_proj: torch.Tensor
    q_norm: torch.Tensor
    k_norm: torch.Tensor
    o_proj: torch.Tensor
    post_attention_layernorm: torch.Tensor
    gate_proj: torch.Tensor
    up_proj: torch.Tensor
    down_proj: torch.Tensor


@dataclass(frozen=True, slots=True)
class Qwen3Weights:
    embed_tokens: torch.Tensor
    layers: tuple[LayerWeights, ...]
    norm: torch.Tensor
    lm_head: torch.Tensor  # the same object as embed_tokens whenever tied


@dataclass(frozen=True, slots=True)
class TieRecord:
    stored: bool
    tied: bool
    max_abs_diff: float | None


@dataclass(frozen=True, slots=True)
class LoadedCheckpoint:
    config: Qwen3Config
    weights: Qwen3Weights
    tie: TieRecord


# ------------------------------------------------------------------------------------ loading

# Rows per chunk when comparing the embedding with a stored head (bounds the fp32 temporaries).
_DIFF_ROWS = 4096
STAGING_BYTES = 4 * 1024 * 1024  # per staging buffer; each reader thread has two
READERS = 8


def _check_arguments(dtype: torch.dtype, device) -> torch.device:
    if dtype not in DTYPES:
        raise ValueError(f"dtype {dtype!r}: expected one of {list(DTYPES)}")
    if not isinstance(device, (str, torch.device)):
        raise ValueError(f"device {device!r}: expected a string or torch.device")
    try:
        device = torch.device(device)
    except RuntimeError as error:
        raise ValueError(f"device {device!r}: {error}") from error
    if device.type == "cpu":
        if device.index not in (None, 0):
            raise ValueError(f"device {device}: only index 0 exists")
    elif device.type == "cuda":
        if not torch.cuda.is_available():
            raise ValueError("device cuda: not available")
        if device.index is not None and device.index >= torch.cuda.device_count():
            raise ValueError(f"device {device}: only {torch.cuda.device_count()} CUDA device(s)")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
    else:
        raise ValueError(f"device {device}: expected cpu or cuda")
    return device


def _max_abs_diff(a: torch.Tensor, b: torch.Tensor) -> float:
    """fp32 max |a - b| over unequal positions (equal ones count 0, so equal infinities give 0)."""
    result = torch.zeros((), dtype=torch.float32, device=a.device)
    for start in range(0, a.shape[0], _DIFF_ROWS):
        x, y = a[start:start + _DIFF_ROWS].float(), b[start:start + _DIFF_ROWS].float()
        result = torch.maximum(result, torch.where(x == y, 0.0, (x - y).abs()).amax())
    return result.item()


def _tie_record(stored: dict[str, torch.Tensor]) -> TieRecord:
    """Tied when the head is not stored, or equals the embedding in value (torch.equal: +0 equals
    -0, NaN equals nothing), as src/ipe/weights.py:113-124 decides it."""
    from ipe_b200.checkpoint import EMBED_TOKENS, LM_HEAD

    if LM_HEAD not in stored:
        return TieRecord(stored=False, tied=True, max_abs_diff=None)
    embed, head = stored[EMBED_TOKENS], stored[LM_HEAD]
    tied = torch.equal(embed, head)
    return TieRecord(stored=True, tied=tied, max_abs_diff=0.0 if tied else _max_abs_diff(embed, head))


def _read_cpu(root, inventory) -> dict[str, torch.Tensor]:
    """bf16 CPU tensors as copy-on-write views of one private mapping per file."""
    import mmap

    stored = {}
    for file in sorted({info.file for info in inventory.values()}):
        with open(root / file, "rb") as handle:
            mapping = mmap.mmap(handle.fileno(), 0, access=mmap.ACCESS_COPY) if (root / file).stat().st_size else None
        for name, info in inventory.items():
            if info.file != file:
                continue
            if info.nbytes == 0:
                stored[name] = torch.empty(info.shape, dtype=torch.bfloat16)
            else:
                flat = torch.frombuffer(mapping, dtype=torch.bfloat16, count=info.nbytes // 2, offset=info.offset)
                stored[name] = flat.view(info.shape)
    return stored


def _read_cuda(root, inventory, device: torch.device, staging_bytes: int, readers: int) -> dict[str, torch.Tensor]:
    """bf16 device tensors, carved (256-byte aligned) from one device allocation, since hundreds of
    separate allocations cost far more than the reads; a stored LM head gets its own allocation,
    so that dropping it when tied frees it. Every payload of every file is streamed by one
    ipe_read_to_device call."""
    from ipe_b200 import _native as nat
    from ipe_b200.checkpoint import LM_HEAD

    lib = nat.load()
    align = 256
    names = [n for n in inventory if n != LM_HEAD]
    layout, total = {}, 0
    for name in names:
        layout[name] = total
        total += (inventory[name].nbytes + align - 1) // align * align
    block = torch.empty(max(total, align), dtype=torch.uint8, device=device)
    stored = {}
    for name in names:
        info = inventory[name]
        stored[name] = block[layout[name]:layout[name] + info.nbytes].view(torch.bfloat16).view(info.shape)
    if LM_HEAD in inventory:
        stored[LM_HEAD] = torch.empty(inventory[LM_HEAD].shape, dtype=torch.bfloat16, device=device)
    files = sorted({info.file for info in inventory.values()})
    ranges = sorted((n for n, i in inventory.items() if i.nbytes), key=lambda n: (files.index(inventory[n].file),
                                                                                 inventory[n].offset))
    count = len(ranges)
    paths = (ctypes.c_char_p * len(files))(*[str(root / f).encode() for f in files])
    file_of = (ctypes.c_int * max(count, 1))(*[files.index(inventory[n].file) for n in ranges])
    offsets = (ctypes.c_uint64 * max(count, 1))(*[inventory[n].offset for n in ranges])
    sizes = (ctypes.c_uint64 * max(count, 1))(*[inventory[n].nbytes for n in ranges])
    dsts = (ctypes.c_void_p * max(count, 1))(*[stored[n].data_ptr() for n in ranges])
    stream = torch.cuda.current_stream(device).cuda_stream
    status = lib.ipe_read_to_device(len(files), paths, count, file_of, offsets, sizes, dsts, staging_bytes, readers,
                                    stream)
    if status == 4:  # IPE_ERR_IO
        raise OSError(lib.ipe_last_error().decode(errors="replace"))
    nat.check(status, "ipe_read_to_device")
    return stored


def load_checkpoint(directory, *, dtype: torch.dtype, device, staging_bytes: int = STAGING_BYTES,
                    readers: int = READERS) -> LoadedCheckpoint:
    """Validate a checkpoint directory from its headers, then load its tensors at `dtype` on
    `device` (src/ipe/weights.py:135-168).

    dtype is bfloat16, float32 or float64; device is cpu or an available CUDA device. On a CUDA
    device every payload is streamed from the files straight into its device tensor by `readers`
    threads, each reading chunks of up to staging_bytes into one of its two pinned buffers while
    the other's host-to-device copy runs; wider dtypes are exact casts made on the device. On the CPU, bf16 tensors are copy-on-write views of
    the files. A stored LM head equal to the embedding is dropped and lm_head is the embedding
    itself. If loading fails after the checks, every held tensor is dropped and the callee frames
    are cleared, so a traceback kept by the caller does not pin the weights. Errors: ValueError
    for dtype or device, ConfigError, CheckpointError, OSError for file access.
    """
    import traceback
    from pathlib import Path

    from ipe_b200.checkpoint import EMBED_TOKENS, FINAL_NORM, LAYER_TENSORS, LM_HEAD, check_mapping, \
        inspect_checkpoint, read_config

    device = _check_arguments(dtype, device)
    root = Path(directory)
    config = read_config(root / "config.json")
    inventory = inspect_checkpoint(root)
    check_mapping(inventory, config)
    stored: dict[str, torch.Tensor] = {}
    loaded: dict[str, torch.Tensor] = {}
    try:
        if device.type == "cuda":
            with torch.cuda.device(device):
                stored = _read_cuda(root, inventory, device, int(staging_bytes), int(readers))
        else:
            stored = _read_cpu(root, inventory)
        tie = _tie_record(stored)
        for name in inventory:
            if not (tie.tied and name == LM_HEAD):
                loaded[name] = stored[name] if dtype == torch.bfloat16 else stored[name].to(dtype)
        stored.clear()
        embed = loaded[EMBED_TOKENS]
        layers = tuple(
            LayerWeights(**{field: loaded[f"model.layers.{layer}.{suffix}"] for field, suffix in LAYER_TENSORS.items()})
            for layer in range(config.num_hidden_layers))
        weights = Qwen3Weights(embed, layers, loaded[FINAL_NORM], embed if tie.tied else loaded[LM_HEAD])
    except BaseException as error:
        stored.clear()
        loaded.clear()
        traceback.clear_frames(error.__traceback__.tb_next)
        raise
    return LoadedCheckpoint(config, weights, tie)
