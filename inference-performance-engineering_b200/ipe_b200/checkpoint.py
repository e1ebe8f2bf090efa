"""Checkpoint directories: safetensors headers, the tensor inventory and its mapping onto the
engine's weights, read from headers alone (no payload is touched here).

Follows the reference's inspection rules (`src/ipe/checkpoint.py:131-217`):
- a directory holds either `model.safetensors` or `model.safetensors.index.json` with exactly the
  shards its weight_map names, and no other `.safetensors` file;
- no tensor is stored twice, and an index maps exactly the stored names;
- every tensor the engine consumes is stored as BF16 with the shape the config implies, nothing
  else is stored, and a stored `lm_head.weight` must have the embedding's shape.

The safetensors format is read directly (8-byte little-endian header length, a UTF-8 JSON header
of `{name: {dtype, shape, data_offsets}}`, then the payload), so each tensor's absolute byte range
in its file is known and the loader can stream payloads straight to the GPU
(`ipe_b200.weights.load_checkpoint`). `config.json` is read for the fields the engine needs
(`read_config`); the reference's full config admission rules are not restated.

Errors: CheckpointError (a ValueError) naming the file or tensor, ConfigError (a ValueError) for
config.json, OSError for file access.
"""

from __future__ import annotations

import json
import math
import os
import struct
from dataclasses import dataclass
from os import PathLike
from pathlib import Path

import torch

from ipe_b200.config import Qwen3Config
from ipe_b200.weights import LAYER_FIELDS, LoadedCheckpoint


class CheckpointError(ValueError):
    """A checkpoint file, index or tensor inventory is invalid or does not match the config."""


class ConfigError(ValueError):
    """config.json is malformed or describes a model the engine does not run."""


@dataclass(frozen=True, slots=True)
class TensorInfo:
    dtype: str               # safetensors dtype string, e.g. "BF16"
    shape: tuple[int, ...]
    file: str                # file name inside the checkpoint directory
    offset: int              # absolute byte offset of the payload in the file
    nbytes: int


SINGLE_FILE = "model.safetensors"
INDEX_FILE = "model.safetensors.index.json"
EMBED_TOKENS = "model.embed_tokens.weight"
FINAL_NORM = "model.norm.weight"
LM_HEAD = "lm_head.weight"
STORED_DTYPE = "BF16"

# Engine field -> checkpoint name suffix after "model.layers.{i}." (the Transformers names).
LAYER_TENSORS = {
    "input_layernorm": "input_layernorm.weight",
    "q_proj": "self_attn.q_proj.weight",
    "k_proj": "self_attn.k_proj.weight",
    "v_proj": "self_attn.v_proj.weight",
    "q_norm": "self_attn.q_norm.weight",
    "k_norm": "self_attn.k_norm.weight",
    "o_proj": "self_attn.o_proj.weight",
    "post_attention_layernorm": "post_attention_layernorm.weight",
    "gate_proj": "mlp.gate_proj.weight",
    "up_proj": "mlp.up_proj.weight",
    "down_proj": "mlp.down_proj.weight",
}
assert tuple(LAYER_TENSORS) == LAYER_FIELDS

ITEM_BYTES = {"BOOL": 1, "U8": 1, "I8": 1, "F8_E4M3": 1, "F8_E5M2": 1, "I16": 2, "U16": 2, "F16": 2, "BF16": 2,
              "I32": 4, "U32": 4, "F32": 4, "I64": 8, "U64": 8, "F64": 8}
_TORCH_DTYPES = {torch.bfloat16: "BF16", torch.float16: "F16", torch.float32: "F32", torch.float64: "F64"}
# The largest header the reader accepts (safetensors itself caps headers at 100 MB).
MAX_HEADER_BYTES = 100 * 1024 * 1024


# ------------------------------------------------------------------------------------ headers

def read_header(path: str | PathLike[str], file: str | None = None) -> dict[str, TensorInfo]:
    """The tensors of one safetensors file, from its header: dtype, shape and absolute byte range.

    Checks that every range lies in the file, matches its dtype and shape, and that no two ranges
    overlap. `file` is the name recorded in each TensorInfo (default: the path's name).
    """
    path = Path(path)
    file = file or path.name
    size = path.stat().st_size
    with open(path, "rb") as handle:
        head = handle.read(8)
        if len(head) < 8:
            raise CheckpointError(f"{file}: shorter than a safetensors header")
        (length,) = struct.unpack("<Q", head)
        if length > MAX_HEADER_BYTES or 8 + length > size:
            raise CheckpointError(f"{file}: header length {length} does not fit the file ({size} bytes)")
        raw = handle.read(length)
    try:
        document = json.loads(raw.decode("utf-8"))
    except (UnicodeDecodeError, ValueError) as error:
        raise CheckpointError(f"{file}: header is not UTF-8 JSON ({error})") from error
    if not isinstance(document, dict):
        raise CheckpointError(f"{file}: header is not a JSON object")
    base, payload = 8 + length, size - 8 - length
    tensors: dict[str, TensorInfo] = {}
    ranges = []
    for name, entry in document.items():
        if name == "__metadata__":
            continue
        try:
            dtype, shape, (begin, end) = entry["dtype"], tuple(entry["shape"]), entry["data_offsets"]
        except (KeyError, TypeError, ValueError) as error:
            raise CheckpointError(f"{file}: {name}: malformed entry {entry!r}") from error
        if dtype not in ITEM_BYTES:
            raise CheckpointError(f"{file}: {name}: unknown dtype {dtype!r}")
        if not all(type(d) is int and d >= 0 for d in shape):
            raise CheckpointError(f"{file}: {name}: bad shape {list(shape)}")
        if not (type(begin) is int and type(end) is int and 0 <= begin <= end <= payload):
            raise CheckpointError(f"{file}: {name}: data_offsets {[begin, end]} outside the {payload}-byte payload")
        if end - begin != math.prod(shape) * ITEM_BYTES[dtype]:
            raise CheckpointError(f"{file}: {name}: {end - begin} bytes for {dtype} {list(shape)}")
        tensors[name] = TensorInfo(dtype, shape, file, base + begin, end - begin)
        ranges.append((begin, end, name))
    ranges.sort()
    for (b0, e0, n0), (b1, _, n1) in zip(ranges, ranges[1:]):
        if b1 < e0:
            raise CheckpointError(f"{file}: {n0} and {n1} overlap")
    return tensors


def _shard_files(root: Path, entries: set[str]) -> tuple[list[str], dict[str, str] | None]:
    """The safetensors files a checkpoint directory must hold, and its index's name -> file map
    (None for a single-file checkpoint). A directory holds exactly one of model.safetensors or an
    index, and no safetensors file the layout does not name."""
    layouts = [name for name in (SINGLE_FILE, INDEX_FILE) if name in entries]
    if len(layouts) != 1:
        raise CheckpointError(f"{root}: expected exactly one of {SINGLE_FILE} or {INDEX_FILE}")
    weight_map = None
    files = [SINGLE_FILE]
    if layouts[0] == INDEX_FILE:
        try:
            weight_map = dict(json.loads((root / INDEX_FILE).read_text(encoding="utf-8"))["weight_map"])
            files = sorted({str(f) for f in weight_map.values()})
        except (ValueError, KeyError, TypeError, AttributeError) as error:
            raise CheckpointError(f"{INDEX_FILE}: malformed ({error!r})") from error
    present = sorted(e for e in entries if e.endswith(".safetensors"))
    if present != files:
        raise CheckpointError(f"{root}: safetensors files {present}, expected {files}")
    return files, weight_map


def inspect_checkpoint(directory: str | PathLike[str]) -> dict[str, TensorInfo]:
    """Every stored tensor's dtype, shape, file and byte range, from headers alone, sorted by name
    (the rules of src/ipe/checkpoint.py:131-164: one layout, no stray files, no tensor stored
    twice, an index that maps exactly the stored names)."""
    root = Path(directory)
    files, weight_map = _shard_files(root, set(os.listdir(root)))
    inventory: dict[str, TensorInfo] = {}
    for file in files:
        header = read_header(root / file, file)
        for name in header.keys() & inventory.keys():
            raise CheckpointError(f"{name}: stored in both {inventory[name].file} and {file}")
        inventory.update(header)
    if weight_map is not None:
        unmatched = sorted(weight_map.keys() ^ inventory.keys())
        if unmatched:
            raise CheckpointError(f"{INDEX_FILE}: names mapped or stored, but not both: {unmatched}")
    return {name: inventory[name] for name in sorted(inventory)}


# ------------------------------------------------------------------------------------ mapping

def layer_shapes(config: Qwen3Config) -> dict[str, tuple[int, ...]]:
    """The [out, in] (or [n]) shape of each per-layer engine field."""
    c = config
    q_out, kv_out = c.num_attention_heads * c.head_dim, c.num_key_value_heads * c.head_dim
    vector, head = (c.hidden_size,), (c.head_dim,)
    into_hidden, from_hidden = (c.hidden_size, c.intermediate_size), (c.intermediate_size, c.hidden_size)
    table = dict(input_layernorm=vector, post_attention_layernorm=vector, q_norm=head, k_norm=head,
                 q_proj=(q_out, c.hidden_size), k_proj=(kv_out, c.hidden_size), v_proj=(kv_out, c.hidden_size),
                 o_proj=(c.hidden_size, q_out), gate_proj=from_hidden, up_proj=from_hidden, down_proj=into_hidden)
    return {field: table[field] for field in LAYER_TENSORS}


def expected_tensors(config: Qwen3Config) -> dict[str, tuple[int, ...]]:
    """Every tensor the engine consumes, with its shape (the optional stored LM head excluded)."""
    per_layer = layer_shapes(config)
    names = [(EMBED_TOKENS, (config.vocab_size, config.hidden_size))]
    names += [(f"model.layers.{i}.{suffix}", per_layer[field]) for i in range(config.num_hidden_layers)
              for field, suffix in LAYER_TENSORS.items()]
    names.append((FINAL_NORM, (config.hidden_size,)))
    return dict(names)


def check_mapping(inventory: dict[str, TensorInfo], config: Qwen3Config) -> None:
    """Every expected tensor stored as BF16 with its shape and nothing else, plus an optional LM
    head of the embedding's shape (src/ipe/checkpoint.py:184-217); one CheckpointError lists every
    problem."""
    required = expected_tensors(config)
    optional = {LM_HEAD: (config.vocab_size, config.hidden_size)}
    missing = sorted(name for name in required if name not in inventory)
    unexpected, mismatched = [], []
    for name in sorted(inventory):
        info = inventory[name]
        shape = required.get(name, optional.get(name))
        if shape is None:
            unexpected.append(f"{name} in {info.file}")
        elif (info.dtype, tuple(info.shape)) != (STORED_DTYPE, shape):
            mismatched.append(f"{name} in {info.file}: {info.dtype} {list(info.shape)}, expected {STORED_DTYPE} "
                              f"{list(shape)}")
    if missing or unexpected or mismatched:
        raise CheckpointError("checkpoint does not match the configuration: "
                              f"{len(missing)} missing {missing}, {len(unexpected)} unexpected {unexpected}, "
                              f"{len(mismatched)} mismatched [{'; '.join(mismatched)}]")


# ------------------------------------------------------------------------------------- config

_DIMENSIONS = ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
               "num_key_value_heads", "head_dim", "max_position_embeddings")


def read_config(path: str | PathLike[str]) -> Qwen3Config:
    """The engine's fields of a Transformers Qwen3 config.json: a dense, tied, SiLU Qwen3 with
    plain (unscaled, full-head) RoPE. ConfigError otherwise."""
    path = Path(path)
    try:
        document = json.loads(path.read_text(encoding="utf-8"))
    except ValueError as error:
        raise ConfigError(f"{path}: {error}") from error
    if not isinstance(document, dict):
        raise ConfigError(f"{path}: expected a JSON object")

    def need(field):
        if field not in document:
            raise ConfigError(f"{path}: {field}: an explicit value is required")
        return document[field]

    for field, expected in (("model_type", "qwen3"), ("hidden_act", "silu"), ("tie_word_embeddings", True)):
        if need(field) != expected:
            raise ConfigError(f"{path}: {field}: only {expected!r} is supported")
    for field in ("attention_bias", "use_sliding_window"):
        if document.get(field, False) is not False:
            raise ConfigError(f"{path}: {field}: only false is supported")
    dims = {}
    for field in _DIMENSIONS:
        value = need(field)
        if type(value) is not int or value < 1:
            raise ConfigError(f"{path}: {field}: expected a positive integer")
        dims[field] = value
    thetas = [document["rope_theta"]] if "rope_theta" in document else []
    for field in ("rope_scaling", "rope_parameters"):
        params = document.get(field)
        if params is None:
            continue
        if not isinstance(params, dict) or any(params.get(k, "default") != "default" for k in ("type", "rope_type")):
            raise ConfigError(f"{path}: {field}: only unscaled default RoPE is supported")
        if params.get("partial_rotary_factor", 1.0) != 1.0:
            raise ConfigError(f"{path}: {field}: only full-head rotary is supported")
        if "rope_theta" in params:
            thetas.append(params["rope_theta"])
    if not thetas or any(type(t) not in (int, float) or not math.isfinite(t) or t <= 0 for t in thetas) \
            or len(set(float(t) for t in thetas)) != 1:
        raise ConfigError(f"{path}: rope_theta: one explicit positive value is required")
    eps = need("rms_norm_eps")
    if type(eps) not in (int, float) or not math.isfinite(eps) or eps <= 0:
        raise ConfigError(f"{path}: rms_norm_eps: expected a positive number")
    if dims["num_attention_heads"] % dims["num_key_value_heads"]:
        raise ConfigError(f"{path}: num_attention_heads must be divisible by num_key_value_heads")
    return Qwen3Config(**dims, rms_norm_eps=float(eps), rope_theta=float(thetas[0]))


def config_document(config: Qwen3Config) -> dict:
    """A Transformers-style config.json object for `config` (what read_config accepts)."""
    return {"architectures": ["Qwen3ForCausalLM"], "model_type": "qwen3", "hidden_act": "silu",
            "tie_word_embeddings": True, "attention_bias": False, "attention_dropout": 0.0,
            "use_sliding_window": False, **{f: getattr(config, f) for f in _DIMENSIONS},
            "rms_norm_eps": config.rms_norm_eps, "rope_theta": config.rope_theta, "torch_dtype": "bfloat16",
            "bos_token_id": 0, "eos_token_id": 0}


# ------------------------------------------------------------------------------------- writer

def _write_file(path: Path, tensors: dict[str, torch.Tensor]) -> None:
    header, offset = {}, 0
    for name, t in tensors.items():
        if t.dtype not in _TORCH_DTYPES:
            raise ValueError(f"{name}: dtype {t.dtype} is not written")
        nbytes = t.numel() * t.element_size()
        header[name] = {"dtype": _TORCH_DTYPES[t.dtype], "shape": list(t.shape), "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
    raw = json.dumps(header, separators=(",", ":")).encode("utf-8")
    raw += b" " * (-(8 + len(raw)) % 8)  # payload 8-byte aligned, as safetensors writers do
    with open(path, "wb") as out:
        out.write(struct.pack("<Q", len(raw)))
        out.write(raw)
        for t in tensors.values():
            data = t.detach().to("cpu").contiguous()
            out.write(data.reshape(-1).view(torch.uint8).numpy().tobytes() if data.numel() else b"")


def write_checkpoint(loaded: LoadedCheckpoint, directory: str | PathLike[str], *, shard_bytes: int | None = None,
                     store_lm_head: bool = False) -> Path:
    """Write `loaded` as a Transformers-style checkpoint directory (config.json, and
    model.safetensors or shards named by model.safetensors.index.json when shard_bytes is set);
    for synthetic models, tests and other engines' benchmarks. store_lm_head also stores the
    head (as lm_head.weight)."""
    root = Path(directory)
    root.mkdir(parents=True, exist_ok=True)
    c, w = loaded.config, loaded.weights
    (root / "config.json").write_text(json.dumps(config_document(c), indent=1), encoding="utf-8")
    tensors = {EMBED_TOKENS: w.embed_tokens}
    for index, layer in enumerate(w.layers):
        for field, suffix in LAYER_TENSORS.items():
            tensors[f"model.layers.{index}.{suffix}"] = getattr(layer, field)
    tensors[FINAL_NORM] = w.norm
    if store_lm_head:
        tensors[LM_HEAD] = w.lm_head
    if shard_bytes is None:
        _write_file(root / SINGLE_FILE, tensors)
        return root
    shards: list[dict[str, torch.Tensor]] = [{}]
    size = 0
    for name, t in tensors.items():
        nbytes = t.numel() * t.element_size()
        if shards[-1] and size + nbytes > shard_bytes:
            shards.append({})
            size = 0
        shards[-1][name] = t
        size += nbytes
    weight_map = {}
    for k, shard in enumerate(shards):
        file = f"model-{k + 1:05d}-of-{len(shards):05d}.safetensors"
        _write_file(root / file, shard)
        weight_map.update({name: file for name in shard})
    (root / INDEX_FILE).write_text(json.dumps({"metadata": {}, "weight_map": weight_map}, indent=1), encoding="utf-8")
    return root
