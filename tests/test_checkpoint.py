"""Checkpoint directories on the CPU: the safetensors header reader and writer against the
`safetensors` package, the inventory and mapping rules (src/ipe/checkpoint.py:131-217), the tie
rule and dtype handling of load_checkpoint (src/ipe/weights.py:113-168), and its errors."""

import json
import struct

import pytest
import torch
from safetensors import safe_open
from safetensors.torch import load_file, save_file

from ipe_b200.checkpoint import (INDEX_FILE, LM_HEAD, SINGLE_FILE, CheckpointError, ConfigError, config_document,
                                 expected_tensors, inspect_checkpoint, read_config, read_header, write_checkpoint)
from ipe_b200.config import Qwen3Config
from ipe_b200.synthetic import random_model
from ipe_b200.weights import LAYER_FIELDS, load_checkpoint

TINY = Qwen3Config(vocab_size=320, hidden_size=256, intermediate_size=384, num_hidden_layers=2, num_attention_heads=4,
                   num_key_value_heads=2, head_dim=128, max_position_embeddings=512, rms_norm_eps=1e-6,
                   rope_theta=1e6)


@pytest.fixture(scope="module")
def tiny():
    return random_model(TINY, seed=3, norm_jitter=0.1)


def _same_weights(a, b):
    wa, wb = a.weights, b.weights
    assert torch.equal(wa.embed_tokens, wb.embed_tokens) and torch.equal(wa.norm, wb.norm)
    assert torch.equal(wa.lm_head, wb.lm_head)
    for la, lb in zip(wa.layers, wb.layers, strict=True):
        for field in LAYER_FIELDS:
            x, y = getattr(la, field), getattr(lb, field)
            assert x.dtype == y.dtype and torch.equal(x.cpu(), y.cpu()), field


def test_single_file_round_trip(tiny, tmp_path):
    write_checkpoint(tiny, tmp_path)
    loaded = load_checkpoint(tmp_path, dtype=torch.bfloat16, device="cpu")
    assert loaded.config == TINY
    _same_weights(loaded, tiny)
    assert loaded.weights.lm_head is loaded.weights.embed_tokens
    assert (loaded.tie.stored, loaded.tie.tied, loaded.tie.max_abs_diff) == (False, True, None)


def test_sharded_round_trip(tiny, tmp_path):
    write_checkpoint(tiny, tmp_path, shard_bytes=300_000)
    index = json.loads((tmp_path / INDEX_FILE).read_text())
    assert len(set(index["weight_map"].values())) > 2
    _same_weights(load_checkpoint(tmp_path, dtype=torch.bfloat16, device="cpu"), tiny)


def test_writer_and_reader_agree_with_the_safetensors_package(tiny, tmp_path):
    write_checkpoint(tiny, tmp_path)
    theirs = load_file(str(tmp_path / SINGLE_FILE))
    assert torch.equal(theirs["model.embed_tokens.weight"], tiny.weights.embed_tokens)
    assert torch.equal(theirs["model.layers.1.mlp.down_proj.weight"], tiny.weights.layers[1].down_proj)
    # their writer, our reader: offsets and shapes from our header parser
    tensors = {"a": torch.randn(3, 5).to(torch.bfloat16), "b": torch.arange(7, dtype=torch.float32),
               "c": torch.randn(2, 2, 2, dtype=torch.float64)}
    save_file(tensors, str(tmp_path / "other.safetensors"), metadata={"format": "pt"})
    info = read_header(tmp_path / "other.safetensors")
    raw = (tmp_path / "other.safetensors").read_bytes()
    dtypes = {"BF16": torch.bfloat16, "F32": torch.float32, "F64": torch.float64}
    with safe_open(str(tmp_path / "other.safetensors"), framework="pt") as handle:
        for name, t in tensors.items():
            assert info[name].shape == tuple(handle.get_slice(name).get_shape())
            assert info[name].dtype == handle.get_slice(name).get_dtype()
            got = torch.frombuffer(bytearray(raw[info[name].offset:info[name].offset + info[name].nbytes]),
                                   dtype=dtypes[info[name].dtype]).view(info[name].shape)
            assert torch.equal(got, t)


def test_stored_heads_and_the_tie_rule(tiny, tmp_path):
    write_checkpoint(tiny, tmp_path / "equal", store_lm_head=True)
    equal = load_checkpoint(tmp_path / "equal", dtype=torch.bfloat16, device="cpu")
    assert (equal.tie.stored, equal.tie.tied, equal.tie.max_abs_diff) == (True, True, 0.0)
    assert equal.weights.lm_head is equal.weights.embed_tokens
    head = tiny.weights.embed_tokens.clone()
    head[5, 7] += 0.25
    w = tiny.weights
    untied = type(tiny)(tiny.config, type(w)(w.embed_tokens, w.layers, w.norm, head), tiny.tie)
    write_checkpoint(untied, tmp_path / "differ", store_lm_head=True)
    differ = load_checkpoint(tmp_path / "differ", dtype=torch.bfloat16, device="cpu")
    assert differ.tie.stored and not differ.tie.tied
    assert differ.tie.max_abs_diff == pytest.approx(abs(head[5, 7].float() - w.embed_tokens[5, 7].float()).item())
    assert differ.weights.lm_head is not differ.weights.embed_tokens
    assert torch.equal(differ.weights.lm_head, head)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_wider_dtypes_are_exact_casts(tiny, tmp_path, dtype):
    write_checkpoint(tiny, tmp_path)
    loaded = load_checkpoint(tmp_path, dtype=dtype, device="cpu")
    assert loaded.weights.layers[0].q_proj.dtype == dtype
    assert torch.equal(loaded.weights.layers[0].q_proj, tiny.weights.layers[0].q_proj.to(dtype))
    assert loaded.weights.lm_head is loaded.weights.embed_tokens


def test_config_document_round_trips():
    import tempfile
    from pathlib import Path

    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "config.json"
        path.write_text(json.dumps(config_document(TINY)))
        assert read_config(path) == TINY
        for change in ({"tie_word_embeddings": False}, {"model_type": "llama"}, {"hidden_act": "gelu"},
                       {"rope_scaling": {"rope_type": "yarn", "factor": 4.0}}, {"rope_theta": -1},
                       {"num_key_value_heads": 3}, {"attention_bias": True}):
            path.write_text(json.dumps({**config_document(TINY), **change}))
            with pytest.raises(ConfigError):
                read_config(path)
        document = config_document(TINY)
        del document["rope_theta"]
        document["rope_parameters"] = {"rope_type": "default", "rope_theta": 5e5}
        path.write_text(json.dumps(document))
        assert read_config(path).rope_theta == 5e5


def _rewrite_single(tmp_path, tiny, edit):
    """Write the tiny model, then rewrite model.safetensors with its tensors dict edited."""
    write_checkpoint(tiny, tmp_path)
    tensors = load_file(str(tmp_path / SINGLE_FILE))
    edit(tensors)
    save_file(tensors, str(tmp_path / SINGLE_FILE))


@pytest.mark.parametrize("edit, words", [
    (lambda t: t.pop("model.layers.1.mlp.up_proj.weight"), "1 missing"),
    (lambda t: t.update({"model.layers.0.extra.weight": torch.zeros(2, dtype=torch.bfloat16)}), "1 unexpected"),
    (lambda t: t.update({"model.norm.weight": t["model.norm.weight"].float()}), "1 mismatched"),
    (lambda t: t.update({"model.layers.0.self_attn.q_norm.weight": torch.ones(64, dtype=torch.bfloat16)}),
     "1 mismatched"),
    (lambda t: t.update({LM_HEAD: torch.zeros(10, 256, dtype=torch.bfloat16)}), "1 mismatched"),
])
def test_mapping_errors(tiny, tmp_path, edit, words):
    _rewrite_single(tmp_path, tiny, edit)
    with pytest.raises(CheckpointError, match=words):
        load_checkpoint(tmp_path, dtype=torch.bfloat16, device="cpu")


def test_directory_layout_errors(tiny, tmp_path):
    write_checkpoint(tiny, tmp_path / "both")
    (tmp_path / "both" / INDEX_FILE).write_text(json.dumps({"weight_map": {}}))
    with pytest.raises(CheckpointError, match="exactly one"):
        inspect_checkpoint(tmp_path / "both")
    write_checkpoint(tiny, tmp_path / "stray")
    save_file({"x": torch.zeros(1)}, str(tmp_path / "stray" / "other.safetensors"))
    with pytest.raises(CheckpointError, match="safetensors files"):
        inspect_checkpoint(tmp_path / "stray")
    write_checkpoint(tiny, tmp_path / "index", shard_bytes=300_000)
    index = json.loads((tmp_path / "index" / INDEX_FILE).read_text())
    index["weight_map"]["model.ghost.weight"] = next(iter(index["weight_map"].values()))
    (tmp_path / "index" / INDEX_FILE).write_text(json.dumps(index))
    with pytest.raises(CheckpointError, match="mapped or stored"):
        inspect_checkpoint(tmp_path / "index")
    (tmp_path / "index" / INDEX_FILE).write_text("{not json")
    with pytest.raises(CheckpointError, match="malformed"):
        inspect_checkpoint(tmp_path / "index")


def test_damaged_files(tiny, tmp_path):
    write_checkpoint(tiny, tmp_path)
    path = tmp_path / SINGLE_FILE
    raw = path.read_bytes()
    path.write_bytes(raw[:-10])  # truncated payload: the last tensor's range leaves the file
    with pytest.raises(CheckpointError, match="outside"):
        inspect_checkpoint(tmp_path)
    (length,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + length])
    first, second = list(header)[:2]
    header[second]["data_offsets"] = [header[first]["data_offsets"][0],
                                      header[first]["data_offsets"][0] + header[second]["data_offsets"][1]
                                      - header[second]["data_offsets"][0]]
    body = json.dumps(header).encode()
    path.write_bytes(struct.pack("<Q", len(body)) + body + raw[8 + length:])
    with pytest.raises(CheckpointError, match="overlap"):
        inspect_checkpoint(tmp_path)
    path.write_bytes(struct.pack("<Q", 1 << 40) + b"{}")
    with pytest.raises(CheckpointError, match="header length"):
        inspect_checkpoint(tmp_path)


def test_argument_errors(tiny, tmp_path):
    write_checkpoint(tiny, tmp_path)
    with pytest.raises(ValueError, match="dtype"):
        load_checkpoint(tmp_path, dtype=torch.float16, device="cpu")
    for device in ("mps", "cpu:1", "tpu", 3):
        with pytest.raises(ValueError):
            load_checkpoint(tmp_path, dtype=torch.bfloat16, device=device)
    if not torch.cuda.is_available():
        with pytest.raises(ValueError, match="not available"):
            load_checkpoint(tmp_path, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(OSError):
        load_checkpoint(tmp_path / "missing", dtype=torch.bfloat16, device="cpu")


def test_expected_tensors_cover_every_layer_field():
    names = expected_tensors(TINY)
    assert len(names) == 2 + TINY.num_hidden_layers * len(LAYER_FIELDS)
    assert names["model.layers.1.self_attn.k_proj.weight"] == (256, 256)


def test_native_reader_rejects_bad_ranges_and_missing_files(tiny, tmp_path):
    """ipe_read_to_device checks the file and every range before any CUDA call."""
    import ctypes

    from ipe_b200 import _native as nat

    write_checkpoint(tiny, tmp_path)
    lib = nat.load()
    paths = (ctypes.c_char_p * 1)(str(tmp_path / SINGLE_FILE).encode())
    missing = (ctypes.c_char_p * 1)(str(tmp_path / "none").encode())
    size = (tmp_path / SINGLE_FILE).stat().st_size
    file_of, offsets, sizes = (ctypes.c_int * 1)(0), (ctypes.c_uint64 * 1)(size - 4), (ctypes.c_uint64 * 1)(8)
    dsts = (ctypes.c_void_p * 1)(16)
    assert lib.ipe_read_to_device(1, paths, 1, file_of, offsets, sizes, dsts, 1 << 20, 2, None) == 1
    assert b"outside" in lib.ipe_last_error()
    assert lib.ipe_read_to_device(1, missing, 1, file_of, offsets, sizes, dsts, 1 << 20, 2, None) == 4
    assert b"cannot open" in lib.ipe_last_error()
    assert lib.ipe_read_to_device(1, paths, 0, None, None, None, None, 1 << 20, 2, None) == 0
    assert lib.ipe_read_to_device(1, paths, 1, file_of, offsets, sizes, dsts, 100, 2, None) == 1
    bad_file = (ctypes.c_int * 1)(1)
    assert lib.ipe_read_to_device(1, paths, 1, bad_file, offsets, sizes, dsts, 1 << 20, 2, None) == 1
    assert lib.ipe_read_to_device(1, paths, 1, file_of, offsets, sizes, dsts, 1 << 20, 0, None) == 1
