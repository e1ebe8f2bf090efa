"""load_checkpoint onto a CUDA device: payloads streamed from the files through pinned staging
buffers (ipe_read_to_device) equal the CPU load bit for bit, for one file and for shards, with a
staging buffer small enough that every tensor spans many chunks and both buffers are reused; and
an Engine built from the loaded checkpoint computes the same logits as one built from the
in-memory model."""

import pytest
import torch

from cases import to_device
from ipe_b200.checkpoint import write_checkpoint
from ipe_b200.config import Qwen3Config
from ipe_b200.engine import Engine
from ipe_b200.synthetic import random_model
from ipe_b200.weights import LAYER_FIELDS, load_checkpoint
from oracle.qwen3 import teacher_forced

pytestmark = pytest.mark.gpu

SMALL = Qwen3Config(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=2,
                    num_attention_heads=8, num_key_value_heads=4, head_dim=128, max_position_embeddings=4096,
                    rms_norm_eps=1e-6, rope_theta=1e6)


@pytest.fixture(scope="module")
def small():
    return random_model(SMALL, seed=5, norm_jitter=0.1)


def _assert_same(gpu, cpu):
    assert gpu.weights.embed_tokens.is_cuda
    assert torch.equal(gpu.weights.embed_tokens.cpu(), cpu.weights.embed_tokens)
    assert torch.equal(gpu.weights.norm.cpu(), cpu.weights.norm)
    for lg, lc in zip(gpu.weights.layers, cpu.weights.layers, strict=True):
        for field in LAYER_FIELDS:
            assert torch.equal(getattr(lg, field).cpu(), getattr(lc, field)), field


@pytest.mark.parametrize("shard_bytes, readers", [(None, 1), (None, 8), (700_000, 3)])
def test_cuda_load_equals_the_source(small, tmp_path, shard_bytes, readers):
    write_checkpoint(small, tmp_path, shard_bytes=shard_bytes)
    gpu = load_checkpoint(tmp_path, dtype=torch.bfloat16, device="cuda", staging_bytes=64 * 1024, readers=readers)
    _assert_same(gpu, small)
    assert gpu.weights.lm_head is gpu.weights.embed_tokens
    assert (gpu.tie.stored, gpu.tie.tied) == (False, True)


def test_cuda_load_of_a_stored_head_and_wider_dtypes(small, tmp_path):
    w = small.weights
    head = w.embed_tokens.clone()
    head[3, 3] = -head[3, 3] - 0.5
    untied = type(small)(small.config, type(w)(w.embed_tokens, w.layers, w.norm, head), small.tie)
    write_checkpoint(untied, tmp_path, store_lm_head=True)
    gpu = load_checkpoint(tmp_path, dtype=torch.float32, device="cuda:0", staging_bytes=8192)
    cpu = load_checkpoint(tmp_path, dtype=torch.float32, device="cpu")
    assert gpu.tie == cpu.tie and not gpu.tie.tied
    assert torch.equal(gpu.weights.lm_head.cpu(), head.float())
    assert torch.equal(gpu.weights.layers[1].down_proj.cpu(), w.layers[1].down_proj.float())


def test_engine_on_a_loaded_checkpoint_matches_the_in_memory_model(small, tmp_path):
    write_checkpoint(small, tmp_path)
    loaded = load_checkpoint(tmp_path, dtype=torch.bfloat16, device="cuda")
    ids = torch.randint(0, SMALL.vocab_size, (2, 40), generator=torch.Generator().manual_seed(8))
    a = teacher_forced(Engine(loaded, batch=2, capacity=48), ids, 32)
    b = teacher_forced(Engine(to_device(small, "cuda"), batch=2, capacity=48), ids, 32)
    assert torch.equal(a, b)
