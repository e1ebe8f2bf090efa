"""Host logic of the tensor-parallel split (ipe_b200.tp), on the CPU: the shard plan partitions
heads, intermediate columns and the vocabulary exactly, the shards reassemble the weights, and
over a 2-rank gloo group the ranks' partial products of a row-parallel layer sum to the unsplit
product (the all-reduce step of the decode and prefill layers)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cases import build
from ipe_b200.config import QWEN3_1_7B
from ipe_b200.tp import interleave_gate_up, shard_layer, shard_plan


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_the_plan_partitions_heads_columns_and_vocabulary(world):
    c = QWEN3_1_7B
    plans = [shard_plan(c, r, world) for r in range(world)]
    assert [p.q0 for p in plans] == [r * c.num_attention_heads // world for r in range(world)]
    assert sum(p.q_heads for p in plans) == c.num_attention_heads
    assert sum(p.kv_heads for p in plans) == c.num_key_value_heads
    assert all(p.q_heads == p.kv_heads * (c.num_attention_heads // c.num_key_value_heads) for p in plans)
    assert sum(p.inter for p in plans) == c.intermediate_size
    offset = 0
    for p in plans:
        assert p.vocab_offset == offset and p.vocab_offset % 32 == 0 and p.vocab_rows > 0
        assert p.parts == (p.vocab_rows + 31) // 32 <= p.parts_max
        offset += p.vocab_rows
    assert offset == c.vocab_size
    assert max(p.vocab_rows for p in plans) - min(p.vocab_rows for p in plans) <= 32


def test_a_model_that_does_not_split_is_rejected():
    with pytest.raises(ValueError, match="KV heads"):
        shard_plan(QWEN3_1_7B, 0, 3)


def test_the_shards_reassemble_the_weights():
    loaded = build("qwen3-1.7b-2layer")
    layer = loaded.weights.layers[0]
    c = loaded.config
    world = 4
    shards = [shard_layer(layer, shard_plan(c, r, world)) for r in range(world)]
    hd, hq, hkv = 128, c.num_attention_heads // world, c.num_key_value_heads // world
    q = torch.cat([s["w_qkv"][:hq * hd] for s in shards])
    k = torch.cat([s["w_qkv"][hq * hd:(hq + hkv) * hd] for s in shards])
    v = torch.cat([s["w_qkv"][(hq + hkv) * hd:] for s in shards])
    assert torch.equal(q, layer.q_proj) and torch.equal(k, layer.k_proj) and torch.equal(v, layer.v_proj)
    assert torch.equal(torch.cat([s["w_o"] for s in shards], 1), layer.o_proj)
    assert torch.equal(torch.cat([s["gate"] for s in shards]), layer.gate_proj)
    assert torch.equal(torch.cat([s["w_down"] for s in shards], 1), layer.down_proj)
    g = interleave_gate_up(shards[1]["gate"], shards[1]["up"])
    assert torch.equal(g[:64], shards[1]["gate"][:64]) and torch.equal(g[64:128], shards[1]["up"][:64])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _row_parallel_worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        loaded = build("qwen3-1.7b-2layer")
        c, layer = loaded.config, loaded.weights.layers[0]
        plan = shard_plan(c, rank, world)
        shard = shard_layer(layer, plan)
        g = torch.Generator().manual_seed(5)
        attn = torch.randn((3, c.num_attention_heads * 128), generator=g)
        act = torch.randn((3, c.intermediate_size), generator=g)
        mine_o = attn[:, plan.q0 * 128:(plan.q0 + plan.q_heads) * 128]
        mine_a = act[:, plan.i0:plan.i0 + plan.inter]
        part_o = mine_o @ shard["w_o"].float().T
        part_d = mine_a @ shard["w_down"].float().T
        dist.all_reduce(part_o)
        dist.all_reduce(part_d)
        if rank == 0:
            torch.save({"o": part_o, "d": part_d, "o_ref": attn @ layer.o_proj.float().T,
                        "d_ref": act @ layer.down_proj.float().T}, os.path.join(out_dir, "result.pt"))
    finally:
        dist.destroy_process_group()


def test_partial_products_summed_over_ranks_equal_the_unsplit_layer(tmp_path):
    world = 2
    mp.spawn(_row_parallel_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    r = torch.load(tmp_path / "result.pt")
    for key in ("o", "d"):
        ref = r[f"{key}_ref"]
        assert torch.allclose(r[key], ref, rtol=1e-4, atol=1e-4 * ref.abs().max().item())
