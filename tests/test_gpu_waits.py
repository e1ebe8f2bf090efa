"""Bounded device-side waits, made to run out without any fault.

Every spin-wait of the one-kernel decode step (grid barriers, shared-memory copies, a peer's parts
in a tensor-parallel step) gives up after `wait_limit_ns`, sets device error 3 and leaves the step
without sampling or advancing the position (src/ipe/engine.py:96-101: a failed step commits
nothing). Two ways to make a wait run out, neither touching memory outside its buffers:

- one GPU: rank 0 of a two-rank tensor-parallel step whose second rank's region is a local buffer
  that nothing writes. Rank 0 pushes its parts into both regions, then polls its own region for the
  peer's parts, which never come.
- two GPUs: rank 1 runs the prefill's collectives and then stops launching decode steps; rank 0's
  `generate` raises with only the prompt committed.
"""

import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cases import build, to_device
from ipe_b200 import _native as nat

pytestmark = pytest.mark.gpu
LIMIT_NS = 20_000_000  # 20 ms


def silent_peer_step(gpu, capacity=64, position=10, limit_ns=LIMIT_NS):
    """Rank 0 of a two-rank step over local buffers; returns (desc, buffers that must stay alive)."""
    import ctypes

    from ipe_b200.model import decode_tiles
    from ipe_b200.tp import HEAD_DIM, _Layer, shard_plan

    c, w, dev = gpu.config, gpu.weights, gpu.weights.embed_tokens.device
    plan = shard_plan(c, 0, 2)
    lib = nat.load()
    keep = {"layers": [_Layer(layer, plan) for layer in w.layers],
            "t_lm": decode_tiles(w.lm_head[plan.vocab_offset:plan.vocab_offset + plan.vocab_rows].contiguous())}
    shape = (c.num_hidden_layers, 1, plan.kv_heads, capacity, HEAD_DIM)
    keep["k"] = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
    keep["v"] = torch.zeros(shape, dtype=torch.bfloat16, device=dev)
    rows = [torch.zeros((1, n), dtype=torch.bfloat16, device=dev) for n in (
        c.hidden_size, c.hidden_size, (plan.q_heads + 2 * plan.kv_heads) * HEAD_DIM, plan.q_heads * HEAD_DIM,
        plan.inter)]
    keep["x"], keep["x_alt"], keep["qkv"], keep["attn"], keep["act"] = rows
    keep["logits"] = torch.zeros((1, plan.vocab_rows), dtype=torch.float32, device=dev)
    keep["partials"] = torch.zeros(plan.parts_max * nat.PARTIAL_WORDS, dtype=torch.float32, device=dev)
    keep["state"] = torch.zeros(nat.STATE_WORDS, dtype=torch.int64, device=dev)
    keep["state"][nat.STATE_POS] = position
    keep["tokens"] = torch.tensor([5], dtype=torch.int64, device=dev)
    keep["cos"] = torch.ones((capacity, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    keep["sin"] = torch.zeros((capacity, HEAD_DIM), dtype=torch.bfloat16, device=dev)
    keep["ws"] = torch.zeros(int(lib.ipe_decode_step_workspace(1, plan.q_heads, plan.kv_heads, capacity)),
                             dtype=torch.uint8, device=dev)
    region = int(lib.ipe_decode_step_comm_bytes(2, 1, c.hidden_size))
    keep["regions"] = [torch.zeros(region, dtype=torch.uint8, device=dev) for _ in range(2)]
    keep["table"] = torch.tensor([r.data_ptr() for r in keep["regions"]], dtype=torch.int64, device=dev)
    descs = (nat.LayerDesc * c.num_hidden_layers)()
    for i, layer in enumerate(keep["layers"]):
        descs[i] = nat.LayerDesc(*(t.data_ptr() for t in (layer.in_norm, layer.post_norm, layer.q_norm, layer.k_norm,
                                                          layer.t_qkv, layer.t_o, layer.t_gate_up, layer.t_down,
                                                          keep["k"][i], keep["v"][i])))
    keep["descs"] = torch.frombuffer(bytearray(ctypes.string_at(ctypes.addressof(descs), ctypes.sizeof(descs))),
                                     dtype=torch.uint8).to(dev)
    d = nat.StepDesc()
    d.layers, d.hidden, d.intermediate = c.num_hidden_layers, c.hidden_size, plan.inter
    d.q_heads, d.kv_heads, d.vocab, d.capacity, d.batch = plan.q_heads, plan.kv_heads, plan.vocab_rows, capacity, 1
    d.eps = c.rms_norm_eps
    d.layer_descs = keep["descs"].data_ptr()
    d.embed, d.lm_head_tiles, d.final_norm = w.embed_tokens.data_ptr(), keep["t_lm"].data_ptr(), w.norm.data_ptr()
    d.cos_table, d.sin_table = keep["cos"].data_ptr(), keep["sin"].data_ptr()
    d.state, d.tokens = keep["state"].data_ptr(), keep["tokens"].data_ptr()
    d.x, d.qkv, d.attn, d.act = (keep[n].data_ptr() for n in ("x", "qkv", "attn", "act"))
    d.logits, d.partials = keep["logits"].data_ptr(), keep["partials"].data_ptr()
    d.workspace, d.workspace_bytes = keep["ws"].data_ptr(), keep["ws"].numel()
    d.tp_world, d.tp_rank, d.tp_peers = 2, 0, keep["table"].data_ptr()
    d.x_alt, d.vocab_offset, d.vocab_total = keep["x_alt"].data_ptr(), plan.vocab_offset, c.vocab_size
    d.wait_limit_ns = limit_ns
    return d, keep


def test_a_wait_for_a_silent_peer_runs_out_and_commits_nothing():
    import ctypes

    gpu = to_device(build("qwen3-1.7b-2layer"), "cuda")
    desc, keep = silent_peer_step(gpu)
    nat.device_error(reset=True)
    torch.cuda.synchronize()
    start = time.perf_counter()
    nat.call("ipe_decode_step", ctypes.addressof(desc), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()  # the kernel returns: every CTA left after the wait ran out
    elapsed = time.perf_counter() - start
    assert nat.device_error(reset=True) == 3
    assert LIMIT_NS / 1e9 <= elapsed < 1.5, elapsed  # gave up after the launch's limit, not the 2 s default
    assert int(keep["state"][nat.STATE_POS]) == 10  # the position did not advance
    words = keep["ws"][:8].view(torch.int32)
    assert int(words[1]) == 1  # the abort flag every CTA saw
    # the context is still usable: a normal one-GPU step runs afterwards
    from ipe_b200.engine import Engine

    engine = Engine(gpu, batch=1, capacity=32)
    out = engine.generate(torch.randint(0, gpu.config.vocab_size, (1, 8)), 3)
    assert out.tokens.shape == (1, 3) and nat.device_error(reset=True) == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, port: int, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    engine = None
    result = {}
    try:
        from ipe_b200.tp import TensorParallelEngine

        gpu = to_device(build("qwen3-1.7b-2layer"), f"cuda:{rank}")
        ids = torch.randint(0, gpu.config.vocab_size, (1, 24), generator=torch.Generator().manual_seed(4))
        engine = TensorParallelEngine(gpu, batch=1, capacity=64, wait_limit_s=LIMIT_NS / 1e9)
        if rank == 0:
            try:
                engine.generate(ids, 3)
                result["raised"] = None
            except RuntimeError as error:
                result["raised"] = str(error)
            result["length"] = engine.length
            try:
                engine.generate(ids, 2)
            except RuntimeError as error:
                result["again"] = str(error)
        else:
            # the same collective steps as rank 0's generate up to its first decode step, then none
            stream = torch.cuda.current_stream().cuda_stream
            engine._set_batch(1)
            engine._run_prefill(ids, 1, ids.shape[1])
            engine._sample(stream)
            torch.cuda.synchronize()
        dist.barrier()
        engine.close()
        engine = None
        torch.save(result, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        if engine is not None:
            engine._graph = None
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_a_rank_that_stops_makes_its_peer_raise_with_the_prompt_committed(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.spawn(_worker, args=(_free_port(), str(tmp_path)), nprocs=2, join=True)
    r0 = torch.load(tmp_path / "rank0.pt")
    assert r0["raised"] is not None and "error 3" in r0["raised"], r0
    assert r0["length"] == 24  # the prompt, and no decode step, is committed
    assert "earlier step failed" in r0["again"]
