"""The tensor-parallel engine on 2 (and, where the box has them, 4 and 8) GPUs in its three step modes (the one-kernel step with its
exchanges inside, per-operator kernels with the peer-memory all-reduce, and with NCCL) against the
single-GPU engine: teacher-forced logits within a few bf16 ulps (the same math; fp32 partial sums
added in another order) and the same greedy tokens on every rank. Each world size is skipped on a
box with fewer GPUs."""

import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cases import build, to_device

pytestmark = pytest.mark.gpu
MODES = ("fused", "nvlink", "nccl")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    engine = None
    try:
        from ipe_b200.engine import Engine
        from ipe_b200.tp import TensorParallelEngine
        from oracle import qwen3 as oq

        gpu = to_device(build("qwen3-1.7b-2layer"), f"cuda:{rank}")
        ids = torch.randint(0, gpu.config.vocab_size, (2, 70), generator=torch.Generator().manual_seed(21))
        result = {}
        for mode in MODES:
            engine = TensorParallelEngine(gpu, batch=2, capacity=96, allreduce=mode)
            result[f"tp_logits_{mode}"] = oq.teacher_forced(engine, ids, 64).cpu()
            result[f"tokens_{mode}"], result[f"logprobs_{mode}"] = engine.generate(ids[:, :40], 12)
            engine.close()
            engine = None
        from ipe_b200 import _native as nat
        result["device_error"] = nat.device_error()
        if rank == 0:
            single = Engine(gpu, batch=2, capacity=96)
            result["logits"] = oq.teacher_forced(single, ids, 64).cpu()
            out = single.generate(ids[:, :40], 12)
            result["ref_tokens"], result["ref_logprobs"] = out.tokens, out.logprobs
        torch.save(result, os.path.join(out_dir, f"rank{rank}.pt"))
    finally:
        if engine is not None:  # an exception left it open: release the captured NCCL work first
            engine._graph = None
        torch.cuda.synchronize()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tensor_parallel_engine_matches_the_single_gpu_engine(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    ranks = [torch.load(tmp_path / f"rank{r}.pt") for r in range(world)]
    r0 = ranks[0]
    ref = r0["logits"]
    for r in ranks:
        assert r["device_error"] == 0
        for mode in MODES:
            assert ((r[f"tp_logits_{mode}"] - ref).abs() <= 4 * 2 ** -8 * ref.abs() + 0.05).all()
            assert torch.equal(r[f"tokens_{mode}"], r0[f"tokens_{mode}"])  # every rank samples the same tokens
        if world == 2:  # two addends sum to the same bits in either order: the peer-memory all-reduce
            assert torch.equal(r["tp_logits_nvlink"], r["tp_logits_nccl"])  # equals NCCL's (not so for more)
    for mode in MODES:
        agree = (r0[f"tokens_{mode}"] == r0["ref_tokens"]).float().mean()
        assert agree > 0.9, (mode, r0[f"tokens_{mode}"], r0["ref_tokens"])
        assert torch.allclose(r0[f"logprobs_{mode}"][:, :1], r0["ref_logprobs"][:, :1], atol=0.05)
