"""Decode / prefill throughput of the Qwen3-1.7B-architecture engine on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload W1|W2-4|W2-16|W3] [--impl ours|reference]

A step is one generation of the workload on one GPU: prefill of B prompts of P random token IDs,
then N new tokens (N-1 decode steps), bf16, random-init weights (N(0, 0.02) matrices, unit norms).
`value` is decode tokens/s over all ranks (B * (N-1) tokens per step per rank, CUDA-event time of
the decode phase, max over ranks); prefill tokens/s is reported beside it. Under torchrun each rank
runs an independent replica on its own GPU (no collective on the data path; weak scaling).
`e2e` times the public `Engine.generate` call with host (pinned) prompt IDs and host results as
the reference harness does: decode tok/s = batch / TPOT, TPOT = (latency(N) - latency(1)) / (N - 1).

`--impl reference` times the reference algorithm's CPU implementation (the restated reference
engine in oracle/, bf16, all host threads) on a bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "inference-performance-engineering_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

import torch  # noqa: E402

WORKLOADS = {  # name: (batch, prompt, new tokens, capacity, temperature)
    "W1": (1, 512, 256, 1024, 0.0),
    "W2-4": (4, 512, 256, 1024, 0.7),
    "W2-16": (16, 512, 256, 1024, 0.7),
    "W3": (1, 4096, 128, 4352, 0.0),
}
METRIC = "decode tok/s & % HBM roofline, Qwen3-1.7B bf16 B=1/4/16; prefill tok/s"
REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during the timed region."""

    def __init__(self, index: int):
        self.index, self.samples, self._stop = index, [], threading.Event()
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self):
        query = "clocks.sm,clocks.max.sm," + ",".join(f"clocks_event_reasons.{r}" for r in REASONS)
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.index), f"--query-gpu={query}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                fields = [f.strip() for f in out.stdout.strip().split(",")]
                if len(fields) == 2 + len(REASONS):
                    self.samples.append(fields)
            except (OSError, subprocess.SubprocessError):
                return
            self._stop.wait(0.2)

    def __enter__(self):
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        mhz = [float(s[0]) for s in self.samples if s[0].replace(".", "").isdigit()]
        mx = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        reasons = sorted({REASONS[i] for s in self.samples for i, v in enumerate(s[2:]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def decode_bytes_per_step(config, batch: int, context: float) -> float:
    """Algorithmic HBM bytes of one decode step: every weight once (bf16) plus the KV cache read
    at the average context, plus the new K/V rows written."""
    c = config
    q, kv = c.num_attention_heads * c.head_dim, c.num_key_value_heads * c.head_dim
    per_layer = (q + 2 * kv) * c.hidden_size + q * c.hidden_size + 3 * c.intermediate_size * c.hidden_size
    weights = 2 * (c.num_hidden_layers * per_layer + c.vocab_size * c.hidden_size)
    kv_token = c.num_hidden_layers * 2 * kv * 2
    return weights + batch * kv_token * (context + 1)


# DRAM bytes of one decode_step_kernel launch measured by ncu (dram__bytes_read.sum +
# dram__bytes_write.sum) on the Qwen3-1.7B architecture at batch 1, cache position 514, with 1 and
# 2 decoder layers: the LM-head part and the per-layer part (captures summarised under profiles/).
NCU_STEP_LAYER_BYTES = (828.229888e6 + 4.516864e6) - (725.452544e6 + 5.074944e6)
NCU_STEP_FIXED_BYTES = 725.452544e6 + 5.074944e6 - NCU_STEP_LAYER_BYTES
NCU_STEP_POSITION = 514


def step_traffic(config, batch: int, position: int) -> float | None:
    """The captured traffic scaled to `layers` layers and `position` (K/V rows grow linearly);
    None where no capture applies (other batch sizes)."""
    if batch != 1 or config.hidden_size != 2048:
        return None
    kv_row = 2 * config.num_key_value_heads * config.head_dim * 2
    layer = NCU_STEP_LAYER_BYTES + kv_row * (position - NCU_STEP_POSITION)
    return NCU_STEP_FIXED_BYTES + config.num_hidden_layers * layer


def time_step_kernel(engine, batch: int, position: int, repeats: int = 10) -> dict:
    """Live CUDA-event timing of the dominant kernel, the one-kernel decode step (ipe_decode_step:
    every layer's weights, the KV cache up to `position` and the LM head in one launch), on the
    launching stream. The state's position is reset before each launch, so every launch does the
    same work; each launch streams 3.4 GB of weights, far above L2, so no flush is needed."""
    from ipe_b200 import _native as nat

    lib = nat.load()
    stream = torch.cuda.current_stream()
    state = engine._buf.state.data_ptr()
    events = []
    for _ in range(repeats + 2):
        nat.check(lib.ipe_state_set(state, nat.STATE_POS, position, stream.cuda_stream), "ipe_state_set")
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        engine._launch_step(batch, False, stream.cuda_stream)
        e1.record(stream)
        events.append((e0, e1))
    torch.cuda.synchronize()
    seconds = statistics.mean(a.elapsed_time(b) for a, b in events[2:]) / 1e3
    return {"kernel": "decode_step_kernel (ipe_decode_step)", "seconds": seconds,
            "bytes": decode_bytes_per_step(engine.loaded.config, batch, position), "position": position}


def time_prefill_kernels(engine, batch: int, prompt: int, repeats: int = 3) -> dict:
    """Live CUDA-event timing of one layer's prefill GEMMs (tcgen05: QKV, o_proj + residual,
    gate/up + SiLU, down_proj + residual) and causal attention at M = batch * prompt rows, cycling
    the layers' real weights. GEMM utilisation = 2*M*N*K / time against the measured bf16 peak."""
    from ipe_b200 import _native as nat

    c, m = engine.loaded.config, engine._model
    lib = nat.load()
    stream = torch.cuda.current_stream()
    rows = batch * prompt
    h, i, q_rows, qkv_rows = c.hidden_size, c.intermediate_size, m.q_rows, m.qkv_rows
    dev = m.device
    a_h = torch.randn((rows, h), device=dev).bfloat16()
    a_q = torch.randn((rows, q_rows), device=dev).bfloat16()
    a_i = torch.randn((rows, i), device=dev).bfloat16()
    out_qkv = torch.empty((rows, qkv_rows), dtype=torch.bfloat16, device=dev)
    out_h = torch.randn((rows, h), device=dev).bfloat16()
    out_i = torch.empty((rows, i), dtype=torch.bfloat16, device=dev)
    shapes = {"qkv": (qkv_rows, h), "o_proj": (h, q_rows), "gate_up": (2 * i, h), "down_proj": (h, i)}

    def launch(kind, layer):
        p = layer.ptr
        if kind == "qkv":
            args = (a_h.data_ptr(), p["w_qkv"], out_qkv.data_ptr(), rows, qkv_rows, h, nat.EPI_STORE, 0)
        elif kind == "o_proj":
            args = (a_q.data_ptr(), p["w_o"], out_h.data_ptr(), rows, h, q_rows, nat.EPI_RESIDUAL, out_h.data_ptr())
        elif kind == "gate_up":
            args = (a_h.data_ptr(), p["w_gate_up"], out_i.data_ptr(), rows, 2 * i, h, nat.EPI_SILU_MUL, 0)
        else:
            args = (a_i.data_ptr(), p["w_down"], out_h.data_ptr(), rows, h, i, nat.EPI_RESIDUAL, out_h.data_ptr())
        nat.check(lib.ipe_gemm(*args, stream.cuda_stream), "ipe_gemm")

    result, total_s, total_flops = {}, 0.0, 0.0
    for kind, (n, k) in shapes.items():
        launch(kind, m.layers[0])
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for r in range(repeats * len(m.layers)):
            launch(kind, m.layers[r % len(m.layers)])
        e1.record(stream)
        e1.synchronize()
        seconds = e0.elapsed_time(e1) / 1e3 / (repeats * len(m.layers))
        flops = 2.0 * rows * n * k
        result[kind] = {"us": round(seconds * 1e6, 2), "tflops": round(flops / seconds / 1e12, 1)}
        total_s += seconds
        total_flops += flops
    # causal attention of the prompt (one layer's cache)
    q = torch.randn((batch, c.num_attention_heads, prompt, 128), device=dev).bfloat16()
    out_a = torch.empty((batch, prompt, q_rows), dtype=torch.bfloat16, device=dev)
    kc, vc = engine._k[0], engine._v[0]

    def attn():
        nat.check(lib.ipe_prefill_attention(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), out_a.data_ptr(), batch,
                                            c.num_attention_heads, c.num_key_value_heads, prompt, engine.capacity,
                                            stream.cuda_stream), "ipe_prefill_attention")

    attn()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(repeats):
        attn()
    e1.record(stream)
    e1.synchronize()
    a_s = e0.elapsed_time(e1) / 1e3 / repeats
    a_flops = 2.0 * 128 * prompt * (prompt + 1) * c.num_attention_heads * batch  # QK^T and PV, causal half
    return {"rows": rows, "gemm": result, "gemm_tflops": round(total_flops / total_s / 1e12, 1),
            "attention": {"us": round(a_s * 1e6, 2), "tflops": round(a_flops / a_s / 1e12, 1)}}


def workload_config(workload: str, world: int, layers: int) -> dict:
    """The `config` of a bench line: the same dict for this engine's arm and the reference arm."""
    batch, prompt, new, capacity, temperature = WORKLOADS[workload]
    return {"workload": f"{workload}: Qwen3-1.7B arch bf16, batch {batch}, prompt {prompt}, {new} new tokens, "
                        f"capacity {capacity}, temperature {temperature}",
            "batch_per_gpu": batch, "prompt": prompt, "new_tokens": new, "capacity": capacity,
            "parallelism": f"dp{world} (independent replicas)", "layers": layers,
            "l2": "weights 3.44 GB per step > 126 MB L2 (no flush needed)"}


def run_ours(args, rank: int, world: int) -> dict | None:
    from ipe_b200 import Engine, QWEN3_1_7B
    from ipe_b200.synthetic import random_model

    batch, prompt, new, capacity, temperature = WORKLOADS[args.workload]
    new = args.new_tokens or new
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(device)
    config = QWEN3_1_7B if not args.layers else dataclasses.replace(QWEN3_1_7B, num_hidden_layers=args.layers)
    loaded = random_model(config, seed=0, device=device, generator_device=device)
    engine = Engine(loaded, batch=batch, capacity=capacity)
    ids_host = torch.randint(0, QWEN3_1_7B.vocab_size, (batch, prompt), generator=torch.Generator().manual_seed(0))
    ids_dev = ids_host.to(device)
    ids_pinned = ids_host.pin_memory()
    stream = torch.cuda.current_stream()

    def one_step(times):
        e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        e0.record(stream)
        engine._generate_on_device(ids_dev, new, temperature, 1234, after_prefill=lambda: e1.record(stream))
        e2.record(stream)
        times.append((e0, e1, e2))

    for _ in range(args.warmup):
        one_step([])
    torch.cuda.synchronize()
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    records = []
    with ClockSampler(device.index) as clocks:
        for _ in range(args.steps):
            one_step(records)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    prefill_s = sum(a.elapsed_time(b) for a, b, _ in records) / 1e3
    decode_s = sum(b.elapsed_time(c) for _, b, c in records) / 1e3
    total_s = sum(a.elapsed_time(c) for a, _, c in records) / 1e3

    # e2e: the public API with host prompt IDs in pinned memory and host results, timed the way the
    # reference harness times engines (bench/run.py:250-274): latency(N) and latency(1) pairs,
    # TPOT = (median latency(N) - median latency(1)) / (N - 1), decode tok/s = batch / TPOT
    def e2e_latency(n_new: int) -> float:
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        out = engine.generate(ids_pinned, n_new, temperature=temperature, seed=1234)
        e.record(stream)
        e.synchronize()
        assert out.tokens.shape == (batch, n_new)
        return s.elapsed_time(e) / 1e3

    e2e_full, e2e_first = [], []
    for _ in range(max(3, min(args.steps, 5))):
        e2e_full.append(e2e_latency(new))
        e2e_first.append(e2e_latency(1))
    e2e_n, e2e_1 = statistics.median(e2e_full), statistics.median(e2e_first)

    kernel = time_step_kernel(engine, batch, prompt + new // 2)
    prefill_kernels = time_prefill_kernels(engine, batch, prompt)
    if world > 1:
        t = torch.tensor([prefill_s, decode_s, total_s, e2e_n, e2e_1, kernel["seconds"]], dtype=torch.float64,
                         device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        prefill_s, decode_s, total_s, e2e_n, e2e_1, kernel["seconds"] = t.tolist()
    if rank != 0:
        return None

    pk = peaks()
    steps = args.steps
    decode_tokens = world * batch * (new - 1) * steps
    value = decode_tokens / decode_s
    context = prompt + (new - 1) / 2
    step_bytes = decode_bytes_per_step(config, batch, context)
    decode_gbs = step_bytes * (new - 1) * steps / decode_s / 1e9  # per GPU
    achieved = kernel["bytes"] / kernel["seconds"] / 1e9
    launches = engine.kernel_launches(prompt, new)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "decode tok/s", "n_gpus": world, "steps": steps,
        "warmup": args.warmup, "ms_per_step": round(total_s / steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) weights, uniform random prompt IDs)",
        "config": workload_config(args.workload, world, config.num_hidden_layers),
        "prefill_tok_s": round(world * batch * prompt * steps / prefill_s, 1),
        "prefill_kernels": dict(prefill_kernels, gemm_frac=round(prefill_kernels["gemm_tflops"] / pk["bf16_tflops"], 4),
                                peak_tflops=pk["bf16_tflops"]),
        "decode_ms_per_token": round(decode_s / ((new - 1) * steps) * 1e3, 4),
        "decode_hbm": {"bytes_per_step": step_bytes, "achieved_gbs": round(decode_gbs, 1), "peak_gbs": pk["hbm_gbs"],
                       "frac": round(decode_gbs / pk["hbm_gbs"], 4), "peak_source": pk["source"]},
        "roofline": {"kernel": kernel["kernel"], "bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / pk["hbm_gbs"], 4),
                     "traffic": step_traffic(config, batch, kernel["position"]),
                     "traffic_source": "ncu dram bytes at 1 and 2 layers, scaled to the layers and position",
                     "bytes_per_launch": kernel["bytes"], "seconds_per_launch": kernel["seconds"],
                     "position": kernel["position"], "peak_source": pk["source"]},
        "e2e": {"value": round(world * batch * (new - 1) / (e2e_n - e2e_1), 2), "unit": "decode tok/s",
                "definition": "Engine.generate(pinned host prompt IDs) -> host Generation, CUDA events around "
                              "each call; TPOT = (median latency(N) - median latency(1)) / (N - 1) over "
                              f"{len(e2e_full)} pairs; value = ranks * batch / TPOT",
                "latency_n_ms": round(e2e_n * 1e3, 3), "latency_1_ms": round(e2e_1 * 1e3, 3),
                "generated_tok_s": round(world * batch * new / e2e_n, 2),
                "h2d_bytes_per_step": batch * prompt * 8, "d2h_bytes_per_step": batch * new * 12 + batch * 8},
        "gpu_launches": launches["generate"] * steps,
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload, samples=args.cpu_decode_steps)
    return line


def run_tp(args, rank: int, world: int) -> dict | None:
    """The tensor-parallel latency case (B=1): the model split over `world` GPUs
    (ipe_b200.tp.TensorParallelEngine; by default the one-kernel step with the exchanges over NVLink
    peer memory inside it), decode tok/s of the W1 generation, device time max over ranks."""
    import torch.distributed as dist

    from ipe_b200 import QWEN3_1_7B
    from ipe_b200.synthetic import random_model
    from ipe_b200.tp import TensorParallelEngine

    batch, prompt, new, capacity, _ = WORKLOADS["W1"]
    new = args.new_tokens or new
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    loaded = random_model(QWEN3_1_7B, seed=0, device=device, generator_device=device)
    engine = TensorParallelEngine(loaded, batch=batch, capacity=capacity, allreduce=args.tp_allreduce)
    ids = torch.randint(0, QWEN3_1_7B.vocab_size, (batch, prompt), generator=torch.Generator().manual_seed(0))
    stream = torch.cuda.current_stream()

    def timed(n_new: int) -> float:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        engine.generate(ids, n_new)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3

    for _ in range(args.warmup):
        timed(new)
    with ClockSampler(device.index) as clocks:
        full = [timed(new) for _ in range(args.steps)]
        first = [timed(1) for _ in range(args.steps)]
    exchange_us = 0.0
    if args.tp_allreduce == "fused":  # one traced step: the staging that waits on the peers' parts
        from ipe_b200 import _native as nat
        from ipe_b200.steptrace import exchange_stage_us, traced_step

        dist.barrier()
        raw = traced_step(engine._step_desc(True), nat.load().ipe_decode_step_grid(), QWEN3_1_7B.num_hidden_layers,
                          stream.cuda_stream, device)
        exchange_us = exchange_stage_us(raw, QWEN3_1_7B.num_hidden_layers)
    t = torch.tensor([sum(full), sum(first), exchange_us], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    engine.close()
    if rank != 0:
        return None
    decode_s = (t[0] - t[1]).item()
    value = batch * (new - 1) * args.steps / decode_s
    return {"metric": "decode tok/s, Qwen3-1.7B bf16 B=1, tensor parallel", "value": round(value, 2),
            "unit": "decode tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(t[0].item() / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init N(0,0.02) weights)",
            "config": {"workload": f"W1 tensor parallel: batch {batch}, prompt {prompt}, {new} new tokens",
                       "parallelism": f"tp{world}", "allreduce": args.tp_allreduce},
            "decode_ms_per_token": round(decode_s / ((new - 1) * args.steps) * 1e3, 4),
            "exchange_stage_us_per_step": round(t[2].item(), 1) if args.tp_allreduce == "fused" else None,
            "clocks": clocks.summary()}


def run_load(args) -> dict:
    """Checkpoint loading onto the GPU (Qwen3-1.7B, random-init, bf16, written once to a temporary
    directory as two safetensors shards): ipe_b200.weights.load_checkpoint, which streams the
    payloads through pinned staging buffers into preallocated device tensors, against the
    reference's procedure restated (one safe_open per file, get_tensor, .to(dtype).to(device) per
    tensor, the tie check on the device). Wall clock from the call to a synchronized device; the
    files are in the page cache for both (each is read once untimed first)."""
    import shutil
    import tempfile

    from safetensors import safe_open

    from ipe_b200 import QWEN3_1_7B
    from ipe_b200.checkpoint import LM_HEAD, inspect_checkpoint, write_checkpoint
    from ipe_b200.synthetic import random_model
    from ipe_b200.weights import load_checkpoint

    device = torch.device("cuda", 0)
    model = random_model(QWEN3_1_7B, seed=0, device="cpu", generator_device=device)
    root = tempfile.mkdtemp(prefix="ipe_ckpt_")
    try:
        write_checkpoint(model, root, shard_bytes=2 * 1024**3)
        del model
        inventory = inspect_checkpoint(root)
        total = sum(info.nbytes for info in inventory.values())

        def ours():
            return load_checkpoint(root, dtype=torch.bfloat16, device=device)

        def restated():
            loaded = {}
            for file in sorted({info.file for info in inventory.values()}):
                with safe_open(f"{root}/{file}", framework="pt", device="cpu") as handle:
                    for name, info in inventory.items():
                        if info.file == file:
                            loaded[name] = handle.get_tensor(name).to(torch.bfloat16).to(device)
            if LM_HEAD in loaded:
                torch.equal(loaded["model.embed_tokens.weight"], loaded[LM_HEAD])
            return loaded

        def timed(fn):
            torch.cuda.synchronize()
            start = time.perf_counter()
            result = fn()
            torch.cuda.synchronize()
            elapsed = time.perf_counter() - start
            del result
            torch.cuda.empty_cache()
            return elapsed

        timed(restated)  # page cache warm for both
        ours_s = [timed(ours) for _ in range(max(1, args.steps))]
        ref_s = [timed(restated) for _ in range(max(1, args.steps))]
    finally:
        shutil.rmtree(root, ignore_errors=True)
    best, ref_best = min(ours_s), min(ref_s)
    return {"metric": "checkpoint load GB/s, Qwen3-1.7B bf16 safetensors -> GPU", "value": round(total / best / 1e9, 3),
            "unit": "GB/s", "n_gpus": 1, "steps": len(ours_s), "warmup": 1, "higher_is_better": True,
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init), 2 safetensors shards, page cache warm",
            "config": {"workload": f"load {total} bytes of Qwen3-1.7B weights to cuda:0"},
            "seconds": [round(t, 4) for t in ours_s],
            "reference_procedure": {"value": round(total / ref_best / 1e9, 3), "unit": "GB/s",
                                    "seconds": [round(t, 4) for t in ref_s],
                                    "what": "safe_open + get_tensor + .to(bf16).to(cuda) per tensor "
                                            "(src/ipe/weights.py:154-161)"}}


def run_compare(args) -> dict:
    """The reference harness's engine comparison (bench/run.py:96-144): the workload's greedy
    generation through each engine's own public API from one checkpoint directory (the random-init
    Qwen3-1.7B written once), host wall clock from the call to a synchronized device, and the
    harness's TPOT = (latency(N) - latency(1)) / (N - 1), prefill = latency(1). Engines: this one
    (load_checkpoint + Engine.generate), Transformers with a static cache (Qwen3ForCausalLM,
    sdpa, bf16), and vLLM (tokens in, no tokenizer, ignore_eos), each where it imports."""
    import gc
    import shutil
    import tempfile

    from ipe_b200 import QWEN3_1_7B
    from ipe_b200.checkpoint import write_checkpoint
    from ipe_b200.engine import Engine
    from ipe_b200.synthetic import random_model
    from ipe_b200.weights import load_checkpoint

    batch, prompt, new, capacity, _ = WORKLOADS[args.workload]
    device = torch.device("cuda", 0)
    root = tempfile.mkdtemp(prefix="ipe_compare_")
    ids = torch.randint(0, QWEN3_1_7B.vocab_size, (batch, prompt), generator=torch.Generator().manual_seed(0))
    engines = {}
    try:
        write_checkpoint(random_model(QWEN3_1_7B, seed=0, device="cpu", generator_device=device), root,
                         shard_bytes=2 * 1024**3)

        def measure(generate) -> dict:
            def latency(n):
                torch.cuda.synchronize()
                start = time.perf_counter()
                tokens = generate(n)
                torch.cuda.synchronize()
                elapsed = time.perf_counter() - start
                if tuple(tokens.shape) != (batch, n):
                    raise RuntimeError(f"expected {n} new tokens per row, got {tuple(tokens.shape)}")
                return elapsed, tokens

            for _ in range(max(1, args.warmup)):
                latency(new)
            full, first, tokens = [], [], None
            for _ in range(max(1, args.steps)):
                t, tokens = latency(new)
                full.append(t)
                first.append(latency(1)[0])
            tpot = (statistics.median(full) - statistics.median(first)) / (new - 1)
            return {"decode_tok_s": round(batch / tpot, 2), "tpot_ms": round(tpot * 1e3, 4),
                    "prefill_ms": round(statistics.median(first) * 1e3, 3),
                    "latency_s": [round(t, 4) for t in full], "first_tokens": tokens[0, :8].tolist()}

        engine = Engine(load_checkpoint(root, dtype=torch.bfloat16, device=device), batch=batch, capacity=capacity)
        engines["ipe_b200"] = measure(lambda n: engine.generate(ids, n).tokens)
        del engine
        gc.collect()
        torch.cuda.empty_cache()
        try:
            from transformers import GenerationConfig, Qwen3ForCausalLM

            model = Qwen3ForCausalLM.from_pretrained(root, dtype=torch.bfloat16, attn_implementation="sdpa")
            model = model.to(device).eval()
            model.generation_config.eos_token_id = None
            config = GenerationConfig(do_sample=False, eos_token_id=None, pad_token_id=0, cache_implementation="static")
            prompt_d, mask = ids.to(device), torch.ones_like(ids, device=device)

            def hf(n):
                with torch.no_grad():
                    out = model.generate(prompt_d, attention_mask=mask, generation_config=config, max_new_tokens=n)
                return out[:, prompt:].cpu()

            engines["transformers_static"] = measure(hf)
            del model
        except Exception as error:  # noqa: BLE001 - an engine that does not run is reported, not fatal
            engines["transformers_static"] = {"unavailable": f"{type(error).__name__}: {error}"[:300]}
        gc.collect()
        torch.cuda.empty_cache()
        try:
            from vllm import LLM, SamplingParams, TokensPrompt

            llm = LLM(model=root, dtype="bfloat16", enable_prefix_caching=False, seed=0, max_model_len=capacity,
                      max_num_seqs=batch, skip_tokenizer_init=True, gpu_memory_utilization=0.5)
            prompts = [TokensPrompt(prompt_token_ids=row.tolist()) for row in ids]

            def vllm_generate(n):
                params = SamplingParams(max_tokens=n, temperature=0.0, ignore_eos=True, detokenize=False)
                outputs = llm.generate(prompts, params, use_tqdm=False)
                return torch.tensor([list(o.outputs[0].token_ids) for o in outputs])

            engines["vllm"] = measure(vllm_generate)
            del llm
        except Exception as error:  # noqa: BLE001
            engines["vllm"] = {"unavailable": f"{type(error).__name__}: {error}"[:300]}
    finally:
        shutil.rmtree(root, ignore_errors=True)
    ours = engines["ipe_b200"]["decode_tok_s"]
    return {"metric": f"decode tok/s by TPOT (harness wall clock), Qwen3-1.7B bf16, {args.workload}", "value": ours,
            "unit": "decode tok/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init checkpoint written once)",
            "config": {"workload": f"{args.workload}: batch {batch}, prompt {prompt}, {new} new tokens, greedy"},
            "engines": engines}


def cpu_baseline(workload: str, samples: int) -> dict:
    """The reference engine's algorithm (oracle/ restatement, bf16, sdpa) on the host cores:
    one prefill of the workload's prompt, then `samples` decode steps (bounded sample)."""
    from ipe_b200 import QWEN3_1_7B
    from ipe_b200.synthetic import random_model
    from oracle import qwen3 as oq

    batch, prompt, _, capacity, _ = WORKLOADS[workload]
    torch.set_num_threads(os.cpu_count() or 1)
    loaded = random_model(QWEN3_1_7B, seed=0)
    ids = torch.randint(0, QWEN3_1_7B.vocab_size, (batch, prompt), generator=torch.Generator().manual_seed(0))
    engine = oq.CachedEngine(loaded, batch=batch, capacity=capacity, dtype=torch.bfloat16, backend="sdpa")
    with torch.no_grad():
        t0 = time.perf_counter()
        logits = engine.prefill(ids)
        t1 = time.perf_counter()
        tokens = logits.argmax(-1)
        logits = engine.decode(tokens)  # warm-up step
        tokens = logits.argmax(-1)
        t2 = time.perf_counter()
        for _ in range(samples):
            tokens = engine.decode(tokens).argmax(-1)
        t3 = time.perf_counter()
    return {"value": round(batch * samples / (t3 - t2), 3), "unit": "decode tok/s", "cores": torch.get_num_threads(),
            "kind": "port", "prefill_tok_s": round(batch * prompt / (t1 - t0), 2),
            "sample": f"{workload}: one {batch}x{prompt} prefill, then {samples} decode steps after one warm-up step"}


def run_reference(args, rank: int) -> dict | None:
    """The CPU reference arm: the restated reference engine on all host threads."""
    if rank != 0:
        return None
    from ipe_b200 import QWEN3_1_7B
    from ipe_b200.synthetic import random_model
    from oracle import qwen3 as oq

    batch, prompt, _, capacity, _ = WORKLOADS[args.workload]
    torch.set_num_threads(os.cpu_count() or 1)
    loaded = random_model(QWEN3_1_7B, seed=0)
    ids = torch.randint(0, QWEN3_1_7B.vocab_size, (batch, prompt), generator=torch.Generator().manual_seed(0))
    per_step = 2
    engine = oq.CachedEngine(loaded, batch=batch, capacity=capacity, dtype=torch.bfloat16, backend="sdpa")
    with torch.no_grad():
        t0 = time.perf_counter()
        tokens = engine.prefill(ids).argmax(-1)
        prefill_s = time.perf_counter() - t0
        for _ in range(args.warmup):
            for _ in range(per_step):
                tokens = engine.decode(tokens).argmax(-1)
        t1 = time.perf_counter()
        for _ in range(args.steps):
            for _ in range(per_step):
                tokens = engine.decode(tokens).argmax(-1)
        elapsed = time.perf_counter() - t1
    value = batch * per_step * args.steps / elapsed
    world = int(os.environ.get("WORLD_SIZE", 1))
    sample = (f"bounded CPU sample of the workload: one {batch}x{prompt} prefill, then {per_step} decode steps per "
              f"step on rank 0 only, every host thread")
    return {"metric": METRIC, "value": round(value, 3), "unit": "decode tok/s", "impl": "reference",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(elapsed / args.steps * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init N(0,0.02) weights, uniform random prompt IDs)",
            "config": workload_config(args.workload, world, QWEN3_1_7B.num_hidden_layers),
            "sample": sample,
            "prefill_tok_s": round(batch * prompt / prefill_s, 2),
            "cpu_baseline": {"value": round(value, 3), "unit": "decode tok/s", "cores": torch.get_num_threads(),
                             "kind": "port", "sample": sample},
            "e2e": {"value": round(value, 3), "unit": "decode tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--workload", default="W1", choices=sorted(WORKLOADS))
    parser.add_argument("--impl", default="ours", choices=("ours", "reference"))
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--cpu-decode-steps", type=int, default=8)
    parser.add_argument("--new-tokens", type=int, default=0, help="override the workload's new tokens (profiling)")
    parser.add_argument("--layers", type=int, default=0, help="fewer decoder layers (profiling only; not a bench line)")
    parser.add_argument("--tp", action="store_true", help="tensor-parallel B=1 latency mode over the launched ranks")
    parser.add_argument("--tp-allreduce", default="fused", choices=("fused", "nvlink", "nccl"))
    parser.add_argument("--load", action="store_true", help="checkpoint loading to the GPU instead of generation")
    parser.add_argument("--compare", action="store_true",
                        help="this engine against Transformers (static cache) and vLLM on the workload")
    args = parser.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    if args.impl == "reference":
        line = run_reference(args, rank)
    elif args.load:
        line = run_load(args) if rank == 0 else None
    elif args.compare:
        line = run_compare(args) if rank == 0 else None
    else:
        if world > 1:
            import datetime

            import torch.distributed as dist
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
        try:
            line = run_tp(args, rank, world) if args.tp else run_ours(args, rank, world)
        finally:
            if world > 1:
                import torch.distributed as dist
                dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
