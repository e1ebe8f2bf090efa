"""Per-phase timeline of the one-kernel decode step, from its device trace (`ipe_decode_step_desc.trace`).

    python -m ipe_b200.steptrace [--batch B] [--prompt P]                # one GPU, Engine
    torchrun --nproc-per-node N -m ipe_b200.steptrace --tp [...]         # N ranks, fused TP step

Builds the random-init Qwen3-1.7B (seed 0, drawn on the GPU), prefills a random prompt, runs a
few generation steps, then times 20 untraced steps (CUDA events) and one traced step, and prints
for each phase kind (embedding, QKV, attention, o_proj, gate/up, down_proj, LM head), summed over
the step's layers:
- stage: from the end of the previous phase (a grid-barrier release, or in a tensor-parallel step
  this CTA's own end of a row-parallel phase) to the phase's activations staged, worst CTA; in a
  tensor-parallel step it includes waiting for the peers' parts;
- work: from the earliest CTA staged to the last CTA's end of the phase;
- barrier: from the last arrival to the first release (negative when the phase ends without a
  grid barrier, as the row-parallel phases of a tensor-parallel step do);
and the sampling tail (CTA 0's exit after the last CTA's end of the LM head).
"""

from __future__ import annotations

import argparse
import ctypes
import os

import torch

from ipe_b200 import _native as nat

KINDS = ("qkv", "attn", "o", "gu", "down")


def traced_step(desc, grid: int, layers: int, stream: int, device: torch.device) -> torch.Tensor:
    """Run one decode step described by `desc` (an ipe_decode_step_desc) with tracing on; returns
    the raw trace [grid, IPE_TRACE_WORDS(layers)] of globaltimer nanoseconds."""
    trace = torch.zeros(grid, nat.trace_words(layers), dtype=torch.int64, device=device)
    traced = nat.StepDesc.from_buffer_copy(desc)
    traced.trace = trace.data_ptr()
    nat.check(nat.load().ipe_decode_step(ctypes.addressof(traced), stream), "ipe_decode_step")
    torch.cuda.synchronize(device)
    return trace.cpu()


def summarize(raw: torch.Tensor, layers: int) -> dict:
    """Per phase kind: [stage, work, barrier] microseconds summed over the step, and the totals."""
    words = nat.trace_words(layers)
    t = (raw - raw[:, 0].min()).double() / 1000.0
    ends = 5 * layers + 2
    table: dict[str, list[float]] = {}
    for p in range(1, ends + 1):
        b = 1 + 5 * (p - 1)
        kind = "embed" if p == 1 else ("lm" if p == ends else KINDS[(p - 2) % 5])
        start = t[:, b - 4] if p > 1 else t[:, 0]
        staged = t[:, b - 3] if p > 1 else t[:, 0]
        row = table.setdefault(kind, [0.0, 0.0, 0.0])
        row[0] += (staged - start).max().item()
        if kind != "attn":  # attention marks no staging; its work is in the barrier that follows
            row[1] += (t[:, b].max() - staged.min()).item()
        row[2] += (t[:, b + 1].min() - t[:, b].max()).item()
    lm_end = t[:, words - 2].max().item()
    return {"phases": table, "lm_end_us": lm_end, "sampling_tail_us": t[0, words - 1].item() - lm_end}


def detail(raw: torch.Tensor, layers: int) -> dict:
    """Per phase kind, microseconds summed over the step's layers, means over the CTAs that stamped
    them (a CTA without units in a phase leaves its tile stamps at zero): [phase span (first CTA's
    start to the next phase's first release), stage (start to activations staged), to first stage
    (staged to the first weight stage ready; attention: the first item's q ready to its P.V done),
    stream (first to last weight stage ready; attention: P.V done to the item merged), tail (last
    stage to the barrier arrival), barrier (last arrival to first release)]."""
    t = (raw - raw[:, 0].min()).double() / 1000.0
    t[raw == 0] = float("nan")
    ends = 5 * layers + 2
    table: dict[str, list[float]] = {}

    def mean(x):
        x = x[~torch.isnan(x)]
        return x.mean().item() if len(x) else 0.0

    def valid(x):
        return x[~torch.isnan(x)]

    for p in range(2, ends + 1):
        b = 1 + 5 * (p - 1)
        kind = "lm" if p == ends else KINDS[(p - 2) % 5]
        rel, staged, first, last, arr, nxt = t[:, b - 4], t[:, b - 3], t[:, b - 2], t[:, b - 1], t[:, b], t[:, b + 1]
        row = table.setdefault(kind, [0.0] * 6)
        end = valid(nxt if p < ends else arr).max() if p < ends else valid(arr).max()
        row[0] += (end - valid(rel).min()).item()
        row[1] += mean(staged - rel)
        row[2] += mean(first - staged)
        row[3] += mean(last - first)
        row[4] += mean(arr - torch.where(torch.isnan(last), staged, last))
        if p < ends:
            row[5] += (valid(nxt).min() - valid(arr).max()).item()
    return table


def format_detail(table: dict) -> str:
    lines = [f"{'phase':6s} {'span':>8s} {'stage':>8s} {'to first':>8s} {'stream':>8s} {'tail':>8s} {'barrier':>8s}"
             "   (us, summed over the step; means over CTAs)"]
    for kind, row in table.items():
        lines.append(f"{kind:6s} " + " ".join(f"{v:8.1f}" for v in row))
    return "\n".join(lines)


def exchange_stage_us(raw: torch.Tensor, layers: int) -> float:
    """Tensor-parallel step: microseconds per step that the CTAs spend, on average, between the end of
    a row-parallel phase (o_proj, down_proj; its parts pushed to every rank) and the next phase's
    activations staged (the peers' parts received, summed into the residual stream, normalised):
    the exposed part of the two exchanges of each layer."""
    t = (raw - raw[:, 0].min()).double() / 1000.0
    total = 0.0
    for p in range(2, 5 * layers + 2):
        kind = KINDS[(p - 2) % 5]
        if kind not in ("gu", "qkv") or (kind == "qkv" and p == 2):
            continue
        b = 1 + 5 * (p - 1)
        total += (t[:, b - 3] - t[:, b - 4]).mean().item()
    return total


def format_summary(summary: dict, untraced_us: float, label: str) -> str:
    lines = [f"{label}: untraced step {untraced_us:.1f} us; LM head done at {summary['lm_end_us']:.1f} us; "
             f"sampling tail {summary['sampling_tail_us']:.1f} us",
             f"{'phase':6s} {'stage':>8s} {'work':>8s} {'barrier':>8s}   (us, summed over the step)"]
    for kind, (stage, work, barrier) in summary["phases"].items():
        lines.append(f"{kind:6s} {stage:8.1f} {work:8.1f} {barrier:8.1f}")
    return "\n".join(lines)


def main() -> None:
    import datetime

    from ipe_b200 import QWEN3_1_7B
    from ipe_b200.synthetic import random_model

    parser = argparse.ArgumentParser(prog="python -m ipe_b200.steptrace")
    parser.add_argument("--batch", type=int, default=1)
    parser.add_argument("--prompt", type=int, default=512)
    parser.add_argument("--tp", action="store_true", help="tensor-parallel fused step over the torchrun ranks")
    parser.add_argument("--detail", action="store_true", help="also print the per-phase means over the CTAs")
    args = parser.parse_args()
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(device)
    if args.tp:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    loaded = random_model(QWEN3_1_7B, seed=0, device=device, generator_device=device)
    ids = torch.randint(0, QWEN3_1_7B.vocab_size, (args.batch, args.prompt), generator=torch.Generator().manual_seed(0))
    if args.tp:
        from ipe_b200.tp import TensorParallelEngine

        engine = TensorParallelEngine(loaded, batch=args.batch, capacity=args.prompt + 64, allreduce="fused")
        engine.generate(ids, 8)
        desc = engine._step_desc(True)
    else:
        from ipe_b200.engine import Engine

        engine = Engine(loaded, batch=args.batch, capacity=args.prompt + 64)
        engine.generate(ids, 8)
        desc = engine._step_descs[(args.batch, True)]
    lib = nat.load()
    stream = torch.cuda.current_stream().cuda_stream
    layers = QWEN3_1_7B.num_hidden_layers
    if args.tp:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(20):
        nat.check(lib.ipe_decode_step(ctypes.addressof(desc), stream), "ipe_decode_step")
    e1.record()
    torch.cuda.synchronize()
    untraced = e0.elapsed_time(e1) / 20 * 1000
    if args.tp:
        dist.barrier()
    raw = traced_step(desc, lib.ipe_decode_step_grid(), layers, stream, device)
    error = nat.device_error()
    summary = summarize(raw, layers)
    if args.tp:
        gathered = [None] * world
        extra = (exchange_stage_us(raw, layers), detail(raw, layers) if args.detail else None)
        dist.all_gather_object(gathered, (summary, untraced, error, extra))
        if rank == 0:
            for r, (s, u, err, (exchange, table)) in enumerate(gathered):
                print(format_summary(s, u, f"rank {r} of {world} (device error {err})"), flush=True)
                print(f"staging after the exchanges: {exchange:.1f} us per step (mean over CTAs)", flush=True)
                if table is not None:
                    print(format_detail(table), flush=True)
        engine.close()
        torch.cuda.synchronize()
        dist.destroy_process_group()
    else:
        print(format_summary(summary, untraced, f"one GPU, batch {args.batch} (device error {error})"), flush=True)
        if args.detail:
            print(format_detail(detail(raw, layers)), flush=True)


if __name__ == "__main__":
    main()
