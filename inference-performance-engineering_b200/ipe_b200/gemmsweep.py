"""Timing of the tcgen05 prefill GEMM (ipe_gemm) on the Qwen3-1.7B layer shapes, for choosing its
output-tile width.

    python -m ipe_b200.gemmsweep 512 4096            # the library's own width choice
    IPE_GEMM_BN=64 python -m ipe_b200.gemmsweep 512  # a forced width (64, 128 or 256, where valid)

For each row count M, times QKV (N 4096, K 2048, store), o_proj (2048 x 2048, residual), gate/up
(12288 x 2048, SiLU*up) and down_proj (2048 x 6144, residual) with CUDA events around 24 launches
that cycle through 8 random weight copies (so B streams from HBM, as across a model's layers), and
prints one JSON line of microseconds and TFLOP/s per GEMM.
"""

from __future__ import annotations

import json
import os
import sys

import torch

from ipe_b200 import _native as nat

SHAPES = {"qkv": (4096, 2048, "store"), "o_proj": (2048, 2048, "residual"), "gate_up": (12288, 2048, "silu"),
          "down_proj": (2048, 6144, "residual")}


def time_gemms(rows: list[int], copies: int = 8, repeats: int = 24) -> dict:
    lib = nat.load()
    dev = torch.device("cuda", torch.cuda.current_device())
    epilogues = {"store": nat.EPI_STORE, "residual": nat.EPI_RESIDUAL, "silu": nat.EPI_SILU_MUL}
    stream = torch.cuda.current_stream().cuda_stream
    out = {}
    for m in rows:
        for name, (n, k, epi_name) in SHAPES.items():
            epi = epilogues[epi_name]
            a = torch.randn((m, k), device=dev).bfloat16()
            weights = [(torch.randn((n, k), device=dev) * 0.02).bfloat16() for _ in range(copies)]
            c = torch.randn((m, n // 2 if epi == nat.EPI_SILU_MUL else n), device=dev).bfloat16()
            residual = c.data_ptr() if epi == nat.EPI_RESIDUAL else 0

            def launch(w):
                nat.check(lib.ipe_gemm(a.data_ptr(), w.data_ptr(), c.data_ptr(), m, n, k, epi, residual, stream),
                          "ipe_gemm")

            for w in weights:
                launch(w)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for r in range(repeats):
                launch(weights[r % copies])
            e1.record()
            e1.synchronize()
            us = e0.elapsed_time(e1) / repeats * 1000
            out[f"{m}/{name}"] = {"us": round(us, 2), "tflops": round(2.0 * m * n * k / us / 1e6, 1)}
    return out


def main() -> None:
    rows = [int(x) for x in sys.argv[1:]] or [512, 4096]
    result = time_gemms(rows)
    print(json.dumps({"bn": os.environ.get("IPE_GEMM_BN", "auto"), "device_error": nat.device_error(), "gemm": result}))


if __name__ == "__main__":
    main()
