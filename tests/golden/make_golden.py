"""Generate the golden vectors under tests/golden/ by running the REFERENCE implementation.

Run in a container that has the reference checkout (read-only is fine):

    python tests/golden/make_golden.py --reference <path of the reference checkout>

It imports the reference package `ipe` from `<reference>/src` (torch CPU), builds seeded synthetic
models with `ipe_b200.synthetic.random_model`, wraps the same tensors in the reference's own
dataclasses, and records what the reference computes:

- `forward_full` logits (bf16/fp32, math/sdpa) and the fp64 oracle
  (`lm_logits(final_hidden(float64))`) at a set of positions;
- the reference `Engine`'s teacher-forced logits and greedy `generate` output;
- the reference rotary tables.

Small-vocabulary models store full logits; full-vocabulary (151,936) models store per-position
summaries (top-16 IDs and values, sum, sum of squares). The tests rebuild the same models and
check `oracle/` against these files; the reference itself is never needed at test time.
"""

from __future__ import annotations

import argparse
import dataclasses
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "inference-performance-engineering_b200"))

from ipe_b200.config import QWEN3_0_6B, QWEN3_1_7B, Qwen3Config  # noqa: E402
from ipe_b200.synthetic import random_model  # noqa: E402

# name -> (config, init arguments, batch, length, prompt, full logits?)
CASES = {
    "small": (Qwen3Config(2048, 256, 512, 2, 4, 2, 128, 8192, 1e-5, 1e4),
              {"seed": 1, "std": 0.06, "norm_jitter": 0.1}, 2, 32, 20, True),
    "mqa": (Qwen3Config(512, 128, 384, 3, 4, 1, 128, 8192, 1e-6, 1e6),
            {"seed": 2, "std": 0.08, "norm_jitter": 0.1}, 2, 32, 20, True),
    "qwen3-0.6b-2layer": (dataclasses.replace(QWEN3_0_6B, num_hidden_layers=2),
                          {"seed": 0, "std": 0.02}, 1, 40, 24, False),
    "qwen3-1.7b-2layer": (dataclasses.replace(QWEN3_1_7B, num_hidden_layers=2),
                          {"seed": 0, "std": 0.02}, 1, 40, 24, False),
}
TOP = 16


def summarize(logits: torch.Tensor) -> dict[str, torch.Tensor]:
    flat = logits.reshape(-1, logits.shape[-1]).double()
    values, ids = flat.topk(TOP, dim=-1)
    return {"top_ids": ids, "top_values": values, "sum": flat.sum(-1), "sumsq": flat.pow(2).sum(-1)}


def to_reference(ipe_weights, ipe_config, loaded):
    c = loaded.config
    config = ipe_config.Qwen3Config(**{f.name: getattr(c, f.name) for f in dataclasses.fields(c)})
    w = loaded.weights
    layers = tuple(ipe_weights.LayerWeights(**{f: getattr(layer, f) for f in layer.__slots__}) for layer in w.layers)
    weights = ipe_weights.Qwen3Weights(w.embed_tokens, layers, w.norm, w.embed_tokens)
    return ipe_weights.LoadedCheckpoint(config, weights, ipe_weights.TieRecord(stored=False, tied=True, max_abs_diff=None))


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of the reference checkout (its src/ holds ipe)")
    parser.add_argument("--only", nargs="*")
    args = parser.parse_args()
    sys.path.insert(0, str(Path(args.reference) / "src"))
    import ipe.config as ipe_config
    import ipe.weights as ipe_weights
    from ipe import ops
    from ipe.engine import Engine
    from ipe.forward import final_hidden, forward_full, lm_logits

    torch.manual_seed(0)
    for name, (config, init, batch, length, prompt, full) in CASES.items():
        if args.only and name not in args.only:
            continue
        loaded = random_model(config, **init)
        ref = to_reference(ipe_weights, ipe_config, loaded)
        ids = torch.randint(0, config.vocab_size, (batch, length), generator=torch.Generator().manual_seed(7))
        positions = list(range(prompt - 1, length))
        out: dict[str, object] = {"token_ids": ids, "positions": torch.tensor(positions), "prompt": prompt,
                                  "embed_checksum": loaded.weights.embed_tokens.double().sum()}
        with torch.no_grad():
            logits = {"oracle": lm_logits(ref, final_hidden(ref, ids, dtype=torch.float64)[:, positions])}
            for dtype in (torch.bfloat16, torch.float32):
                for backend in ("math", "sdpa"):
                    key = f"forward_{str(dtype)[6:]}_{backend}"
                    logits[key] = forward_full(ref, ids, dtype=dtype, backend=backend, logit_positions=positions)
                engine = Engine(ref, batch=batch, capacity=length + 1, dtype=dtype, backend="sdpa")
                steps = [engine.prefill(ids[:, :prompt])]
                steps += [engine.decode(ids[:, p]) for p in range(prompt, length)]
                logits[f"engine_{str(dtype)[6:]}_sdpa"] = torch.stack(steps, dim=1)
                generated = engine.generate(ids[:, :prompt], 12)
                out[f"generate_{str(dtype)[6:]}_tokens"] = generated.tokens
                out[f"generate_{str(dtype)[6:]}_logprobs"] = generated.logprobs
            cos, sin = ops.rotary_tables(torch.arange(length + 1), config.head_dim, config.rope_theta, torch.bfloat16)
            out["rotary_cos_bf16"], out["rotary_sin_bf16"] = cos, sin
        for key, value in logits.items():
            out[key] = value if full else summarize(value)
        target = HERE / f"{name}.pt"
        torch.save(out, target)
        print(f"{name}: wrote {target.stat().st_size / 1e3:.0f} kB")


if __name__ == "__main__":
    main()
