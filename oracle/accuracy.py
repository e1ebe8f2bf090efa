"""The reference's accuracy rule, restated. TEST INFRASTRUCTURE ONLY.

Follows `tests/needs_torch/accuracy.py:16-45`: per position, against fp64 oracle logits,
e = max|logit - oracle| over the vocabulary and kl = KL(oracle || candidate). A candidate passes
when median(e) and max(e) are within 2x, and mean(kl) within 4x, of the largest such summary among
the reference variants on the same positions; NaN fails.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

FACTORS = {"median_abs": 2.0, "max_abs": 2.0, "mean_kl": 4.0}


@dataclass(frozen=True)
class Errors:
    max_abs: torch.Tensor  # per position, fp64
    kl: torch.Tensor  # per position, fp64

    def summary(self) -> dict[str, float]:
        return {"median_abs": self.max_abs.median().item(), "max_abs": self.max_abs.max().item(),
                "mean_kl": self.kl.mean().item()}


def errors(oracle: torch.Tensor, logits: torch.Tensor) -> Errors:
    """Per-position errors of logits [..., V] against fp64 oracle logits of the same shape."""
    vocab = oracle.shape[-1]
    o = oracle.reshape(-1, vocab).double()
    x = logits.reshape(-1, vocab).double().to(o.device)
    log_o, log_x = torch.log_softmax(o, dim=-1), torch.log_softmax(x, dim=-1)
    kl = (log_o.exp() * (log_o - log_x)).sum(-1).clamp_min(0)
    return Errors((x - o).abs().amax(-1), kl)


def concat(parts: list[Errors]) -> Errors:
    return Errors(torch.cat([p.max_abs.cpu() for p in parts]), torch.cat([p.kl.cpu() for p in parts]))


def failures(candidate: Errors, references: list[Errors], factors: dict[str, float] | None = None) -> list[str]:
    """The summaries the candidate exceeds; empty when it passes."""
    factors = FACTORS if factors is None else factors
    mine = candidate.summary()
    scale = {name: max(r.summary()[name] for r in references) for name in factors}
    return [f"{name} {mine[name]:.3e} > {factor} x {scale[name]:.3e}"
            for name, factor in factors.items() if not mine[name] <= factor * scale[name]]
