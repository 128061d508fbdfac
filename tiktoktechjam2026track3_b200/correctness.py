"""Correctness gates for the Transformer forward pass.

Two gates, both reported by the tests and the bench:

* `compare_outputs` — the reference harness's strict elementwise rule
  (transformer_benchmark/correctness.py:40-109): an element passes iff both values are finite and
  |opt - ref| < atol OR |opt - ref| < rtol * |ref|. Same result fields as the reference's
  AccuracyResult.
* `baseline_gate` — the acceptance rule of this build: against the fp32 result of the
  reference computation on the same (bf16-rounded) weights and inputs, the bf16 output must satisfy
      max |y - r|  <=  2^-7 * max |r|
  with every element finite (0 NaN/Inf). Also reports the elementwise
  max |y - r| / max(1, |r|) as a diagnostic.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import torch

GATE_RELATIVE_TOLERANCE = 2.0**-7


@dataclass
class AccuracyResult:
    passed: bool
    total_elements: int
    failed_elements: int
    max_abs_error: float
    max_relative_error: float
    mean_abs_error: float
    failed_feature_dims: List[int]
    worst_index: Tuple[int, ...]
    reference_at_worst: float
    optimized_at_worst: float


def compare_outputs(reference: torch.Tensor, optimized: torch.Tensor, rtol: float, atol: float) -> AccuracyResult:
    """The reference harness's strict OR rule (transformer_benchmark/correctness.py:40-109)."""
    if reference.shape != optimized.shape:
        raise AssertionError(
            f"shape mismatch: baseline={tuple(reference.shape)}, optimized={tuple(optimized.shape)}"
        )
    ref = reference.detach().float()
    opt = optimized.detach().float()
    finite = torch.isfinite(ref) & torch.isfinite(opt)
    abs_error = (opt - ref).abs()
    passed_mask = finite & ((abs_error < atol) | (abs_error < rtol * ref.abs()))
    failed_mask = ~passed_mask
    failed = int(failed_mask.sum().item())
    flat_worst = int(abs_error.reshape(-1).argmax().item())
    worst = []
    rem = flat_worst
    for size in reversed(reference.shape):
        worst.append(rem % size)
        rem //= size
    worst_index = tuple(reversed(worst))
    rel = abs_error / ref.abs().clamp_min(1e-12)
    if reference.ndim == 0:
        dims = [0] if failed else []
    elif reference.ndim == 1:
        dims = torch.nonzero(failed_mask, as_tuple=False).flatten().tolist()
    else:
        dims = torch.nonzero(failed_mask.any(dim=tuple(range(reference.ndim - 1))), as_tuple=False).flatten().tolist()
    return AccuracyResult(
        passed=failed == 0,
        total_elements=reference.numel(),
        failed_elements=failed,
        max_abs_error=float(abs_error.max().item()),
        max_relative_error=float(rel.max().item()),
        mean_abs_error=float(abs_error.mean().item()),
        failed_feature_dims=dims,
        worst_index=worst_index,
        reference_at_worst=float(ref[worst_index].item()),
        optimized_at_worst=float(opt[worst_index].item()),
    )


@dataclass
class GateResult:
    passed: bool
    max_abs_error: float
    max_abs_reference: float
    normwise_error: float  # max|y - r| / max|r|
    elementwise_error: float  # max |y - r| / max(1, |r|)
    nonfinite: int
    tolerance: float = GATE_RELATIVE_TOLERANCE


def baseline_gate(output: torch.Tensor, reference_fp32: torch.Tensor) -> GateResult:
    """max|y - r| <= 2^-7 * max|r| and no NaN/Inf in y."""
    y = output.detach().float()
    r = reference_fp32.detach().float().to(y.device)
    nonfinite = int((~torch.isfinite(y)).sum().item())
    err = (y - r).abs()
    max_err = float(err.max().item()) if err.numel() else 0.0
    max_ref = float(r.abs().max().item()) if r.numel() else 0.0
    elem = float((err / r.abs().clamp_min(1.0)).max().item()) if err.numel() else 0.0
    normwise = max_err / max_ref if max_ref > 0 else max_err
    passed = nonfinite == 0 and max_err <= GATE_RELATIVE_TOLERANCE * max_ref
    return GateResult(passed, max_err, max_ref, normwise, elem, nonfinite)
