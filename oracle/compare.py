"""Accuracy gate, restating ``compare_outputs`` (torch_transformer_benchmark.py:1616-1697).

Per element: ``abs(opt - ref) <= atol OR abs(opt - ref) <= rtol * abs(ref)``,
with any non-finite value on either side counted as a failure (:1650-1657).
This is the exact OR condition, not ``torch.isclose`` (which adds the two).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import torch

ATOL = 2e-3   # torch_transformer_benchmark.py:1960 (argparse default), the harness gate
RTOL = 2e-2   # :1959


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


def compare_outputs(reference: torch.Tensor, optimized: torch.Tensor,
                    rtol: float = RTOL, atol: float = ATOL) -> AccuracyResult:
    if reference.shape != optimized.shape:
        raise AssertionError(f"shape mismatch: baseline={tuple(reference.shape)}, "
                             f"optimized={tuple(optimized.shape)}")
    ref = reference.detach().double().cpu()
    opt = optimized.detach().double().cpu()
    finite = torch.isfinite(ref) & torch.isfinite(opt)
    err = (opt - ref).abs()
    passed = finite & ((err <= atol) | (err <= rtol * ref.abs()))
    failed = ~passed
    n_failed = int(failed.sum())
    err_f = torch.where(torch.isfinite(err), err, torch.full_like(err, float("inf")))
    flat = int(err_f.reshape(-1).argmax()) if err.numel() else 0
    idx = []
    rem = flat
    for size in reversed(reference.shape):
        idx.append(rem % size)
        rem //= size
    worst = tuple(reversed(idx))
    rel = err / ref.abs().clamp_min(1e-12)
    if reference.ndim >= 2:
        dims = torch.nonzero(failed.any(dim=tuple(range(reference.ndim - 1))),
                             as_tuple=False).flatten().tolist()
    else:
        dims = torch.nonzero(failed, as_tuple=False).flatten().tolist()
    return AccuracyResult(
        passed=n_failed == 0,
        total_elements=reference.numel(),
        failed_elements=n_failed,
        max_abs_error=float(err_f.max()) if err.numel() else 0.0,
        max_relative_error=float(rel.max()) if err.numel() else 0.0,
        mean_abs_error=float(err.mean()) if err.numel() else 0.0,
        failed_feature_dims=dims,
        worst_index=worst,
        reference_at_worst=float(ref[worst]) if err.numel() else 0.0,
        optimized_at_worst=float(opt[worst]) if err.numel() else 0.0,
    )
