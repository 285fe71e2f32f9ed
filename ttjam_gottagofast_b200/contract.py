"""Input generator and accuracy gate of the forward-pass contract.

Both mirror the reference contract so that parity runs here read like the
reference's own accuracy runs:

* `generate_random_case` follows torch_transformer_benchmark.py:234-272 call for
  call (one `torch.Generator` on the given device, `randn` then `randint`), so the
  same seed gives the same x and mask as the reference on the same device type.
  CPU and CUDA generators differ, so callers generate on CPU and copy.
* `compare_outputs` is the element-wise gate of :289-356:
  ``abs(opt-ref) <= atol OR abs(opt-ref) <= rtol*abs(ref)``, and both finite.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Tuple

import torch

# Defaults of the contract's CLI (torch_transformer_benchmark.py:618-619).
RTOL = 0.02
ATOL = 0.002


def generate_random_case(config, device, dtype, seed: int, padding_ratio: float,
                         input_scale: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """torch_transformer_benchmark.py:234-272."""
    device = torch.device(device)
    generator = torch.Generator(device=device)
    generator.manual_seed(seed)
    x = torch.randn(config.batch_size, config.seq_len, config.d_model,
                    generator=generator, device=device, dtype=dtype)
    x = x * input_scale
    if padding_ratio <= 0:
        mask = torch.ones(config.batch_size, config.seq_len, device=device,
                          dtype=torch.bool)
        return x, mask
    min_valid = max(1, int(round(config.seq_len * (1.0 - padding_ratio))))
    lengths = torch.randint(low=min_valid, high=config.seq_len + 1,
                            size=(config.batch_size,), generator=generator,
                            device=device)
    positions = torch.arange(config.seq_len, device=device)[None, :]
    mask = positions < lengths[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


@dataclass
class AccuracyResult:
    """torch_transformer_benchmark.py:275-286."""

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
    """torch_transformer_benchmark.py:289-356 (exact OR rule, not torch.isclose)."""
    if reference.shape != optimized.shape:
        raise AssertionError(f"shape mismatch: baseline={tuple(reference.shape)}, "
                             f"optimized={tuple(optimized.shape)}")
    ref = reference.detach().float().cpu()
    opt = optimized.detach().float().cpu()
    finite = torch.isfinite(ref) & torch.isfinite(opt)
    err = (opt - ref).abs()
    passed_mask = finite & ((err <= atol) | (err <= rtol * ref.abs()))
    failed_mask = ~passed_mask
    failed = int(failed_mask.sum().item())
    if ref.numel() == 0:
        return AccuracyResult(True, 0, 0, 0.0, 0.0, 0.0, [], (), 0.0, 0.0)
    flat_worst = int(torch.nan_to_num(err, nan=float("inf")).reshape(-1).argmax().item())
    idx = []
    rem = flat_worst
    for size in reversed(ref.shape):
        idx.append(rem % size)
        rem //= size
    worst = tuple(reversed(idx))
    rel = err / ref.abs().clamp_min(1e-12)
    if ref.ndim >= 2:
        dims = tuple(range(ref.ndim - 1))
        failed_dims = torch.nonzero(failed_mask.any(dim=dims)).flatten().tolist()
    else:
        failed_dims = torch.nonzero(failed_mask).flatten().tolist()
    return AccuracyResult(
        passed=failed == 0, total_elements=ref.numel(), failed_elements=failed,
        max_abs_error=float(err.max().item()), max_relative_error=float(rel.max().item()),
        mean_abs_error=float(err.mean().item()), failed_feature_dims=failed_dims,
        worst_index=worst, reference_at_worst=float(ref[worst].item()),
        optimized_at_worst=float(opt[worst].item()))


# The five input variants the reference's evaluation harness checks every
# candidate on (tools/harness.py:121-127).
HARNESS_VARIANTS = [
    {"name": "normal", "seed": 11, "input_scale": 1.0, "padding_ratio": 0.0},
    {"name": "large_scale", "seed": 22, "input_scale": 8.0, "padding_ratio": 0.0},
    {"name": "small_scale", "seed": 33, "input_scale": 0.05, "padding_ratio": 0.0},
    {"name": "padded", "seed": 44, "input_scale": 1.0, "padding_ratio": 0.3},
    {"name": "padded_heavy", "seed": 55, "input_scale": 2.0, "padding_ratio": 0.7},
]
