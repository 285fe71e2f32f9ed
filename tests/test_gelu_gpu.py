"""The GELU every schedule applies after ffn_in, against a float64 GELU.

F.gelu(approximate="none") (torch_transformer_benchmark.py:141) is
x * Phi(x). The kernels compute Phi from the Numerical Recipes Chebyshev fit of
erfc (fractional error below 1.2e-7); this checks the device function itself,
through tt_test_gelu, over a dense grid, random arguments and edge values."""
import math

import pytest
import torch

from ttjam_gottagofast_b200 import _lib

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _gelu_dev(x):
    lib = _lib.load()
    y = torch.empty_like(x)
    _lib.check(lib.tt_test_gelu(x.data_ptr(), y.data_ptr(), x.numel(),
                                torch.cuda.current_stream().cuda_stream), "tt_test_gelu", lib)
    torch.cuda.synchronize()
    return y


def _gelu_f64(x):
    """x * erfc(-x / sqrt 2) / 2 in float64: no cancellation in either tail."""
    x64 = x.double()
    return 0.5 * x64 * torch.special.erfc(-x64 / math.sqrt(2.0))


def test_gelu_matches_float64_to_fp32_accuracy():
    g = torch.Generator().manual_seed(3)
    xs = torch.cat([
        torch.linspace(-12.0, 12.0, 2_000_001),
        torch.randn(1_000_000, generator=g) * 3.0,
        torch.randn(100_000, generator=g) * 1e-3,
        torch.tensor([0.0, -0.0, 1e-30, -1e-30, 1e-6, -1e-6, 30.0, -30.0, 1e4, -1e4,
                      65504.0, -65504.0, 3e38, -3e38]),
    ]).float()
    y = _gelu_dev(xs.to(DEV)).cpu()
    ref = _gelu_f64(xs)
    err = (y.double() - ref).abs()
    bound = 1e-6 * xs.double().abs() + 1e-37
    worst = int(torch.argmax(err / bound))
    print(f"max abs error {float(err.max()):.3e}; worst relative to the bound at x={float(xs[worst])}: "
          f"{float(err[worst] / bound[worst]):.3f}")
    assert torch.isfinite(y).all()
    assert bool((err <= bound).all())
    # no worse than torch's own fp32 GELU (erff) by more than the bound
    t32 = torch.nn.functional.gelu(xs.to(DEV), approximate="none").cpu().double()
    assert float(err.max()) <= float((t32 - ref).abs().max()) + 1e-6 * 12


def test_gelu_special_values():
    x = torch.tensor([float("inf"), float("-inf"), float("nan"), 0.0], device=DEV)
    y = _gelu_dev(x).cpu()
    assert y[0] == float("inf")
    assert math.isnan(float(y[1])) and math.isnan(float(y[2]))   # as 0.5*x*(1+erf(x/sqrt2))
    assert y[3] == 0.0
