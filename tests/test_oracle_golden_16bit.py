"""The oracle's 16-bit path against the reference's own 16-bit outputs (CPU only).

The reference runs a float16 / bfloat16 benchmark by moving model and input to
that dtype (torch_transformer_benchmark.py:225-231, :698-699); its bfloat16
outputs, and the fp32 outputs of the same 16-bit weights and inputs, were
recorded by tests/golden/make_golden_16bit.py.
"""
import numpy as np
import pytest
import torch

from conftest import GOLDENS_16BIT, GOLDEN_16BIT_IDS
from oracle import reference_model as oracle
from ttjam_gottagofast_b200.contract import generate_random_case


def _params16(case):
    p = oracle.init_params(case.config, seed=case.meta["model_seed"])
    return {k: v.to(case.dtype) for k, v in p.items()}


@pytest.mark.parametrize("case", GOLDENS_16BIT, ids=GOLDEN_16BIT_IDS)
def test_16bit_weights_regenerate_from_seed(case):
    """init_params(seed) rounded to the dtype is the reference module after
    `.to(dtype)`: the checksums of the widened weights match."""
    p = _params16(case)
    for k, (s, a) in case.meta["param_checksums"].items():
        assert float(p[k].double().sum()) == s, k
        assert float(p[k].double().abs().sum()) == a, k


@pytest.mark.parametrize("case", GOLDENS_16BIT, ids=GOLDEN_16BIT_IDS)
def test_16bit_inputs_regenerate_from_seed(case):
    m = case.meta
    x, mask = generate_random_case(case.config, "cpu", case.dtype, m["data_seed"],
                                   m["padding_ratio"], m["input_scale"])
    assert x.dtype == case.dtype
    assert np.array_equal(x.float().numpy(), case.x)
    assert np.array_equal(mask.numpy(), case.mask)


@pytest.mark.parametrize("case", GOLDENS_16BIT, ids=GOLDEN_16BIT_IDS)
def test_oracle_16bit_forward_matches_reference(case):
    """The oracle in the 16-bit dtype runs the reference's ops in its order on
    the same CPU: bit for bit the reference's 16-bit output."""
    p = _params16(case)
    x = torch.from_numpy(case.x).to(case.dtype)
    mask = torch.from_numpy(case.mask)
    y = oracle.forward(p, case.config, x, mask)
    assert y.dtype == case.dtype
    assert np.array_equal(y.float().numpy(), case.y)


@pytest.mark.parametrize("case", GOLDENS_16BIT, ids=GOLDEN_16BIT_IDS)
def test_oracle_fp32_value_of_16bit_model_matches_reference(case):
    p = {k: v.float() for k, v in _params16(case).items()}
    x = torch.from_numpy(case.x)
    mask = torch.from_numpy(case.mask)
    y = oracle.forward(p, case.config, x, mask).numpy()
    np.testing.assert_allclose(y, case.y_f32, rtol=0, atol=2e-6)


def test_reference_16bit_forward_is_outside_the_fp32_gate():
    """Why 16-bit parity is stated against the fp32 value of the 16-bit model:
    the reference's own bfloat16 forward misses the contract's fp32 gate
    (abs 2e-3 or rel 2e-2) on every case."""
    from ttjam_gottagofast_b200.contract import compare_outputs
    for case in GOLDENS_16BIT:
        res = compare_outputs(torch.from_numpy(case.y_f32), torch.from_numpy(case.y))
        assert not res.passed, case.name
