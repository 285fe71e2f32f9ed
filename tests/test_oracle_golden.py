"""The oracle restatement against the reference's own outputs (CPU only)."""
import numpy as np
import pytest
import torch

from conftest import GOLDENS, GOLDEN_IDS
from oracle import reference_model as oracle
from ttjam_gottagofast_b200.contract import generate_random_case


@pytest.mark.parametrize("case", GOLDENS, ids=GOLDEN_IDS)
def test_weights_regenerate_from_seed(case):
    """init_params(seed) reproduces the reference module's weights bit for bit
    (checked against the parameter checksums stored with each golden)."""
    p = oracle.init_params(case.config, seed=case.meta["model_seed"])
    ref = case.meta["param_checksums"]
    assert set(p) == set(ref)
    for k, (s, a) in ref.items():
        assert float(p[k].double().sum()) == s, k
        assert float(p[k].double().abs().sum()) == a, k


@pytest.mark.parametrize("case", GOLDENS, ids=GOLDEN_IDS)
def test_inputs_regenerate_from_seed(case):
    m = case.meta
    if m["mask_kind"] == "holes":
        pytest.skip("explicit non-prefix mask, stored in the fixture")
    x, mask = generate_random_case(case.config, "cpu", torch.float32, m["data_seed"],
                                   m["padding_ratio"], m["input_scale"])
    assert np.array_equal(x.numpy(), case.x)
    assert np.array_equal(mask.numpy(), case.mask)


@pytest.mark.parametrize("case", GOLDENS, ids=GOLDEN_IDS)
def test_oracle_matches_reference_goldens(case):
    """Same ops in the same order on the same CPU: equal to rounding."""
    if case.meta["d_model"] >= 1024 and case.meta["num_layers"] > 4:
        pass  # still fast enough at the reduced batch/sequence of the fixture
    p = oracle.init_params(case.config, seed=case.meta["model_seed"])
    x = torch.from_numpy(case.x)
    mask = torch.from_numpy(case.mask) if case.uses_mask else None
    y = oracle.forward(p, case.config, x, mask).numpy()
    assert np.isfinite(y).all()
    np.testing.assert_allclose(y, case.y, rtol=0, atol=2e-6)


def test_oracle_batch_chunking_is_exact():
    case = next(g for g in GOLDENS if g.name == "C_small")
    p = oracle.init_params(case.config)
    x, mask = torch.from_numpy(case.x), torch.from_numpy(case.mask)
    a = oracle.forward(p, case.config, x, mask)
    b = oracle.forward(p, case.config, x, mask, batch_chunk=1)
    assert torch.equal(a, b)


@pytest.mark.parametrize("case", GOLDENS, ids=GOLDEN_IDS)
def test_oracle_query_chunking_matches_reference_goldens(case):
    """The query-blocked attention (for sequences too long for one [S,S] score
    tensor) against the reference's own outputs: blocks of 16 query rows,
    causal key truncation included, agree with the reference to rounding."""
    p = oracle.init_params(case.config, seed=case.meta["model_seed"])
    x = torch.from_numpy(case.x)
    mask = torch.from_numpy(case.mask) if case.uses_mask else None
    y = oracle.forward(p, case.config, x, mask, query_chunk=16).numpy()
    assert np.isfinite(y).all()
    np.testing.assert_allclose(y, case.y, rtol=0, atol=1e-5)
