"""Host-side contract: config validation, the accuracy gate, module structure."""
import pytest
import torch

from conftest import GOLDENS
from oracle import reference_model as oracle
from ttjam_gottagofast_b200 import (TransformerConfig, UserOptimizedTransformer,
                                    build_model, compare_outputs, load_from_baseline)
from ttjam_gottagofast_b200.config import WORKLOADS


def _cfg(**kw):
    base = dict(batch_size=2, seq_len=4, d_model=128, num_heads=4, ffn_dim=128,
                num_layers=2, causal=True)
    base.update(kw)
    return TransformerConfig(**base)


@pytest.mark.parametrize("field,value,msg", [
    ("batch_size", 0, "batch_size must be positive"),
    ("seq_len", -1, "seq_len must be positive"),
    ("d_model", 0, "d_model must be positive"),
    ("num_heads", 0, "num_heads must be positive"),
    ("num_heads", 3, "must be divisible by"),
    ("ffn_dim", 0, "ffn_dim must be positive"),
    ("num_layers", 0, "num_layers must be positive"),
])
def test_validate_matches_reference_rules(field, value, msg):
    with pytest.raises(ValueError, match=msg):
        _cfg(**{field: value}).validate()


def test_workloads_are_valid():
    for w in WORKLOADS.values():
        w.config.validate()


def test_gate_is_exact_or_rule():
    ref = torch.tensor([1.0, 100.0, 0.0, 1.0])
    # 0.0019 abs passes by atol; 1.9 on 100 passes by rtol; 0.003 on 0 fails
    opt = torch.tensor([1.0019, 101.9, 0.003, 1.0])
    r = compare_outputs(ref, opt)
    assert not r.passed and r.failed_elements == 1 and r.failed_feature_dims == [2]
    assert compare_outputs(ref, torch.tensor([1.0019, 101.9, 0.0019, 1.0])).passed


def test_gate_rejects_non_finite():
    ref = torch.zeros(3)
    assert not compare_outputs(ref, torch.tensor([0.0, float("nan"), 0.0])).passed
    assert not compare_outputs(ref, torch.tensor([0.0, float("inf"), 0.0])).passed


def test_state_dict_names_match_reference():
    case = GOLDENS[0]
    model = UserOptimizedTransformer(case.config)
    assert set(model.state_dict()) == set(case.meta["param_checksums"])


def test_same_seed_same_weights_as_reference():
    cfg = WORKLOADS["B1"].config
    torch.manual_seed(1234)
    model = UserOptimizedTransformer(cfg)
    p = oracle.init_params(cfg, seed=1234)
    sd = model.state_dict()
    assert all(torch.equal(sd[k], p[k]) for k in p)


def test_candidate_hooks_load_baseline_weights():
    cfg = WORKLOADS["B1"].config
    torch.manual_seed(7)
    baseline = UserOptimizedTransformer(cfg)   # same parameter names as the reference
    model = build_model(cfg, None)
    load_from_baseline(model, baseline)
    for k, v in baseline.state_dict().items():
        assert torch.equal(model.state_dict()[k], v)


def test_forward_refuses_cpu_input():
    model = UserOptimizedTransformer(WORKLOADS["B1"].config)
    with pytest.raises(RuntimeError, match="CUDA only"):
        model(torch.zeros(4, 16, 128))


def test_load_state_dict_invalidates_packed_image():
    model = UserOptimizedTransformer(WORKLOADS["B1"].config)
    model._image = torch.zeros(1)
    model._image_key = "stale"
    model.load_state_dict(model.state_dict())
    assert model._image is None
