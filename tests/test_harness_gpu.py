"""The reference harness's per-case checks (tests/harness_run.py, a restatement
of tools/harness.py) on three official cases, with fewer timing repeats than
the full run: the candidate file loaded by path, built from the contract
module's baseline, five input variants through the accuracy gate, the
anti-caching check, the wall/event <= 1.6 stream gate, and the global torch
flags unchanged."""
import pytest

pytestmark = pytest.mark.gpu


def test_restated_harness_on_three_official_cases():
    import harness_run
    args = harness_run.parse_args(["--warmup", "5", "--repeats", "10", "--rounds", "2"])
    report = harness_run.run({2, 7, 12}, args)
    for case in report["cases"]:
        assert case["status"] == "ok", case
        assert case["candidate_class_mro"][:2] == ["UserOptimizedTransformer", "TTForward"]
        assert case["candidate_class_mro"][2] == "BaselineTransformer"
        assert all(v["passed"] for v in case["correctness"]["variants"])
        assert case["input_dependence_ok"]
        assert case["wall_to_event_ratio"] < 1.6
    assert report["env_unchanged"], (report["env_before"], report["env_after"])
    assert report["failed_cases"] == []
