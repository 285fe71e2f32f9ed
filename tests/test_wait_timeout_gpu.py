"""A bounded device wait that runs out ends its kernel cleanly.

tt_test_arm_wait_timeout arms a one-shot test switch: in the next launch of
the single-CTA split-precision GEMM, CTA 0's TMA producer never starts the
loads of its first k-block, so nothing ever completes that pipeline stage --
a wait on a flag that nothing sets. The bounded waits held up by it (here
2^20 cycles, about half a millisecond) run out; the kernel latches
TT_ERR_DEVICE_TIMEOUT with the detail code of the first one, stops issuing work,
waits for the copies and MMAs it had started, frees its tensor memory and
returns. The test checks the latched status, then that the process's next
forward passes (on this model and on a second tensor-core model, so tensor
memory is allocated again on every SM) with a clean status word. No GPU fault,
trap or unbounded wait is involved.
"""
import ctypes

import pytest
import torch

from oracle import reference_model as oracle
from ttjam_gottagofast_b200 import UserOptimizedTransformer, _lib, compare_outputs
from ttjam_gottagofast_b200 import generate_random_case
from ttjam_gottagofast_b200.config import TransformerConfig

DEV = "cuda:0"
# Detail codes of the waits that the stalled stage holds up; all start at
# once, so whichever reaches its budget first latches the status: the
# producer's wait for the stage's release (0x1000), the MMA thread's wait for
# its loads (0x2000), the epilogue's wait for the accumulator (0x3000). The
# drain waits (0x1F00, 0x2F00) must never run out.
STALLED_WAITS = (0x1000, 0x2000, 0x3000)


def _model(cfg, seed):
    params = oracle.init_params(cfg, seed=seed, device=DEV)
    model = UserOptimizedTransformer(cfg).to(DEV).eval()
    model.load_state_dict(params, strict=True)
    return model, params


@pytest.mark.gpu
def test_wait_that_runs_out_latches_timeout_and_the_next_forward_is_clean():
    # d_model 256 and 128 tokens: no LayerNorm-prologue GEMM (d > 128) and
    # far too few 256-row pair tiles, so the q|k|v projection runs on the
    # single-CTA kernel (12 CTAs of 128 x 64 tiles, 8 k-blocks, 6 stages)
    cfg = TransformerConfig(2, 64, 256, 4, 256, 1, True)
    model, params = _model(cfg, seed=8)
    lib = model._lib
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 9, 0.3, 1.0)
    x, mask = x.to(DEV), mask.to(DEV)
    ref = oracle.forward(params, cfg, x, mask)
    assert model.forward_plan(2, 64) == "ops_tc"
    with torch.inference_mode():
        y0 = model(x, mask)
    assert model.read_device_status() == (0, 0)
    assert compare_outputs(ref, y0).passed

    assert lib.tt_test_arm_wait_timeout(20) == 0
    with torch.inference_mode():
        model(x, mask)
    code, detail = model.read_device_status()
    assert code == _lib.TT_ERR_DEVICE_TIMEOUT, (code, detail)
    assert detail in STALLED_WAITS, hex(detail)

    # the switch was one-shot; the context and every SM's tensor memory are usable
    for _ in range(3):
        with torch.inference_mode():
            y = model(x, mask)
        res = compare_outputs(ref, y)
        assert res.passed, res
        assert model.read_device_status() == (0, 0)
    other = TransformerConfig(16, 512, 512, 8, 1024, 2, True)
    model2, params2 = _model(other, seed=10)
    x2, m2 = generate_random_case(other, "cpu", torch.float32, 12, 0.5, 1.0)
    x2, m2 = x2.to(DEV), m2.to(DEV)
    with torch.inference_mode():
        y2 = model2(x2, m2)
    idx = torch.tensor([0, 7, 15], device=DEV)
    res = compare_outputs(oracle.forward(params2, other, x2[idx], m2[idx]), y2[idx])
    assert res.passed, res
    assert model2.read_device_status() == (0, 0)


def test_arm_rejects_budgets_out_of_range_without_arming():
    lib = _lib.load()
    for bad in (0, 15, 29, -1):
        assert lib.tt_test_arm_wait_timeout(bad) == _lib.TT_ERR_INVALID_ARGUMENT
    assert "budget_log2" in _lib.last_error(lib)


def test_arm_is_declared_for_the_c_abi():
    import os
    import re
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    text = open(os.path.join(root, "include", "ttjam_b200.h")).read()
    assert re.search(r"int tt_test_arm_wait_timeout\(int budget_log2\);", text)
    assert hasattr(_lib.load(), "tt_test_arm_wait_timeout")
    assert isinstance(ctypes.c_int(0).value, int)
