"""float16 / bfloat16 models and inputs on the GPU (tt_forward_typed).

The reference benchmarks a 16-bit model by moving the model and its input to
that dtype (torch_transformer_benchmark.py:225-231, :698-699). This build
widens the 16-bit weights and input exactly to fp32, runs the fp32-accurate
schedules, and rounds the output once to the dtype. So the anchor for parity
is the fp32 value of the 16-bit model (the reference module run in fp32 on the
same 16-bit weights and input): the output must be that value rounded once,
which passes the contract's gate (abs 2e-3 OR rel 2e-2) with room to spare.
The reference's own 16-bit forward, which rounds after every operation, lands
farther from that value (and outside the gate; see the CPU test of the
goldens): each test checks that this build's output is at least as close.
"""
import pytest
import torch

from conftest import GOLDENS_16BIT, GOLDEN_16BIT_IDS
from oracle import reference_model as oracle
from ttjam_gottagofast_b200 import UserOptimizedTransformer, compare_outputs, generate_random_case
from ttjam_gottagofast_b200.config import WORKLOADS
from ttjam_gottagofast_b200.contract import ATOL, RTOL

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
PLANS = ("cluster", "ops_ffma", "ops_tc", "tile")


@pytest.fixture(autouse=True)
def strict_fp32():
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


def _models(cfg, dtype, seed=1234):
    """(16-bit model, fp32 model of the same widened weights, fp32 params)."""
    p16 = {k: v.to(dtype) for k, v in oracle.init_params(cfg, seed=seed, device=DEV).items()}
    m16 = UserOptimizedTransformer(cfg).to(DEV).eval()
    m16.load_state_dict(p16, strict=True)
    m16 = m16.to(dtype)
    p32 = {k: v.float() for k, v in p16.items()}
    m32 = UserOptimizedTransformer(cfg).to(DEV).eval()
    m32.load_state_dict(p32, strict=True)
    return m16, m32, p32


def _plans(model, b, s):
    import ctypes
    from ttjam_gottagofast_b200 import _lib
    return [p for p in PLANS
            if model._lib.tt_forward_plan(ctypes.byref(_lib.make_config(model.config, p)), b, s) > 0]


def _check_16bit(m16, m32, x16, mask, y_f32, y_ref16, label):
    """For every applicable schedule: y is this build's fp32 forward of the
    widened model and input rounded once to the dtype (bit for bit), passes the
    gate against the fp32 value y_f32, and is at least as close to it as the
    reference's own 16-bit forward y_ref16."""
    ref_err = float((y_ref16.float() - y_f32).abs().max()) if y_ref16 is not None else None
    for plan in _plans(m16, x16.shape[0], x16.shape[1]):
        m16.set_plan(plan)
        m32.set_plan(plan)
        try:
            with torch.inference_mode():
                y = m16(x16, mask)
                y32 = m32(x16.float(), mask)
        finally:
            m16.set_plan("auto")
            m32.set_plan("auto")
        torch.cuda.synchronize()
        assert y.dtype == x16.dtype and y.shape == x16.shape
        assert torch.equal(y, y32.to(x16.dtype)), f"{label}[{plan}]: not the rounded fp32 forward"
        res = compare_outputs(y_f32, y.float(), rtol=RTOL, atol=ATOL)
        err = float((y.float() - y_f32).abs().max())
        print(f"{label}[{plan}]: max_abs vs fp32 value {err:.3e}; reference 16-bit forward "
              f"{ref_err if ref_err is None else f'{ref_err:.3e}'}; gate passed={res.passed}")
        assert res.passed, (label, plan, res)
        if ref_err is not None:
            assert err <= ref_err, (label, plan, err, ref_err)
        if mask is not None:
            assert (y[~mask] == 0).all()
    assert m16.read_device_status() == (0, 0)


@pytest.mark.parametrize("case", GOLDENS_16BIT, ids=GOLDEN_16BIT_IDS)
def test_16bit_golden_parity(case):
    """Against the reference's own outputs: its fp32 value of the 16-bit model
    and its 16-bit forward (both recorded by make_golden_16bit.py)."""
    m16, m32, _ = _models(case.config, case.dtype, case.meta["model_seed"])
    x16 = torch.from_numpy(case.x).to(DEV).to(case.dtype)
    mask = torch.from_numpy(case.mask).to(DEV)
    _check_16bit(m16, m32, x16, mask, torch.from_numpy(case.y_f32).to(DEV),
                 torch.from_numpy(case.y).to(DEV), case.name)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["f16", "bf16"])
@pytest.mark.parametrize("name,variant", [
    ("B1", {}), ("A", {}), ("C", {}), ("A", {"input_scale": 8.0, "padding_ratio": 0.3}),
    ("D", {}), ("D", {"input_scale": 1.0, "padding_ratio": 0.5}),
], ids=["B1", "A", "C", "A_x8_padded", "D", "D_x1_padded"])
def test_16bit_workloads_against_the_oracle(name, variant, dtype):
    """The workloads at full size in float16 and bfloat16 against the oracle
    run on the GPU: in fp32 (TF32 off) for the fp32 value, and in the dtype
    for the reference's own 16-bit forward."""
    w = WORKLOADS[name]
    cfg = w.config
    m16, m32, p32 = _models(cfg, dtype)
    x16, mask = generate_random_case(cfg, "cpu", dtype, 101234,
                                     variant.get("padding_ratio", w.padding_ratio),
                                     variant.get("input_scale", w.input_scale))
    x16, mask = x16.to(DEV), mask.to(DEV)
    y_f32 = oracle.forward(p32, cfg, x16.float(), mask, batch_chunk=4)
    p16 = {k: v.to(dtype) for k, v in p32.items()}
    y_ref16 = oracle.forward(p16, cfg, x16, mask, batch_chunk=4)
    _check_16bit(m16, m32, x16, mask, y_f32, y_ref16, f"{name}{variant}/{dtype}")


def test_16bit_weights_with_fp32_input():
    """The parameters' dtype and the input's are independent: bfloat16 weights
    with a float32 input give a float32 output, equal to the fp32 model of the
    widened weights."""
    cfg = WORKLOADS["C"].config
    m16, m32, _ = _models(cfg, torch.bfloat16)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 7, 0.5, 8.0)
    x, mask = x.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        y = m16(x, mask)
        y32 = m32(x, mask)
    assert y.dtype == torch.float32
    assert torch.equal(y, y32)


def test_16bit_launch_count_and_unaligned_weights():
    """A 16-bit call is two launches more than the fp32 one (the widening of x
    and the rounding of y), both visible to the launch probe; weights that
    live at odd offsets of one flat buffer pack like aligned ones."""
    import ctypes
    cfg = WORKLOADS["B1"].config
    m16, m32, p32 = _models(cfg, torch.float16)
    x16, mask = generate_random_case(cfg, "cpu", torch.float16, 3, 0.0, 1.0)
    x16, mask = x16.to(DEV), mask.to(DEV)
    lib = m16._lib
    with torch.inference_mode():
        y_ref = m16(x16, mask)
        torch.cuda.synchronize()
        assert lib.tt_launch_probe_start(64) == 0
        try:
            y = m16(x16, mask)
            torch.cuda.synchronize()
            ms = (ctypes.c_float * 64)()
            kinds = (ctypes.c_int32 * 64)()
            n = lib.tt_launch_probe_read(ms, kinds, 64)
        finally:
            lib.tt_launch_probe_start(0)
    fp32_launches = lib.tt_forward_launch_count(ctypes.byref(m16._cfg), *x16.shape[:2])
    assert n == fp32_launches + 2
    assert list(kinds)[0] == 10 and list(kinds)[n - 1] == 10
    assert torch.equal(y, y_ref)
    # the same weights at 2-byte offsets inside one flat fp16 buffer
    sd = m16.state_dict()
    total = sum(v.numel() + 1 for v in sd.values())
    flat = torch.empty(total, dtype=torch.float16, device=DEV)
    views, off = {}, 1
    for k, v in sd.items():
        views[k] = flat[off:off + v.numel()].view(v.shape)
        views[k].copy_(v)
        off += v.numel() + 1
    m_odd = UserOptimizedTransformer(cfg).to(DEV).eval().to(torch.float16)
    for name, prm in m_odd.named_parameters():
        prm.data = views[name]
    m_odd.invalidate()
    assert any(p.data_ptr() % 16 for p in m_odd.parameters())
    with torch.inference_mode():
        y_odd = m_odd(x16, mask)
    assert torch.equal(y_odd, y_ref)


def test_16bit_calls_replayed_from_the_graph_cache():
    """The same 16-bit call twice with the same buffers: the second replays the
    cached CUDA graph of the per-op schedule (on the fp32 copies in the
    workspace) between the two conversion kernels; same bits, and new inputs
    in the same buffers give the new forward."""
    import ctypes
    from ttjam_gottagofast_b200 import _lib
    cfg = WORKLOADS["C"].config
    m16, m32, _ = _models(cfg, torch.bfloat16)
    lib = m16._lib
    x1, mask = generate_random_case(cfg, "cpu", torch.bfloat16, 21, 0.5, 8.0)
    x2, _ = generate_random_case(cfg, "cpu", torch.bfloat16, 22, 0.5, 8.0)
    x1, x2, mask = x1.to(DEV), x2.to(DEV), mask.to(DEV)
    image = m16._ensure_image(torch.device(DEV))
    c = m16._cfg
    b, s = x1.shape[:2]
    nbytes = lib.tt_typed_workspace_bytes(ctypes.byref(c), _lib.TT_DTYPE_BF16, b, s)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    xbuf = x1.clone()
    y = torch.empty_like(x1)
    outs = []
    stream = torch.cuda.current_stream().cuda_stream
    for xin in (x1, x1, x2):
        xbuf.copy_(xin)
        rc = lib.tt_forward_typed(ctypes.byref(c), image.data_ptr(), _lib.TT_DTYPE_BF16,
                                  xbuf.data_ptr(), mask.data_ptr(), b, s, y.data_ptr(),
                                  ws.data_ptr(), nbytes, stream)
        _lib.check(rc, "tt_forward_typed", lib)
        torch.cuda.synchronize()
        outs.append(y.clone())
    assert m16.forward_plan(b, s) == "ops_tc"
    assert torch.equal(outs[0], outs[1])
    with torch.inference_mode():
        ref2 = m32(x2.float(), mask).to(torch.bfloat16)
    assert torch.equal(outs[2], ref2)
    assert not torch.equal(outs[2], outs[0])
