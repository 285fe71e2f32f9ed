"""tt_forward_host: one forward step from and to host buffers in one call.

The call copies x and the mask into its workspace, runs tt_forward's schedule
and copies y back, all on the caller's stream. The output must be bit for bit
tt_forward's on device copies of the same inputs (the same kernels run on the
same values), on every kind of schedule."""
import ctypes

import pytest
import torch

from oracle import reference_model as oracle
from ttjam_gottagofast_b200 import UserOptimizedTransformer, _lib, generate_random_case
from ttjam_gottagofast_b200.config import OFFICIAL, WORKLOADS

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _model(cfg):
    m = UserOptimizedTransformer(cfg).to(DEV).eval()
    m.load_state_dict(oracle.init_params(cfg, seed=1234, device=DEV), strict=True)
    return m


def _host_call(model, xh, mh, yh):
    lib = model._lib
    b, s = xh.shape[:2]
    cfg = model._cfg
    image = model._ensure_image(torch.device(DEV))
    nbytes = lib.tt_host_workspace_bytes(ctypes.byref(cfg), b, s)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.tt_forward_host(ctypes.byref(cfg), image.data_ptr(), xh.data_ptr(),
                             None if mh is None else mh.data_ptr(), b, s, yh.data_ptr(),
                             ws.data_ptr(), nbytes, stream)
    _lib.check(rc, "tt_forward_host", lib)
    torch.cuda.current_stream().synchronize()


@pytest.mark.parametrize("name,plan,pad,use_mask,pinned", [
    ("B1", "auto", 0.0, True, True),       # cluster schedule
    ("B2", "auto", 0.0, False, True),      # cluster schedule, no mask
    ("A", "tile", 0.3, True, True),        # tile schedule, forced
    ("case1", "auto", 0.5, True, True),    # tile schedule by default (8192 rows)
    ("C", "auto", 0.5, True, True),        # per-op tensor-core schedule
    ("C", "ops_ffma", 0.5, True, False),   # per-op FFMA schedule, pageable buffers
])
def test_host_forward_matches_device_forward(name, plan, pad, use_mask, pinned):
    w = OFFICIAL[name] if name.startswith("case") else WORKLOADS[name]
    cfg = w.config
    model = _model(cfg)
    model.set_plan(plan)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 5, pad, 2.0)
    xh, mh = (x.pin_memory(), mask.pin_memory()) if pinned else (x, mask)
    if not use_mask:
        mh = None
    yh = torch.full_like(xh, float("nan"))
    if pinned:
        yh = yh.pin_memory()
    _host_call(model, xh, mh, yh)
    with torch.inference_mode():
        y = model(x.to(DEV), None if mh is None else mask.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(yh, y.cpu()), name
    # and through the module's host-buffer call, twice (buffers reused)
    out = torch.empty_like(xh)
    if pinned:
        out = out.pin_memory()
    for _ in range(2):
        with torch.inference_mode():
            model.forward_host(xh, mh, out=out, slices=1)
        torch.cuda.synchronize()
        assert torch.equal(out, y.cpu())
    assert model.read_device_status() == (0, 0)


def test_host_step_keeps_inputs_alive_until_copied():
    """A temporary pinned input dropped right after the call still reaches the
    device intact: the module holds it until its stream has passed the copy."""
    cfg = WORKLOADS["B1"].config
    model = _model(cfg)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 9, 0.0, 1.0)
    with torch.inference_mode():
        ref = model(x.to(DEV), mask.to(DEV)).cpu()
    outs = []
    for _ in range(8):
        out = torch.empty_like(x).pin_memory()
        model.forward_host(x.clone().pin_memory(), mask.clone().pin_memory(), out=out)
        # fresh pinned blocks of the same size, written at once
        junk = [torch.full_like(x, 1e30).pin_memory() for _ in range(2)]
        outs.append(out)
        del junk
    torch.cuda.synchronize()
    for out in outs:
        assert torch.equal(out, ref)


def test_small_host_steps_copy_with_kernels():
    """x up to 1 MiB in page-locked buffers: the copies are small kernels
    (TT_KERNEL_CONVERT in the launch probe) around the forward's own launch;
    pageable buffers take DMA copies (no such launches). Same bits either way."""
    cfg = WORKLOADS["B1"].config
    model = _model(cfg)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 12, 0.5, 1.0)
    assert not bool(mask.all())
    lib = model._lib
    with torch.inference_mode():
        ref = model(x.to(DEV), mask.to(DEV)).cpu()

    def kinds_of(xh, mh, yh):
        torch.cuda.synchronize()
        assert lib.tt_launch_probe_start(16) == 0
        try:
            _host_call(model, xh, mh, yh)
            ms = (ctypes.c_float * 16)()
            kinds = (ctypes.c_int32 * 16)()
            n = lib.tt_launch_probe_read(ms, kinds, 16)
        finally:
            lib.tt_launch_probe_start(0)
        return list(kinds)[:n]

    yh = torch.empty_like(x).pin_memory()
    # x and the mask in, the forward, y out
    assert kinds_of(x.pin_memory(), mask.pin_memory(), yh) == [10, 10, 8, 10]
    assert torch.equal(yh, ref)
    y2 = torch.empty_like(x)
    assert kinds_of(x, mask, y2) == [8]
    assert torch.equal(y2, ref)
