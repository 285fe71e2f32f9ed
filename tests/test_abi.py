"""The C ABI library: loads, exports every declared symbol, validates without a GPU."""
import ctypes
import os
import re

import pytest

from ttjam_gottagofast_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    inc = os.path.join(ROOT, "include")
    for fn in os.listdir(inc):
        if fn.endswith(".h"):
            text = open(os.path.join(inc, fn)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names |= set(re.findall(r"\b(tt_[a-z_0-9]+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def lib():
    return _lib.load()


def test_library_is_sm100a_build_in_tree(lib):
    assert os.path.dirname(_lib.lib_path()).endswith("ttjam_gottagofast_b200")
    assert lib.tt_abi_version() == _lib.TT_ABI_VERSION


def test_every_declared_symbol_is_exported(lib):
    decl = declared_symbols()
    assert decl, "no declarations parsed"
    assert decl <= set(_lib.EXPORTED) | decl
    for name in decl:
        assert hasattr(lib, name), name


def _cfg(d=128, h=4, f=128, l=4, causal=1, plan="auto"):
    c = _lib.TTConfig()
    c.d_model, c.num_heads, c.ffn_dim, c.num_layers, c.causal = d, h, f, l, causal
    c.plan = _lib.PLAN_IDS[plan]
    return c


def _ops_cfg():
    """The d128 model forced onto a per-op schedule: its calls check their
    workspace before anything is launched, with or without a GPU (the automatic
    plan may pick a single-launch schedule, which takes no workspace)."""
    return _cfg(plan="ops_ffma")


def test_validate_config_codes(lib):
    assert lib.tt_validate_config(ctypes.byref(_cfg())) == 0
    assert lib.tt_validate_config(ctypes.byref(_cfg(h=3))) == _lib.TT_ERR_INVALID_CONFIG
    assert "divisible" in _lib.last_error(lib)
    assert lib.tt_validate_config(ctypes.byref(_cfg(l=0))) == _lib.TT_ERR_INVALID_CONFIG
    assert lib.tt_validate_config(ctypes.byref(_cfg(d=1024, h=2))) == _lib.TT_ERR_UNSUPPORTED
    assert lib.tt_validate_config(None) == _lib.TT_ERR_INVALID_ARGUMENT
    bad = _cfg()
    bad.plan = 9
    assert lib.tt_validate_config(ctypes.byref(bad)) == _lib.TT_ERR_INVALID_CONFIG
    bad = _cfg()
    bad.reserved = 1
    assert lib.tt_validate_config(ctypes.byref(bad)) == _lib.TT_ERR_INVALID_CONFIG
    bad = _cfg()
    bad.flags = 2
    assert lib.tt_validate_config(ctypes.byref(bad)) == _lib.TT_ERR_INVALID_CONFIG
    ok = _cfg()
    ok.flags = _lib.TT_FLAG_FP32_ONLY
    assert lib.tt_validate_config(ctypes.byref(ok)) == 0


def test_image_and_workspace_sizes(lib):
    c = _cfg()
    n = lib.tt_image_bytes(ctypes.byref(c))
    per_layer = (4 * 128 * 128 + 2 * 128 * 128) * 4
    # fp32 weights plus their fp16 hi/lo split (same bytes again) for the
    # tensor-core schedule
    assert 2 * 4 * per_layer < n < 2 * 4 * per_layer + 64 * 1024
    odd = _cfg(d=30, h=3, f=30)   # no split when fp16 rows are not 16-byte multiples
    assert lib.tt_image_bytes(ctypes.byref(odd)) < 2 * 4 * (4 * 30 * 30 + 2 * 30 * 30) * 4
    ws = lib.tt_workspace_bytes(ctypes.byref(_ops_cfg()), 4, 24)
    assert ws >= 96 * (3 * 128 + 128 + 128) * 4
    assert lib.tt_image_bytes(ctypes.byref(_cfg(h=3))) == 0


def test_forward_argument_errors_need_no_gpu(lib):
    c = _ops_cfg()
    rc = lib.tt_forward(ctypes.byref(c), None, None, None, 4, 16, None, None, 0, None)
    assert rc == _lib.TT_ERR_INVALID_ARGUMENT
    # sizes are checked before anything is launched
    rc = lib.tt_forward(ctypes.byref(c), 256, 512, None, 4, 24, 1024, 2048, 16, None)
    assert rc == _lib.TT_ERR_WORKSPACE
    assert "workspace" in _lib.last_error(lib)
    rc = lib.tt_forward(ctypes.byref(c), 256, 512, None, -1, 16, 1024, 2048, 16, None)
    assert rc == _lib.TT_ERR_INVALID_ARGUMENT
    # empty batch is a no-op
    assert lib.tt_forward(ctypes.byref(c), None, None, None, 0, 16, None, None, 0, None) == 0


def test_pack_argument_errors_need_no_gpu(lib):
    c = _cfg()
    rc = lib.tt_pack_image(ctypes.byref(c), None, None, None, None, 0, None)
    assert rc == _lib.TT_ERR_INVALID_ARGUMENT


def test_forward_plan(lib):
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(_cfg(d=512, h=8, f=2048, l=6)),
                                               16, 1024)]
    forced = _cfg()
    forced.plan = _lib.PLAN_IDS["ops_ffma"]
    assert lib.tt_forward_plan(ctypes.byref(forced), 4, 16) == 2
    assert lib.tt_forward_launch_count(ctypes.byref(forced), 4, 16) == 5 * 4 + 1
    # the cluster schedule never applies at d_model 512
    big = _cfg(d=512, h=8, f=2048, l=6)
    big.plan = _lib.PLAN_IDS["cluster"]
    assert lib.tt_forward_plan(ctypes.byref(big), 4, 16) == _lib.TT_ERR_UNSUPPORTED


def test_fp32_only_flag_keeps_auto_plan_off_the_split_schedule(lib):
    d_cfg = _cfg(d=512, h=8, f=2048, l=6)
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(d_cfg), 16, 1024)] == "ops_tc"
    d_cfg.flags = _lib.TT_FLAG_FP32_ONLY
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(d_cfg), 16, 1024)] == "ops_ffma"
    forced = _cfg(d=512, h=8, f=2048, l=6)
    forced.plan = _lib.PLAN_IDS["ops_ffma"]
    # the workspace is the FFMA schedule's
    assert (lib.tt_workspace_bytes(ctypes.byref(d_cfg), 16, 1024) ==
            lib.tt_workspace_bytes(ctypes.byref(forced), 16, 1024))
    assert lib.tt_forward_launch_count(ctypes.byref(d_cfg), 16, 1024) == 5 * 6 + 1
    # a forced split schedule stays forced
    d_cfg.plan = _lib.PLAN_IDS["ops_tc"]
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(d_cfg), 16, 1024)] == "ops_tc"


def test_tile_plan_takes_batches_of_short_sequences_of_the_d128_model(lib):
    # d_model = ffn_dim = 128, 4 heads, seq dividing 128, at least one tile of
    # 128 rows (official case 1: batch 64 x 128; workload A: batch 8 x 128)
    a = _cfg()
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(a), 64, 128)] == "tile"
    assert lib.tt_forward_launch_count(ctypes.byref(a), 64, 128) == 1
    assert lib.tt_workspace_bytes(ctypes.byref(a), 64, 128) == 0
    # (seq 128: never the cluster schedule, which takes short sequences on a GPU)
    for b, s in ((1, 128), (8, 128), (16, 128), (10000, 128), (4, 32)):
        assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(a), b, s)] == "tile"
    # fewer rows than a tile (without a GPU, where the cluster schedule is not
    # offered), seq not a divisor of 128, or another head count: the per-op
    # schedule
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(a), 4, 16)] == "ops_tc"
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(a), 32, 512)] == "ops_tc"
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(a), 100, 24)] == "ops_tc"
    h2 = _cfg(h=2)
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(h2), 64, 128)] == "ops_tc"
    # fp16 pieces: never under TT_FLAG_FP32_ONLY unless forced; forced, any
    # number of rows
    a.flags = _lib.TT_FLAG_FP32_ONLY
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(a), 64, 128)] == "ops_ffma"
    a.plan = _lib.PLAN_IDS["tile"]
    assert _lib.PLAN_NAMES[lib.tt_forward_plan(ctypes.byref(a), 8, 128)] == "tile"
    assert lib.tt_forward_launch_count(ctypes.byref(a), 8, 128) == 1
    assert lib.tt_forward_plan(ctypes.byref(a), 32, 512) == _lib.TT_ERR_UNSUPPORTED
    assert lib.tt_forward_plan(ctypes.byref(h2), 64, 128) > 0
    h2.plan = _lib.PLAN_IDS["tile"]
    assert lib.tt_forward_plan(ctypes.byref(h2), 64, 128) == _lib.TT_ERR_UNSUPPORTED
    bad = _cfg()
    bad.plan = 5
    assert lib.tt_validate_config(ctypes.byref(bad)) == _lib.TT_ERR_INVALID_CONFIG


def test_fp16_operand_bound_argument_errors_need_no_gpu(lib):
    b = ctypes.c_float(0)
    assert lib.tt_fp16_operand_bound(ctypes.byref(_cfg()), None, ctypes.byref(b),
                                     None) == _lib.TT_ERR_INVALID_ARGUMENT
    assert lib.tt_fp16_operand_bound(ctypes.byref(_cfg()), 256, None,
                                     None) == _lib.TT_ERR_INVALID_ARGUMENT


def test_launch_count_includes_the_row_scan_of_gemm_heavy_shapes(lib):
    e = _cfg(d=1024, h=16, f=4096, l=12)
    # 7 launches per layer, the final LayerNorm, and the live-row scan
    assert lib.tt_forward_launch_count(ctypes.byref(e), 64, 2048) == 7 * 12 + 1 + 1
    # fewer than 1024 rows: no scan
    small = _cfg(d=1024, h=16, f=4096, l=12)
    assert lib.tt_forward_launch_count(ctypes.byref(small), 1, 512) == 7 * 12 + 1
    # the d128 model: its GEMMs are latency-bound, no scan (workload C; workload
    # A, whose LayerNorm-prologue GEMMs take 5 launches per layer)
    d128 = _cfg()
    d128.plan = _lib.PLAN_IDS["ops_tc"]
    assert lib.tt_forward_launch_count(ctypes.byref(d128), 32, 512) == 7 * 4 + 1
    assert lib.tt_forward_launch_count(ctypes.byref(d128), 8, 128) == 5 * 4 + 1


def test_typed_entry_points_need_no_gpu_for_their_checks(lib):
    """The 16-bit entry points: workspace sizes (fp32 copies of x and y ahead
    of the schedule's own scratch) and argument checks before any launch."""
    c = _ops_cfg()
    b, s = 4, 24
    base = lib.tt_workspace_bytes(ctypes.byref(c), b, s)
    assert lib.tt_typed_workspace_bytes(ctypes.byref(c), _lib.TT_DTYPE_F32, b, s) == base
    io = (b * s * 128 * 4 + 255) // 256 * 256
    for dt in (_lib.TT_DTYPE_F16, _lib.TT_DTYPE_BF16):
        assert lib.tt_typed_workspace_bytes(ctypes.byref(c), dt, b, s) == 2 * io + base
    assert lib.tt_typed_workspace_bytes(ctypes.byref(c), 7, b, s) == 0
    # whatever the schedule (a single-launch one needs no scratch of its own),
    # the fp32 copies come first
    assert lib.tt_typed_workspace_bytes(ctypes.byref(c), _lib.TT_DTYPE_BF16, 4, 16) == \
        2 * ((4 * 16 * 128 * 4 + 255) // 256 * 256) + lib.tt_workspace_bytes(ctypes.byref(c), 4, 16)
    rc = lib.tt_forward_typed(ctypes.byref(c), 256, 7, 512, None, b, s, 1024, 2048, 1 << 30, None)
    assert rc == _lib.TT_ERR_INVALID_ARGUMENT and "dtype" in _lib.last_error(lib)
    rc = lib.tt_forward_typed(ctypes.byref(c), 256, _lib.TT_DTYPE_F16, 512, None, b, s, 1024,
                              2048, 16, None)
    assert rc == _lib.TT_ERR_WORKSPACE and "tt_typed_workspace_bytes" in _lib.last_error(lib)
    rc = lib.tt_forward_typed(ctypes.byref(c), 256, _lib.TT_DTYPE_BF16, 512, None, b, s, 1024,
                              None, 1 << 30, None)
    assert rc == _lib.TT_ERR_INVALID_ARGUMENT
    rc = lib.tt_forward_typed(ctypes.byref(c), 256, _lib.TT_DTYPE_BF16, 520, None, b, s, 1024,
                              2048, 1 << 30, None)
    assert rc == _lib.TT_ERR_INVALID_ARGUMENT and "aligned" in _lib.last_error(lib)
    assert lib.tt_forward_typed(ctypes.byref(c), None, _lib.TT_DTYPE_F16, None, None, 0, s,
                                None, None, 0, None) == 0
    rc = lib.tt_pack_image_typed(ctypes.byref(c), 5, None, None, None, None, 0, None)
    assert rc == _lib.TT_ERR_INVALID_ARGUMENT and "dtype" in _lib.last_error(lib)
    rc = lib.tt_pack_image_typed(ctypes.byref(c), _lib.TT_DTYPE_BF16, None, None, None, None, 0,
                                 None)
    assert rc == _lib.TT_ERR_INVALID_ARGUMENT


def test_host_entry_point_checks_need_no_gpu(lib):
    """tt_forward_host: device room for x, y and the mask ahead of the
    schedule's own scratch, and the checks made before anything is enqueued."""
    c = _ops_cfg()
    b, s = 4, 24
    base = lib.tt_workspace_bytes(ctypes.byref(c), b, s)
    io = (b * s * 128 * 4 + 255) // 256 * 256
    assert lib.tt_host_workspace_bytes(ctypes.byref(c), b, s) == 2 * io + 256 + base
    assert lib.tt_forward_host(ctypes.byref(c), None, None, None, b, s, None, None, 0, None) == \
        _lib.TT_ERR_INVALID_ARGUMENT
    assert lib.tt_forward_host(ctypes.byref(c), None, None, None, 0, s, None, None, 0, None) == 0
    rc = lib.tt_forward_host(ctypes.byref(c), 256, 4096, None, b, s, 8192, 2048, 16, None)
    assert rc == _lib.TT_ERR_WORKSPACE and "tt_host_workspace_bytes" in _lib.last_error(lib)
    rc = lib.tt_forward_host(ctypes.byref(c), 256, 4096, None, b, s, 8192, 2056, 1 << 30, None)
    assert rc == _lib.TT_ERR_INVALID_ARGUMENT and "aligned" in _lib.last_error(lib)
