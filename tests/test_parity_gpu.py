"""Parity of the CUDA forward (through the C ABI) against the reference.

Two anchors:
* the golden fixtures, produced by the reference module itself on CPU;
* the oracle restatement run on the same device in strict fp32 (TF32 off) at
  the full sizes of every workload, sequence-sliced where the reference's
  [B,H,S,S] tensor would be large.

Tolerance: the reference's accuracy gate, element-wise
abs(opt - ref) <= 0.002 OR abs(opt - ref) <= 0.02 * abs(ref), all finite
(torch_transformer_benchmark.py:309-316, defaults :618-619).
"""
import pytest
import torch

from conftest import GOLDENS, GOLDEN_IDS
from oracle import reference_model as oracle
from ttjam_gottagofast_b200 import UserOptimizedTransformer, compare_outputs, generate_random_case
from ttjam_gottagofast_b200.config import WORKLOADS
from ttjam_gottagofast_b200.contract import ATOL, HARNESS_VARIANTS, RTOL

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(autouse=True)
def strict_fp32():
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old


_MODELS = {}


def model_for(cfg, seed=1234):
    key = (cfg.d_model, cfg.num_heads, cfg.ffn_dim, cfg.num_layers, cfg.causal, seed)
    if key not in _MODELS:
        if len(_MODELS) > 3:
            _MODELS.clear()
        params = oracle.init_params(cfg, seed=seed, device=DEV)
        model = UserOptimizedTransformer(cfg).to(DEV).eval()
        model.load_state_dict(params, strict=True)
        _MODELS[key] = (model, params)
    return _MODELS[key]


def applicable_plans(model, b, s):
    """Every kernel schedule that can run [b, s] for this model."""
    import ctypes
    from ttjam_gottagofast_b200 import _lib
    out = []
    for name in ("cluster", "ops_ffma", "ops_tc", "tile"):
        cfg = _lib.make_config(model.config, name)
        if model._lib.tt_forward_plan(ctypes.byref(cfg), b, s) > 0:
            out.append(name)
    return out


def run_plans(model, x, mask):
    """{plan: output} for every applicable schedule, then back to "auto"."""
    outs = {}
    try:
        for plan in applicable_plans(model, x.shape[0], x.shape[1]):
            model.set_plan(plan)
            with torch.inference_mode():
                outs[plan] = model(x, mask)
    finally:
        model.set_plan("auto")
    assert outs
    return outs


def check(ref, out, label):
    res = compare_outputs(ref, out, rtol=RTOL, atol=ATOL)
    print(f"{label}: max_abs={res.max_abs_error:.3e} max_rel={res.max_relative_error:.3e} "
          f"failed={res.failed_elements}/{res.total_elements}")
    assert res.passed, (label, res)
    return res


@pytest.mark.parametrize("case", GOLDENS, ids=GOLDEN_IDS)
def test_golden_parity(case):
    model, _ = model_for(case.config, case.meta["model_seed"])
    x = torch.from_numpy(case.x).to(DEV)
    mask = torch.from_numpy(case.mask).to(DEV) if case.uses_mask else None
    for plan, y in run_plans(model, x, mask).items():
        torch.cuda.synchronize()
        check(torch.from_numpy(case.y), y.cpu(), f"{case.name}[{plan}]")
        if mask is not None:
            assert (y[~mask] == 0).all(), "padded rows must be exactly zero"
    assert model.read_device_status() == (0, 0)


def _full_size_case(name, variant):
    w = WORKLOADS[name]
    cfg = w.config
    model, params = model_for(cfg)
    seed = variant.get("seed", 101234)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, seed,
                                   variant.get("padding_ratio", w.padding_ratio),
                                   variant.get("input_scale", w.input_scale))
    x, mask = x.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        y = model(x, mask)
    return cfg, params, x, mask, y


def test_small_shapes_run_in_one_launch():
    """The launch-bound workloads take a single-launch schedule: the cluster
    forward for B1 and B2, the tile forward for the reference's official case
    1 (batch 64 x 128 of the d128 model)."""
    import ctypes
    from ttjam_gottagofast_b200.config import OFFICIAL
    for w, plan in ((WORKLOADS["B1"], "cluster"), (WORKLOADS["B2"], "cluster"),
                    (OFFICIAL["case1"], "tile")):
        cfg = w.config
        model, _ = model_for(cfg)
        assert model.forward_plan(cfg.batch_size, cfg.seq_len) == plan
        assert model._lib.tt_forward_launch_count(ctypes.byref(model._cfg), cfg.batch_size,
                                                  cfg.seq_len) == 1


# Shapes of the tile forward the goldens do not reach: masks with holes,
# non-causal sequences longer than one token, a partial last tile (rows not a
# multiple of 128), one layer, and each input scale of the harness.
TILE_CASES = [
    # batch, seq, causal, layers, padding ratio, input scale, holes
    (3, 32, 1, 2, 0.5, 1.0, True),
    (3, 64, 0, 2, 0.5, 1.0, False),
    (5, 16, 0, 1, 0.0, 1.0, True),
    (3, 128, 1, 1, 0.4, 8.0, False),
    (7, 64, 1, 3, 0.3, 0.05, False),
    (2, 2, 1, 2, 0.0, 1.0, False),
    (33, 128, 1, 4, 0.5, 1.0, True),
]


@pytest.mark.parametrize("variant", HARNESS_VARIANTS, ids=[v["name"] for v in HARNESS_VARIANTS])
def test_tile_forward_workload_A_variants(variant):
    """Workload A (batch 8 x 128, which the default picks the per-op schedule
    for) forced onto the tile forward, at each harness input variant."""
    w = WORKLOADS["A"]
    cfg = w.config
    model, params = model_for(cfg)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, variant.get("seed", 101234),
                                   variant.get("padding_ratio", w.padding_ratio),
                                   variant.get("input_scale", w.input_scale))
    x, mask = x.to(DEV), mask.to(DEV)
    model.set_plan("tile")
    try:
        with torch.inference_mode():
            y = model(x, mask)
    finally:
        model.set_plan("auto")
    ref = oracle.forward(params, cfg, x, mask)
    check(ref, y, f"A[tile]/{variant['name']}")
    assert (y[~mask] == 0).all()
    assert model.read_device_status() == (0, 0)


@pytest.mark.parametrize("case", TILE_CASES, ids=[f"b{c[0]}_s{c[1]}_c{c[2]}_l{c[3]}"
                                                  f"_x{c[5]}{'_holes' if c[6] else ''}"
                                                  for c in TILE_CASES])
def test_tile_forward_matches_oracle(case):
    from ttjam_gottagofast_b200.config import TransformerConfig
    b, s, causal, layers, pad, scale, holes = case
    cfg = TransformerConfig(b, s, 128, 4, 128, layers, bool(causal))
    model, params = model_for(cfg, seed=777)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 4242 + b * s, pad, scale)
    if holes:
        g = torch.Generator().manual_seed(b * 1000 + s)
        mask = mask & (torch.rand(b, s, generator=g) > 0.25)
        mask[:, 0] = True
    x, mask = x.to(DEV), mask.to(DEV)
    model.set_plan("tile")
    try:
        assert model.forward_plan(b, s) == "tile"
        with torch.inference_mode():
            y = model(x, mask)
            y2 = model(x, mask)
    finally:
        model.set_plan("auto")
    ref = oracle.forward(params, cfg, x, mask)
    check(ref, y, f"tile b{b} s{s} causal{causal} L{layers} x{scale}")
    assert (y[~mask] == 0).all(), "padded rows must be exactly zero"
    assert torch.equal(y, y2), "the tile forward is deterministic"
    assert model.read_device_status() == (0, 0)


SMALL_WORKLOAD_CASES = [(n, v) for n in ("A", "B1", "B2", "C")
                        for v in [{"name": "own"}] + HARNESS_VARIANTS]


@pytest.mark.parametrize("name,variant", SMALL_WORKLOAD_CASES,
                         ids=[f"{n}-{v['name']}" for n, v in SMALL_WORKLOAD_CASES])
def test_workload_parity_full_size(name, variant):
    cfg, params, x, mask, y = _full_size_case(name, variant)
    ref = oracle.forward(params, cfg, x, mask, batch_chunk=8)
    model, _ = model_for(cfg)
    for plan, out in run_plans(model, x, mask).items():
        check(ref, out, f"{name}/{variant['name']}[{plan}]")


D_E_VARIANTS = [{"name": "own"}] + HARNESS_VARIANTS


@pytest.mark.parametrize("variant", D_E_VARIANTS, ids=[v["name"] for v in D_E_VARIANTS])
def test_workload_D_parity_full_size(variant):
    """D (d512 h8 ffn2048 L6, batch 16 x 1024) at full size, every sequence,
    at its own x0.05 inputs and at each harness variant (x1, x8, x0.05,
    padded, heavily padded)."""
    cfg, params, x, mask, y = _full_size_case("D", variant)
    ref = oracle.forward(params, cfg, x, mask, batch_chunk=2)
    check(ref, y, f"D/{variant['name']}")
    assert (y[~mask] == 0).all()
    model, _ = model_for(cfg)
    assert model.forward_plan(cfg.batch_size, cfg.seq_len) == "ops_tc"
    assert model.read_device_status() == (0, 0)


@pytest.mark.parametrize("variant", D_E_VARIANTS, ids=[v["name"] for v in D_E_VARIANTS])
def test_workload_E_parity_sequence_sample(variant):
    """Full-size E forward (d1024 h16 ffn4096 L12, batch 64 x 2048) at its own
    inputs and at each harness variant; the oracle checks 8 sequences per
    variant -- the shortest, the longest and six spread over the batch
    (sequences are independent)."""
    cfg, params, x, mask, y = _full_size_case("E", variant)
    lengths = mask.sum(1)
    picks = {int(lengths.argmin()), int(lengths.argmax())}
    for i in range(0, cfg.batch_size, cfg.batch_size // 8):
        if len(picks) >= 8:
            break
        picks.add(i + 3)
    picks = sorted(picks)
    assert len(picks) == 8
    idx = torch.tensor(picks, device=DEV)
    ref = oracle.forward(params, cfg, x[idx], mask[idx], batch_chunk=1)
    check(ref, y[idx], f"E/{variant['name']}/seqs{picks}")
    assert torch.isfinite(y).all()
    assert (y[~mask] == 0).all()
    model, _ = model_for(cfg)
    assert model.forward_plan(cfg.batch_size, cfg.seq_len) == "ops_tc"
    assert model.read_device_status() == (0, 0)


def _lengths_mask(b, s, lengths):
    m = torch.zeros(b, s, dtype=torch.bool)
    for i, n in enumerate(lengths):
        m[i, :n] = True
    return m


@pytest.mark.parametrize("seq,kind", [(300, "prefix"), (512, "prefix"), (1000, "prefix"),
                                      (512, "holes"), (384, "none")])
def test_dead_row_tiles_are_skipped_safely(seq, kind):
    """GEMM-heavy shapes skip the 128-row tiles of the batch that hold only
    rows past each sequence's last valid key (rounded up to 64). Sequence
    lengths here include 0 (all padding), 1, odd lengths and full ones; a
    sequence length that is not a multiple of 64 or 256 puts sequence
    boundaries inside tiles; a mask with holes skips only its trailing part.
    Every schedule matches the oracle and padded rows are exactly 0."""
    from ttjam_gottagofast_b200.config import TransformerConfig
    b = 6
    cfg = TransformerConfig(batch_size=b, seq_len=seq, d_model=256, num_heads=4, ffn_dim=512,
                            num_layers=2, causal=True)
    model, params = model_for(cfg, seed=77)
    g = torch.Generator().manual_seed(seq)
    x = torch.randn(b, seq, 256, generator=g)
    if kind == "none":
        mask = None
    elif kind == "prefix":
        lengths = [0, 1, seq, seq // 3 + 1, seq - 63, 2 * seq // 3 - 5]
        mask = _lengths_mask(b, seq, lengths)
    else:
        mask = _lengths_mask(b, seq, [seq, seq // 2, 300, 5, seq, 257])
        mask[0, 100:300] = False   # a hole wider than a 256-row tile
        mask[4, 10:20] = False
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
        mask = mask.to(DEV)
    x = x.to(DEV)
    ref = oracle.forward(params, cfg, x, mask)
    for plan, y in run_plans(model, x, mask).items():
        check(ref, y, f"dead rows s{seq} {kind}[{plan}]")
        assert torch.isfinite(y).all()
        if mask is not None:
            assert (y[~mask] == 0).all()
    assert model.read_device_status() == (0, 0)


@pytest.mark.parametrize("seq", [512, 200])
def test_dead_row_tiles_on_the_cta_pair_gemm(seq):
    """A batch large enough for the CTA-pair GEMM, whose two CTAs take two
    live 128-row tiles of the list (adjacent or not): random lengths from 0 to
    seq, so live tiles come in odd numbers and one CTA of the last pair gets
    rows past the matrix."""
    from ttjam_gottagofast_b200.config import TransformerConfig
    b = 96 if seq == 200 else 48
    cfg = TransformerConfig(batch_size=b, seq_len=seq, d_model=256, num_heads=4, ffn_dim=512,
                            num_layers=2, causal=True)
    model, params = model_for(cfg, seed=78)
    g = torch.Generator().manual_seed(1000 + seq)
    x = torch.randn(b, seq, 256, generator=g)
    lengths = torch.randint(0, seq + 1, (b,), generator=g).tolist()
    lengths[0], lengths[1] = 0, seq
    mask = _lengths_mask(b, seq, lengths)
    x = x.masked_fill(~mask[..., None], 0).to(DEV)
    mask = mask.to(DEV)
    with torch.inference_mode():
        y = model(x, mask)
    picks = [0, 1, 2, b // 2, b - 1]
    idx = torch.tensor(picks, device=DEV)
    ref = oracle.forward(params, cfg, x[idx], mask[idx])
    check(ref, y[idx], f"dead rows on the pair GEMM s{seq}/seqs{picks}")
    assert torch.isfinite(y).all()
    assert (y[~mask] == 0).all()
    assert model.read_device_status() == (0, 0)


def _inflated_v_model(plan="auto"):
    """A d256 model (a tensor-core shape) whose v_proj weights are scaled by
    1e5: its v values and attention contexts reach ~1e5-1e6, beyond the
    largest fp16 value, while every fp32 intermediate stays finite."""
    from ttjam_gottagofast_b200.config import TransformerConfig
    cfg = TransformerConfig(batch_size=3, seq_len=96, d_model=256, num_heads=4, ffn_dim=256,
                            num_layers=2, causal=True)
    params = dict(oracle.init_params(cfg, seed=2024, device=DEV))
    for l in range(cfg.num_layers):
        key = f"layers.{l}.attention.v_proj.weight"
        params[key] = params[key] * 1e5
    model = UserOptimizedTransformer(cfg).to(DEV).eval()
    model.load_state_dict(params, strict=True)
    model.set_plan(plan)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 8, 0.3, 1.0)
    return cfg, params, model, x.to(DEV), mask.to(DEV)


def test_fp16_range_bound_keeps_such_a_model_on_fp32_schedules():
    """The packed weights bound every activation the split-precision schedule
    holds as fp16 pieces; past 65504 the automatic plan runs the FFMA schedule
    on the GPU (never the CPU) and matches the oracle."""
    cfg, params, model, x, mask = _inflated_v_model()
    with torch.inference_mode():
        y = model(x, mask)
    assert model.fp16_operand_bound > 65504.0
    assert model.forward_plan(cfg.batch_size, cfg.seq_len) == "ops_ffma"
    ref = oracle.forward(params, cfg, x, mask)
    assert ref.abs().max() > 0
    check(ref, y, "inflated v, automatic plan")
    assert model.read_device_status() == (0, 0)


def test_forced_split_schedule_latches_range_error():
    """Forcing the split-precision schedule on that model fails loudly: the
    q|k|v epilogue latches TT_ERR_DEVICE_RANGE in the status word and the
    output is not finite; it never returns silently wrong numbers."""
    from ttjam_gottagofast_b200 import _lib
    cfg, params, model, x, mask = _inflated_v_model("ops_tc")
    with torch.inference_mode():
        y = model(x, mask)
    code, detail = model.read_device_status()
    assert code == _lib.TT_ERR_DEVICE_RANGE, (code, detail)
    assert not torch.isfinite(y).all()
    model.set_plan("auto")
    with torch.inference_mode():
        y2 = model(x, mask)
    check(oracle.forward(params, cfg, x, mask), y2, "inflated v, back on the automatic plan")
    assert model.read_device_status() == (0, 0)


@pytest.mark.parametrize("name", ["A", "C", "D", "E"])
def test_default_models_stay_on_split_precision(name):
    cfg = WORKLOADS[name].config
    model, _ = model_for(cfg)
    model._ensure_image(torch.device(DEV))
    assert 0 < model.fp16_operand_bound < 65504.0 / 8
    assert model._cfg.flags == 0


OFFICIAL_CASES = [f"case{c}" for c in range(1, 14)]


@pytest.mark.parametrize("name", OFFICIAL_CASES)
def test_official_case_parity_sequence_sample(name):
    """The reference's official shapes 1-13 (tools/shapes.py:9-24) at full
    size through the default schedule; the oracle checks the first, a middle
    and the last sequence (sequences are independent)."""
    from ttjam_gottagofast_b200.config import OFFICIAL
    w = OFFICIAL[name]
    cfg = w.config
    model, params = model_for(cfg)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 101234, w.padding_ratio,
                                   w.input_scale)
    x, mask = x.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        y = model(x, mask)
    picks = sorted({0, cfg.batch_size // 2, cfg.batch_size - 1})
    idx = torch.tensor(picks, device=DEV)
    ref = oracle.forward(params, cfg, x[idx], mask[idx], batch_chunk=1)
    check(ref, y[idx], f"{name}[{model.forward_plan(cfg.batch_size, cfg.seq_len)}]/seqs{picks}")
    assert torch.isfinite(y).all()
    assert model.read_device_status() == (0, 0)


def test_output_depends_on_input_and_is_fresh():
    """The reference harness's anti-caching check (tools/harness.py:156-173):
    seeds 101, 202, 101 -- outputs held at the same time."""
    cfg = WORKLOADS["A"].config
    model, _ = model_for(cfg)
    outs = []
    for seed in (101, 202, 101):
        x, mask = generate_random_case(cfg, "cpu", torch.float32, seed, 0.0, 1.0)
        with torch.inference_mode():
            outs.append(model(x.to(DEV), mask.to(DEV)))
    assert not torch.equal(outs[0], outs[1])
    assert torch.equal(outs[0], outs[2])
    assert outs[0].data_ptr() != outs[2].data_ptr()


def test_weight_update_repacks():
    cfg = WORKLOADS["B1"].config
    model = UserOptimizedTransformer(cfg).to(DEV)
    params = oracle.init_params(cfg, seed=5, device=DEV)
    model.load_state_dict(params)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 3, 0.0, 1.0)
    x, mask = x.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        y0 = model(x, mask)
    with torch.no_grad():
        model.layers[0].ffn_out.bias.add_(0.5)      # in-place write: version counter
    params["layers.0.ffn_out.bias"] = params["layers.0.ffn_out.bias"] + 0.5
    with torch.inference_mode():
        y1 = model(x, mask)
    ref = oracle.forward(params, cfg, x, mask)
    assert not torch.equal(y0, y1)
    check(ref, y1, "after in-place update")


@pytest.mark.parametrize("d,h", [(128, 4), (256, 4), (128, 1), (256, 1)],
                         ids=["hd32", "hd64", "hd128", "hd256"])
def test_peaked_scores_rescale_the_context(d, h):
    """Scores spread over hundreds of log2 units (q_proj weights x 32), so that
    rows raise their softmax reference max at later key tiles and the
    attention rescales the context it holds in tensor memory, rows of one warp
    at different tiles. Every applicable schedule against the oracle, key
    padding included."""
    from ttjam_gottagofast_b200.config import TransformerConfig
    cfg = TransformerConfig(batch_size=2, seq_len=300, d_model=d, num_heads=h, ffn_dim=128,
                            num_layers=1, causal=True)
    params = dict(oracle.init_params(cfg, seed=4321, device=DEV))
    params["layers.0.attention.q_proj.weight"] = params["layers.0.attention.q_proj.weight"] * 32
    model = UserOptimizedTransformer(cfg).to(DEV).eval()
    model.load_state_dict(params, strict=True)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 77, 0.3, 1.0)
    x, mask = x.to(DEV), mask.to(DEV)
    ref = oracle.forward(params, cfg, x, mask)
    for plan, y in run_plans(model, x, mask).items():
        check(ref, y, f"peaked d{d} h{h}[{plan}]")
    assert model.read_device_status() == (0, 0)


@pytest.mark.parametrize("name", ["B1", "A", "C"])
def test_no_mask_and_all_true_mask_agree(name):
    """mask=None and an all-true mask give the same bits on every schedule
    (forward_host relies on it to skip an all-true mask's copy)."""
    w = WORKLOADS[name]
    cfg = w.config
    model, _ = model_for(cfg)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 9, 0.0, w.input_scale)
    x, mask = x.to(DEV), mask.to(DEV)
    assert bool(mask.all())
    try:
        for plan in applicable_plans(model, x.shape[0], x.shape[1]):
            model.set_plan(plan)
            with torch.inference_mode():
                assert torch.equal(model(x, None), model(x, mask)), plan
    finally:
        model.set_plan("auto")


def test_runs_on_current_stream():
    cfg = WORKLOADS["B1"].config
    model, params = model_for(cfg)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 4, 0.0, 1.0)
    x, mask = x.to(DEV), mask.to(DEV)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s), torch.inference_mode():
        y = model(x, mask)
    s.synchronize()
    check(oracle.forward(params, cfg, x, mask), y, "side stream")


@pytest.mark.parametrize("name,plan", [("B1", "cluster"), ("A", "ops_ffma"), ("A", "ops_tc"),
                                       ("C", "ops_tc")])
def test_launch_probe_brackets_every_launch(name, plan):
    """tt_launch_probe_* sees every launch of a forward, in schedule order,
    each with a positive device time."""
    import ctypes
    from ttjam_gottagofast_b200 import _lib
    cfg = WORKLOADS[name].config
    model, _ = model_for(cfg)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 5, 0.0, 1.0)
    x, mask = x.to(DEV), mask.to(DEV)
    lib = model._lib
    model.set_plan(plan)
    try:
        n = lib.tt_forward_launch_count(ctypes.byref(model._cfg), cfg.batch_size, cfg.seq_len)
        assert lib.tt_launch_probe_start(2 * n) == 0
        with torch.inference_mode():
            model(x, mask)
            model(x, mask)
        ms = (ctypes.c_float * (2 * n))()
        kinds = (ctypes.c_int32 * (2 * n))()
        assert lib.tt_launch_probe_read(ms, kinds, 2 * n) == 2 * n
        assert lib.tt_launch_probe_read(ms, kinds, 2 * n) == 0  # read restarts the count
    finally:
        lib.tt_launch_probe_start(0)
        model.set_plan("auto")
    names = [_lib.KERNEL_KINDS[k] for k in kinds]
    # the tensor-core schedule folds both LayerNorms into the GEMMs that read
    # them for small problems (5 launches per layer then, else 7)
    fused = plan == "ops_tc" and n == 5 * cfg.num_layers + 1
    per_layer = {"cluster": [],
                 "ops_ffma": ["qkv", "attention", "out_proj", "ffn_in", "ffn_out"],
                 "ops_tc": (["qkv", "attention", "out_proj", "ffn_in", "ffn_out"] if fused else
                            ["layernorm", "qkv", "attention", "out_proj", "layernorm",
                             "ffn_in", "ffn_out"])}[plan]
    # tensor-core shapes with d_model >= 256 and at least 1024 rows start with
    # the live-row scan
    scan = (["row_scan"] if plan == "ops_tc" and cfg.d_model >= 256 and
            cfg.batch_size * cfg.seq_len >= 1024 else [])
    one = (["whole_forward"] if plan == "cluster"
           else scan + per_layer * cfg.num_layers + ["final_norm"])
    assert names == one * 2
    assert all(t > 0 for t in ms)


@pytest.mark.parametrize("name,plan", [("A", "ops_tc"), ("A", "ops_ffma"), ("C", "ops_tc")])
def test_graph_replay_matches_direct_launch(name, plan):
    """From the second call with the same pointers on, the per-op schedules
    replay a cached CUDA graph. A replay computes from the buffers' current
    contents and is bit-identical to a direct launch (the launch probe forces
    direct launches)."""
    import ctypes
    from ttjam_gottagofast_b200 import _lib
    cfg = WORKLOADS[name].config
    model, _ = model_for(cfg)
    lib = model._lib
    x1, m1 = generate_random_case(cfg, "cpu", torch.float32, 11, 0.25, 1.0)
    x2, m2 = generate_random_case(cfg, "cpu", torch.float32, 12, 0.25, 1.0)
    b, s = x1.shape[:2]
    c = _lib.make_config(model.config, plan)
    image = model._ensure_image(torch.device(DEV))
    x, m = x1.to(DEV), m1.to(DEV)
    y = torch.empty_like(x)
    ws_bytes = lib.tt_workspace_bytes(ctypes.byref(c), b, s)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream

    def fwd():
        assert lib.tt_forward(ctypes.byref(c), image.data_ptr(), x.data_ptr(), m.data_ptr(), b, s,
                              y.data_ptr(), ws.data_ptr(), ws_bytes, stream) == 0
        return y.clone()

    outs = [fwd() for _ in range(4)]  # direct, capture + replay, replay, replay
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    x.copy_(x2.to(DEV))
    m.copy_(m2.to(DEV))
    got = fwd()  # the same graph, new buffer contents
    assert lib.tt_launch_probe_start(1000) == 0
    try:
        ref = fwd()
    finally:
        lib.tt_launch_probe_start(0)
    assert torch.equal(got, ref)
    assert not torch.equal(got, outs[0])
    torch.cuda.synchronize()
    assert model.read_device_status() == (0, 0)


def test_forward_inside_caller_graph_capture():
    """A caller capturing its stream gets the forward's launches in its own
    graph (the library's graph cache stays out of the way)."""
    cfg = WORKLOADS["A"].config
    model, _ = model_for(cfg)
    x, m = generate_random_case(cfg, "cpu", torch.float32, 13, 0.25, 1.0)
    x, m = x.to(DEV), m.to(DEV)
    with torch.inference_mode():
        ref = model(x, m)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side), torch.inference_mode():
        model(x, m)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g), torch.inference_mode():
        out = model(x, m)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("slices", [1, 3, 4])
def test_forward_host_matches_device_forward(slices):
    """forward_host: host buffers in and out, the batch in slices whose copies
    overlap the compute on their own streams; the result equals the device
    forward's (the same row computations) and the current stream is ordered
    after the last copy."""
    from ttjam_gottagofast_b200.config import TransformerConfig
    cfg = TransformerConfig(batch_size=7, seq_len=256, d_model=256, num_heads=4, ffn_dim=512,
                            num_layers=2, causal=True)
    model, params = model_for(cfg, seed=31)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 17, 0.5, 1.0)
    xh, mh = x.pin_memory(), mask.pin_memory()
    with torch.inference_mode():
        ref_dev = model(x.to(DEV), mask.to(DEV)).cpu()
        out = model.forward_host(xh, mh, slices=slices)
    torch.cuda.current_stream().synchronize()
    res = compare_outputs(ref_dev, out)
    assert res.passed and res.max_abs_error <= 1e-5, res
    assert (out[~mask] == 0).all()
    check(oracle.forward(params, cfg, x.to(DEV), mask.to(DEV)).cpu(), out, f"host x{slices}")
