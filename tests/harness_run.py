#!/usr/bin/env python3
"""The reference evaluation harness's per-case checks, run against this build.

Restates tools/harness.py for one candidate against the eager baseline:

* the candidate file is loaded by path as a top-level module named
  "candidate" (`load_module`, :40-47), the contract module as "bench";
* models are built as `build_models` does (:84-108): baseline
  `bench.BaselineTransformer(config)`, candidate `build_model(config, bench)`
  -> `.to(device, dtype).eval()` -> `load_from_baseline(model, baseline)`;
* correctness over the five input variants with the contract's gate
  (`check_correctness`, :121-153);
* the anti-caching check (`check_output_depends_on_input`, :156-173);
* paired, rotating-order event timing of baseline and candidate plus the
  synchronised wall-clock pass, and the wall/event <= 1.6 stream-escape gate
  (`time_models`, :189-238, :313-327);
* the torch global-flag snapshot before and after (`env_snapshot`, :54-63);
* status per case and the geomean speedup over the "ok" cases (:378-420).

The contract module is `harness_bench.py` beside this file (the reference's
own file is not present where the GPU runs); its baseline is the oracle
restatement of the reference forward, fp32 eager with TF32 off (the harness
never enables TF32).

    python tests/harness_run.py [--cases 1,2,...] [--out report.json]
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import math
import os
import statistics
import sys
import time
import traceback

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CANDIDATE = os.path.join(ROOT, "ttjam_gottagofast_b200", "candidate.py")
BENCH = os.path.join(HERE, "harness_bench.py")

VARIANTS = [  # tools/harness.py:121-127
    {"name": "normal", "seed": 11, "input_scale": 1.0, "padding_ratio": 0.0},
    {"name": "large_scale", "seed": 22, "input_scale": 8.0, "padding_ratio": 0.0},
    {"name": "small_scale", "seed": 33, "input_scale": 0.05, "padding_ratio": 0.0},
    {"name": "padded", "seed": 44, "input_scale": 1.0, "padding_ratio": 0.3},
    {"name": "padded_heavy", "seed": 55, "input_scale": 2.0, "padding_ratio": 0.7},
]


def load_module(path, name):
    """tools/harness.py:40-47."""
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def env_snapshot():
    """tools/harness.py:54-63."""
    return {
        "matmul_tf32": torch.backends.cuda.matmul.allow_tf32,
        "cudnn_tf32": torch.backends.cudnn.allow_tf32,
        "cudnn_benchmark": torch.backends.cudnn.benchmark,
        "float32_matmul_precision": torch.get_float32_matmul_precision(),
        "grad_enabled": torch.is_grad_enabled(),
        "default_dtype": str(torch.get_default_dtype()),
        "num_threads": torch.get_num_threads(),
    }


def check_correctness(bench, baseline, model, config, device, dtype, rtol, atol):
    """tools/harness.py:130-153."""
    results, ok = [], True
    for v in VARIANTS:
        x, mask = bench.generate_random_case(config, device, dtype, v["seed"],
                                             v["padding_ratio"], v["input_scale"])
        with torch.inference_mode():
            ref = baseline(x, mask)
            got = model(x, mask)
        res = bench.compare_outputs(ref, got, rtol=rtol, atol=atol)
        results.append({"variant": v["name"], "passed": bool(res.passed),
                        "max_abs": res.max_abs_error, "max_rel": res.max_relative_error})
        ok = ok and bool(res.passed)
        del x, mask, ref, got
        torch.cuda.empty_cache()
    return {"passed": ok, "variants": results}


def check_output_depends_on_input(bench, model, config, device, dtype):
    """tools/harness.py:156-173."""
    x1, m1 = bench.generate_random_case(config, device, dtype, 101, 0.0, 1.0)
    x2, m2 = bench.generate_random_case(config, device, dtype, 202, 0.0, 1.0)
    with torch.inference_mode():
        o1 = model(x1, m1)
        o2 = model(x2, m2)
        o1b = model(x1, m1)
    differs = not torch.allclose(o1.float(), o2.float(), rtol=1e-3, atol=1e-3)
    repeatable = torch.allclose(o1.float(), o1b.float(), rtol=1e-3, atol=1e-3)
    return bool(differs and repeatable)


def wall_time_model(model, x, mask, device, repeats):
    """tools/harness.py:180-186."""
    torch.cuda.synchronize(device)
    t0 = time.perf_counter()
    with torch.inference_mode():
        for _ in range(repeats):
            model(x, mask)
    torch.cuda.synchronize(device)
    return (time.perf_counter() - t0) * 1e3 / repeats


def time_models(bench, models, x, mask, device, warmup, repeats, rounds):
    """tools/harness.py:189-238: paired rounds in rotating order, then a
    synchronised wall-clock pass in reverse order."""
    names = list(models)
    samples = {n: [] for n in names}
    for m in models.values():
        bench.warmup_model(m, x, mask, warmup, device)
    order = names
    for r in range(rounds):
        shift = r % len(names)
        order = names[shift:] + names[:shift]
        if (r // len(names)) % 2:
            order.reverse()
        for n in order:
            samples[n].extend(bench.benchmark_once(models[n], x, mask, repeats, device))
    wall = {n: wall_time_model(models[n], x, mask, device, repeats) for n in reversed(order)}
    return {n: {"median_ms": statistics.median(samples[n]), "min_ms": min(samples[n]),
                "wall_ms": wall[n], "n": len(samples[n])} for n in names}


def evaluate_case(bench, candidate, shape, device, args):
    """tools/harness.py:241-345 for one case (the baseline always fits here:
    cases 1-13)."""
    out = {"case": shape[0], "shape": dict(zip(
        ("batch_size", "d_model", "num_heads", "seq_len", "num_layers", "ffn_dim"), shape[1:]))}
    s = out["shape"]
    config = bench.TransformerConfig(batch_size=s["batch_size"], seq_len=s["seq_len"],
                                     d_model=s["d_model"], num_heads=s["num_heads"],
                                     ffn_dim=s["ffn_dim"], num_layers=s["num_layers"],
                                     causal=True)
    dtype = torch.float32
    try:
        baseline = bench.BaselineTransformer(config).to(device=device, dtype=dtype).eval()
        model = candidate.build_model(config, bench)
        model = model.to(device=device, dtype=dtype).eval()
        candidate.load_from_baseline(model, baseline)
        out["candidate_class_mro"] = [c.__name__ for c in type(model).__mro__[:3]]
    except Exception as e:  # noqa: BLE001 - the harness reports, not raises
        out["status"] = "build_error"
        out["error"] = f"{type(e).__name__}: {e}"
        return out
    try:
        corr = check_correctness(bench, baseline, model, config, device, dtype,
                                 args.rtol, args.atol)
        out["correctness"] = corr
        if not corr["passed"]:
            out["status"] = "incorrect"
            return out
        out["input_dependence_ok"] = check_output_depends_on_input(bench, model, config,
                                                                   device, dtype)
        if not out["input_dependence_ok"]:
            out["status"] = "integrity_failed"
            return out
        x, mask = bench.generate_random_case(config, device, dtype, args.seed + 100000,
                                             0.0, 1.0)
        t = time_models(bench, {"candidate": model, "baseline": baseline}, x, mask, device,
                        args.warmup, args.repeats, args.rounds)
        out["candidate"], out["baseline"] = t["candidate"], t["baseline"]
        out["speedup"] = t["baseline"]["median_ms"] / t["candidate"]["median_ms"]
        ratio = t["candidate"]["wall_ms"] / max(t["candidate"]["median_ms"], 1e-9)
        out["wall_to_event_ratio"] = round(ratio, 3)
        out["stream_ok"] = ratio < args.max_wall_ratio
        out["status"] = "ok" if out["stream_ok"] else "integrity_failed"
        out["plan"] = model.forward_plan(config.batch_size, config.seq_len)
        out["device_status"] = list(model.read_device_status())
        if out["device_status"] != [0, 0]:
            out["status"] = "runtime_error"
    except torch.cuda.OutOfMemoryError as e:
        out["status"] = "oom"
        out["error"] = str(e).split("\n")[0]
    except Exception as e:  # noqa: BLE001
        out["status"] = "runtime_error"
        out["error"] = f"{type(e).__name__}: {e}"
        out["traceback"] = traceback.format_exc()[-1500:]
    finally:
        torch.cuda.empty_cache()
    return out


def run(cases, args):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, HERE)
    device = torch.device("cuda")
    bench = load_module(BENCH, "bench")
    candidate = load_module(CANDIDATE, "candidate")
    from ttjam_gottagofast_b200.config import OFFICIAL_TABLE
    env_before = env_snapshot()
    report = {"candidate": os.path.basename(CANDIDATE), "dtype": "float32",
              "gpu": torch.cuda.get_device_name(device), "torch": torch.__version__,
              "timestamp": time.strftime("%Y-%m-%dT%H:%M:%S"), "cases": []}
    for row in OFFICIAL_TABLE:
        if row[0] in cases:
            r = evaluate_case(bench, candidate, row, device, args)
            report["cases"].append(r)
            print(f"case {r['case']:>2}  {r['status']:<16} speedup="
                  f"{r.get('speedup', float('nan')):.3f} wall/event="
                  f"{r.get('wall_to_event_ratio')} {r.get('error', '')}", flush=True)
    env_after = env_snapshot()
    report["env_before"], report["env_after"] = env_before, env_after
    report["env_unchanged"] = env_before == env_after
    speedups = [c["speedup"] for c in report["cases"] if c.get("status") == "ok"]
    report["failed_cases"] = [c["case"] for c in report["cases"] if c["status"] != "ok"]
    report["n_scored"] = len(speedups)
    report["geomean_speedup"] = (math.exp(statistics.fmean(math.log(s) for s in speedups))
                                 if speedups else 0.0)
    return report


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--cases", default=",".join(str(c) for c in range(1, 14)))
    p.add_argument("--rtol", type=float, default=0.02)
    p.add_argument("--atol", type=float, default=0.002)
    p.add_argument("--seed", type=int, default=1234)
    p.add_argument("--warmup", type=int, default=20)
    p.add_argument("--repeats", type=int, default=50)
    p.add_argument("--rounds", type=int, default=3)
    p.add_argument("--max-wall-ratio", type=float, default=1.6)
    p.add_argument("--out", default="")
    return p.parse_args(argv)


def main(argv=None):
    args = parse_args(argv)
    cases = {int(c) for c in args.cases.split(",") if c.strip()}
    report = run(cases, args)
    blob = json.dumps(report, indent=2)
    if args.out:
        with open(args.out, "w") as fh:
            fh.write(blob)
    print(f"scored {report['n_scored']} cases | geomean {report['geomean_speedup']:.4f}x | "
          f"failed {report['failed_cases']} | env_unchanged {report['env_unchanged']}")
    return 0 if not report["failed_cases"] and report["env_unchanged"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
