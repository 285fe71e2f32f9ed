"""The harness candidate file loads the way the reference harness loads it.

tools/harness.py:40-47 loads `--candidate` by path as a top-level module named
"candidate", with no parent package, and tools/harness.py:84-99 then builds the
model with `build_model(config, bench)`, `.to(device, dtype).eval()` and
`load_from_baseline(model, baseline)`. Run in a fresh interpreter whose
sys.path does not hold this repository, from another directory, so nothing but
the candidate file itself can make the package importable. No GPU is needed:
construction, weight copy and `.to()` never launch a kernel.
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r"""
import importlib.util, json, sys
sys.path = [p for p in sys.path if p not in ("", ".", ROOT) and not p.startswith(ROOT + "/")]

def load_module(path, name):  # tools/harness.py:40-47
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod

try:
    import ttjam_gottagofast_b200
    importable_before = True
except ImportError:
    importable_before = False
candidate = load_module(ROOT + "/ttjam_gottagofast_b200/candidate.py", "candidate")
bench = load_module(ROOT + "/tests/harness_bench.py", "bench")
import torch
cfg = bench.TransformerConfig(batch_size=2, seq_len=8, d_model=64, num_heads=4, ffn_dim=96,
                              num_layers=2, causal=True)
torch.manual_seed(7)
baseline = bench.BaselineTransformer(cfg).to(device="cpu", dtype=torch.float32).eval()
torch.manual_seed(7)
seeded = candidate.build_model(cfg, bench)
model = candidate.build_model(cfg, bench).to(device="cpu", dtype=torch.float32).eval()
candidate.load_from_baseline(model, baseline)
same_init = all(torch.equal(a, b) for a, b in zip(baseline.state_dict().values(),
                                                  seeded.state_dict().values()))
same_weights = all(torch.equal(a, b) for a, b in zip(baseline.state_dict().values(),
                                                     model.state_dict().values()))
plain = candidate.build_model(cfg)
print(json.dumps({
    "importable_before": importable_before,
    "class": type(model).__name__,
    "is_baseline_subclass": isinstance(model, bench.BaselineTransformer),
    "keys_equal": list(model.state_dict()) == list(baseline.state_dict()),
    "same_init": same_init,
    "same_weights": same_weights,
    "plain_class": type(plain).__name__,
    "plain_keys_equal": list(plain.state_dict()) == list(baseline.state_dict()),
}))
"""


def test_candidate_loads_by_path_without_package_on_sys_path():
    env = {k: v for k, v in os.environ.items() if k != "PYTHONPATH"}
    code = "ROOT = " + repr(ROOT) + "\n" + SCRIPT
    res = subprocess.run([sys.executable, "-c", code], cwd="/tmp", env=env,
                         capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-3000:]
    out = json.loads(res.stdout.strip().splitlines()[-1])
    assert out["importable_before"] is False, "the test must start without the package"
    assert out["class"] == "UserOptimizedTransformer"
    assert out["is_baseline_subclass"], "build_model(config, bench) subclasses bench's baseline"
    assert out["keys_equal"] and out["same_init"] and out["same_weights"], out
    assert out["plain_class"] == "UserOptimizedTransformer" and out["plain_keys_equal"]
