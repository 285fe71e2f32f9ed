"""The C ABI from a plain C host (tests/c_abi/c_host.c): no Python and no torch
in the call path. The program includes include/ttjam_b200.h, links
libttjam_b200.so and the CUDA runtime, packs a model image from raw device
buffers, checks the fp16 operand bound, runs tt_forward twice (the second call
replays the cached graph) and tt_forward_noalloc, and writes the outputs; the
test compares them with the oracle under the contract's accuracy gate
(abs <= 0.002 OR abs <= 0.02*|ref|). Building it needs only gcc and the CUDA
headers; running it needs a GPU."""
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

from ttjam_gottagofast_b200 import _lib, compare_outputs, generate_random_case
from ttjam_gottagofast_b200.config import TransformerConfig

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "c_abi", "c_host.c")
CUDA = "/usr/local/cuda"


def build_c_host(out_dir):
    lib_dir = os.path.dirname(_lib.lib_path())
    exe = os.path.join(out_dir, "c_host")
    cmd = [shutil.which("gcc") or "gcc", "-O2", "-std=c11", "-Wall", "-Werror",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"), SRC,
           "-L", lib_dir, "-lttjam_b200", "-L", os.path.join(CUDA, "lib64"), "-lcudart",
           f"-Wl,-rpath,{lib_dir}", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}", "-o", exe]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
    return exe


def test_c_host_builds_against_the_header(tmp_path):
    _lib.load()  # the library is built
    exe = build_c_host(str(tmp_path))
    assert os.access(exe, os.X_OK)


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(3, 100, 128, 4, 256, 2, 0.4), (2, 256, 512, 8, 1024, 2, 0.5)],
                         ids=["d128_s100_padded", "d512_s256_padded"])
def test_c_host_forward_matches_oracle(tmp_path, shape):
    from oracle import reference_model as oracle
    b, s, d, h, f, layers, pad = shape
    cfg = TransformerConfig(b, s, d, h, f, layers, True)
    params = oracle.init_params(cfg, seed=404)
    x, mask = generate_random_case(cfg, "cpu", torch.float32, 405, pad, 1.0)
    work = str(tmp_path)
    with open(os.path.join(work, "cfg.txt"), "w") as fh:
        fh.write(f"{d} {h} {f} {layers} 1 {b} {s} 1\n")
    np.concatenate([v.reshape(-1).numpy() for v in params.values()]).astype(np.float32).tofile(
        os.path.join(work, "params.bin"))
    x.numpy().astype(np.float32).tofile(os.path.join(work, "x.bin"))
    mask.numpy().astype(np.uint8).tofile(os.path.join(work, "mask.bin"))
    exe = build_c_host(work)
    res = subprocess.run([exe, work], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stdout + res.stderr
    fields = res.stdout.split()
    info = dict(zip(fields[0::2], fields[1::2]))
    assert info["status"] == "0" and info["noalloc"] == "0", res.stdout
    dev = torch.device("cuda:0")
    with torch.inference_mode():
        ref = oracle.forward({k: v.to(dev) for k, v in params.items()}, cfg, x.to(dev),
                             mask.to(dev)).cpu()
    for name in ("y.bin", "y_noalloc.bin"):
        y = torch.from_numpy(np.fromfile(os.path.join(work, name), dtype=np.float32)).view(b, s, d)
        r = compare_outputs(ref, y)
        assert r.passed, (name, r)
        assert (y[~mask] == 0).all()
