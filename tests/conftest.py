import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs 2 or more GPUs")


def pytest_collection_modifyitems(config, items):
    import torch
    have_gpu = torch.cuda.is_available()
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords and not have_gpu:
            item.add_marker(skip)


class GoldenCase:
    def __init__(self, meta, arrays):
        self.meta = meta
        self.name = meta["name"]
        self.x = arrays[self.name + "/x"]
        self.mask = arrays[self.name + "/mask"]
        self.y = arrays[self.name + "/y"]

    @property
    def config(self):
        from ttjam_gottagofast_b200.config import TransformerConfig
        m = self.meta
        return TransformerConfig(batch_size=m["batch_size"], seq_len=m["seq_len"],
                                 d_model=m["d_model"], num_heads=m["num_heads"],
                                 ffn_dim=m["ffn_dim"], num_layers=m["num_layers"],
                                 causal=m["causal"])

    @property
    def uses_mask(self):
        return self.meta["mask_kind"] != "none"


def load_goldens():
    with open(os.path.join(GOLDEN_DIR, "manifest.json")) as fh:
        manifest = json.load(fh)
    arrays = np.load(os.path.join(GOLDEN_DIR, "goldens.npz"))
    return [GoldenCase(m, arrays) for m in manifest["cases"]]


GOLDENS = load_goldens()
GOLDEN_IDS = [g.name for g in GOLDENS]


class GoldenCase16(GoldenCase):
    """A 16-bit golden: x and the reference's 16-bit output `y` (as float32,
    exact), and `y_f32`, the reference module's fp32 forward of the same
    16-bit weights and input (make_golden_16bit.py)."""

    def __init__(self, meta, arrays):
        super().__init__(meta, arrays)
        self.y_f32 = arrays[self.name + "/y_f32"]

    @property
    def dtype(self):
        import torch
        return getattr(torch, self.meta["dtype"])


def load_goldens_16bit():
    with open(os.path.join(GOLDEN_DIR, "manifest_16bit.json")) as fh:
        manifest = json.load(fh)
    arrays = np.load(os.path.join(GOLDEN_DIR, "goldens_16bit.npz"))
    return [GoldenCase16(m, arrays) for m in manifest["cases"]]


GOLDENS_16BIT = load_goldens_16bit()
GOLDEN_16BIT_IDS = [g.name for g in GOLDENS_16BIT]


@pytest.fixture(scope="session")
def goldens():
    return GOLDENS
