"""Generate the golden fixtures from the reference module itself.

Run in a container that has the reference source tree (it is imported by path,
never copied):

    python tests/golden/make_golden.py /root/reference

For every case it builds `BaselineTransformer` under `torch.manual_seed(seed)`
exactly as the contract's CLI does (torch_transformer_benchmark.py:683-699),
draws x and the mask with the contract's `generate_random_case` on CPU
(:234-272) -- or uses an explicit mask for the non-prefix cases -- runs the
reference forward in fp32 under inference_mode on CPU, and stores x, mask, the
output and a checksum of every parameter in `goldens.npz`, with the case list
in `manifest.json`. The tests regenerate weights from the seed and compare the
checksums, so a change in torch's RNG shows up as a checksum failure rather
than a parity failure.
"""
from __future__ import annotations

import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, (B, S, D, H, F, L, causal), data seed, input scale, padding ratio, mask kind)
CASES = [
    ("A", (8, 128, 128, 4, 128, 4, True), 101234, 1.0, 0.0, "gen"),
    ("B1", (4, 16, 128, 4, 128, 4, True), 101234, 1.0, 0.0, "gen"),
    ("B2", (32, 1, 128, 4, 128, 4, True), 101234, 1.0, 0.0, "gen"),
    # the reference harness's five variants (tools/harness.py:121-127) at B2 S64
    ("h_normal", (2, 64, 128, 4, 128, 4, True), 11, 1.0, 0.0, "gen"),
    ("h_large_scale", (2, 64, 128, 4, 128, 4, True), 22, 8.0, 0.0, "gen"),
    ("h_small_scale", (2, 64, 128, 4, 128, 4, True), 33, 0.05, 0.0, "gen"),
    ("h_padded", (2, 64, 128, 4, 128, 4, True), 44, 1.0, 0.3, "gen"),
    ("h_padded_heavy", (2, 64, 128, 4, 128, 4, True), 55, 2.0, 0.7, "gen"),
    # each large workload's own distribution at a reduced batch/sequence
    ("C_small", (4, 128, 128, 4, 128, 4, True), 101234, 8.0, 0.5, "gen"),
    ("D_small", (1, 64, 512, 8, 2048, 6, True), 101234, 0.05, 0.0, "gen"),
    ("E_small", (2, 48, 1024, 16, 4096, 12, True), 101234, 1.0, 0.5, "gen"),
    # shapes from the reference's official table (tools/shapes.py:9-24) at small B/S
    ("d32_hd8", (3, 17, 32, 4, 32, 4, True), 7, 1.0, 0.5, "gen"),
    ("h1_hd128", (2, 33, 128, 1, 128, 4, True), 8, 1.0, 0.0, "gen"),
    ("h16_hd8", (2, 20, 128, 16, 128, 4, True), 9, 1.0, 0.3, "gen"),
    ("d1024_h4_hd256", (1, 24, 1024, 4, 1024, 1, True), 10, 1.0, 0.0, "gen"),
    # head dims 16 and 8 on the tensor-core attention (8 runs padded to 16):
    # several query and key tiles, padding, the last head's box past the row
    ("h4_hd16", (2, 70, 64, 4, 96, 2, True), 17, 1.0, 0.4, "gen"),
    ("h8_hd8_s150", (2, 150, 64, 8, 64, 2, True), 18, 1.0, 0.3, "gen"),
    # semantics corners
    ("noncausal_padded", (3, 19, 128, 4, 128, 2, False), 12, 1.0, 0.5, "gen"),
    ("seq1_noncausal", (5, 1, 128, 4, 128, 2, False), 13, 1.0, 0.0, "gen"),
    ("holes_causal", (3, 24, 128, 4, 128, 2, True), 14, 1.0, 0.0, "holes"),
    ("holes_noncausal", (3, 24, 128, 4, 128, 2, False), 15, 1.0, 0.0, "holes"),
    ("nomask_causal", (2, 40, 64, 2, 96, 2, True), 16, 1.0, 0.0, "none"),
]
MODEL_SEED = 1234


def load_reference(root):
    path = os.path.join(root, "torch_transformer_benchmark.py")
    spec = importlib.util.spec_from_file_location("ttb_reference", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ttb_reference"] = mod
    spec.loader.exec_module(mod)
    return mod


def param_checksums(sd):
    return {k: [float(v.double().sum()), float(v.double().abs().sum())]
            for k, v in sd.items()}


def holes_mask(b, s, seed):
    """A non-prefix mask: random holes, sequence 0 starts with a masked token and
    the last sequence is fully masked (every query of it has no valid key)."""
    g = torch.Generator().manual_seed(seed)
    m = torch.rand(b, s, generator=g) > 0.35
    m[0, 0] = False
    m[-1, :] = False
    return m


def main(root):
    ref = load_reference(root)
    arrays, manifest = {}, []
    for name, (b, s, d, h, f, l, causal), seed, scale, pad, kind in CASES:
        cfg = ref.TransformerConfig(batch_size=b, seq_len=s, d_model=d, num_heads=h,
                                    ffn_dim=f, num_layers=l, causal=causal)
        cfg.validate()
        torch.manual_seed(MODEL_SEED)
        model = ref.BaselineTransformer(cfg).eval()
        x, mask = ref.generate_random_case(cfg, torch.device("cpu"), torch.float32,
                                           seed, pad, scale)
        if kind == "holes":
            mask = holes_mask(b, s, seed)
            x = x.masked_fill(~mask[..., None], 0)
        with torch.inference_mode():
            y = model(x, None if kind == "none" else mask)
        assert torch.isfinite(y).all(), name
        arrays[name + "/x"] = x.numpy()
        arrays[name + "/mask"] = mask.numpy()
        arrays[name + "/y"] = y.numpy()
        manifest.append({
            "name": name, "batch_size": b, "seq_len": s, "d_model": d, "num_heads": h,
            "ffn_dim": f, "num_layers": l, "causal": causal, "data_seed": seed,
            "input_scale": scale, "padding_ratio": pad, "mask_kind": kind,
            "model_seed": MODEL_SEED, "param_checksums": param_checksums(model.state_dict()),
        })
        print(f"{name}: y {tuple(y.shape)} max|y|={float(y.abs().max()):.4f}")
    np.savez_compressed(os.path.join(HERE, "goldens.npz"), **arrays)
    with open(os.path.join(HERE, "manifest.json"), "w") as fh:
        json.dump({"torch": torch.__version__, "cases": manifest}, fh, indent=1)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
