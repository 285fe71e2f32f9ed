"""Generate the 16-bit golden fixtures from the reference module itself.

Run in a container that has the reference source tree (it is imported by path,
never copied):

    python tests/golden/make_golden_16bit.py /root/reference

The reference benchmarks a 16-bit model by moving the model and its input to
that dtype (torch_transformer_benchmark.py:225-231, :698-699). For every case
this builds `BaselineTransformer` under `torch.manual_seed(seed)`, moves it to
bfloat16 (the 16-bit type the reference's CLI allows on CPU, :662-666), draws
x and the mask with the contract's `generate_random_case` in bfloat16 on CPU
(:234-272), and records two outputs of the reference module:

* `y`: its bfloat16 forward, what the reference computes for that model;
* `y_f32`: the same module moved back to float32 (the bfloat16 weights widen
  exactly) run on the widened input: the fp32 value of the 16-bit model.

Both go to `goldens_16bit.npz` as float32 arrays (exact for bfloat16 values),
with the case list in `manifest_16bit.json`.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from make_golden import MODEL_SEED, load_reference, param_checksums  # noqa: E402

# (name, (B, S, D, H, F, L, causal), data seed, input scale, padding ratio)
CASES = [
    ("B1_bf16", (4, 16, 128, 4, 128, 4, True), 101234, 1.0, 0.0),
    ("h_large_scale_bf16", (2, 64, 128, 4, 128, 4, True), 22, 8.0, 0.0),
    ("h_padded_bf16", (2, 64, 128, 4, 128, 4, True), 44, 1.0, 0.3),
    ("D_small_bf16", (1, 64, 512, 8, 2048, 6, True), 101234, 0.05, 0.0),
]


def main(root):
    ref = load_reference(root)
    arrays, manifest = {}, []
    for name, (b, s, d, h, f, l, causal), seed, scale, pad in CASES:
        cfg = ref.TransformerConfig(batch_size=b, seq_len=s, d_model=d, num_heads=h,
                                    ffn_dim=f, num_layers=l, causal=causal)
        cfg.validate()
        torch.manual_seed(MODEL_SEED)
        model = ref.BaselineTransformer(cfg).eval().to(dtype=torch.bfloat16)
        x, mask = ref.generate_random_case(cfg, torch.device("cpu"), torch.bfloat16,
                                           seed, pad, scale)
        with torch.inference_mode():
            y = model(x, mask)
            model32 = model.to(dtype=torch.float32)
            y32 = model32(x.float(), mask)
        assert torch.isfinite(y.float()).all() and torch.isfinite(y32).all(), name
        arrays[name + "/x"] = x.float().numpy()
        arrays[name + "/mask"] = mask.numpy()
        arrays[name + "/y"] = y.float().numpy()
        arrays[name + "/y_f32"] = y32.numpy()
        manifest.append({
            "name": name, "dtype": "bfloat16", "batch_size": b, "seq_len": s, "d_model": d,
            "num_heads": h, "ffn_dim": f, "num_layers": l, "causal": causal,
            "data_seed": seed, "input_scale": scale, "padding_ratio": pad, "mask_kind": "gen",
            "model_seed": MODEL_SEED,
            "param_checksums": param_checksums(model32.state_dict()),
        })
        err = float((y.float() - y32).abs().max())
        print(f"{name}: y {tuple(y.shape)} max|y|={float(y32.abs().max()):.4f} "
              f"max|y_bf16 - y_f32|={err:.4f}")
    np.savez_compressed(os.path.join(HERE, "goldens_16bit.npz"), **arrays)
    with open(os.path.join(HERE, "manifest_16bit.json"), "w") as fh:
        json.dump({"torch": torch.__version__, "cases": manifest}, fh, indent=1)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
