"""Stand-in for the reference contract module, as the evaluation harness uses it.

The reference harness (tools/harness.py) is driven by the contract module
torch_transformer_benchmark.py, which it loads by path as `bench`. That module
is not available where the GPU runs, so this file provides the same names with
the same behaviour, built from this repository's restatements:

* `TransformerConfig`, `generate_random_case`, `compare_outputs`,
  `copy_model_weights` -- the package's interface copies (:29-56, :234-272,
  :289-356, :203-213);
* `BaselineTransformer` -- the reference's parameter structure (:59-172) whose
  forward is the oracle restatement of `BaselineTransformer.forward` in fp32
  eager torch, i.e. the same ATen ops in the same order;
* `warmup_model` / `benchmark_once` -- the contract's timing helpers
  (:459-507): CUDA events recorded on the current stream around each call.

Test infrastructure only: the oracle is the checker, never the measured path.
"""
from __future__ import annotations

from typing import List, Optional

import torch
import torch.nn as nn

from oracle import reference_model as _oracle
from ttjam_gottagofast_b200.candidate import copy_model_weights  # noqa: F401
from ttjam_gottagofast_b200.config import TransformerConfig  # noqa: F401
from ttjam_gottagofast_b200.contract import compare_outputs, generate_random_case  # noqa: F401
from ttjam_gottagofast_b200.model import TransformerBlock


class BaselineTransformer(nn.Module):
    """torch_transformer_benchmark.py:149-172: same submodules, same
    construction order (so the same seeded weights), eager fp32 forward."""

    def __init__(self, config) -> None:
        super().__init__()
        self.config = config
        self.layers = nn.ModuleList([
            TransformerBlock(config.d_model, config.num_heads, config.ffn_dim)
            for _ in range(config.num_layers)])
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, x: torch.Tensor,
                valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        params = dict(self.named_parameters())
        return _oracle._forward(params, self.config, x, valid_token_mask)


def warmup_model(model: nn.Module, x: torch.Tensor, valid_mask: torch.Tensor,
                 iterations: int, device: torch.device) -> None:
    """torch_transformer_benchmark.py:459-474."""
    with torch.inference_mode():
        for _ in range(iterations):
            model(x, valid_mask)
    if device.type == "cuda":
        torch.cuda.synchronize(device)


def benchmark_once(model: nn.Module, x: torch.Tensor, valid_mask: torch.Tensor,
                   iterations: int, device: torch.device) -> List[float]:
    """torch_transformer_benchmark.py:477-507 (the CUDA branch): one event
    pair per call, recorded on the current stream."""
    samples_ms: List[float] = []
    with torch.inference_mode():
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(iterations)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(iterations)]
        torch.cuda.synchronize(device)
        for i in range(iterations):
            starts[i].record()
            model(x, valid_mask)
            ends[i].record()
        torch.cuda.synchronize(device)
        samples_ms.extend(s.elapsed_time(e) for s, e in zip(starts, ends))
    return samples_ms
