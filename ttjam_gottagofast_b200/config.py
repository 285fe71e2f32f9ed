"""Shape record of the pre-norm Transformer forward and the named workloads.

`TransformerConfig` mirrors the reference contract's frozen dataclass
(torch_transformer_benchmark.py:29-56): same field names, same order, same
`validate()` rules and messages, so a reference config object and this one are
interchangeable wherever only the fields are read.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict


@dataclass(frozen=True)
class TransformerConfig:
    """torch_transformer_benchmark.py:29-37."""

    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        """torch_transformer_benchmark.py:39-56 (same checks, same messages)."""
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.d_model <= 0:
            raise ValueError("d_model must be positive")
        if self.num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(
                f"d_model ({self.d_model}) must be divisible by "
                f"num_heads ({self.num_heads})"
            )
        if self.ffn_dim <= 0:
            raise ValueError("ffn_dim must be positive")
        if self.num_layers <= 0:
            raise ValueError("num_layers must be positive")

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads


@dataclass(frozen=True)
class Workload:
    """A named input distribution over one config, as generate_random_case draws it
    (torch_transformer_benchmark.py:234-272)."""

    name: str
    config: TransformerConfig
    input_scale: float
    padding_ratio: float
    description: str


def _cfg(b, s, d, h, f, l, causal=True):
    return TransformerConfig(batch_size=b, seq_len=s, d_model=d, num_heads=h,
                             ffn_dim=f, num_layers=l, causal=causal)


# The five workloads this implementation is measured and parity-checked on.
# Padding ratio 0.5 draws lengths uniformly from [S/2, S] (about 25% padding),
# torch_transformer_benchmark.py:261-270.
WORKLOADS: Dict[str, Workload] = {
    "A": Workload("A", _cfg(8, 128, 128, 4, 128, 4), 1.0, 0.0,
                  "d128 h4 ffn128 L4 causal, batch 8 x seq 128, x~N(0,1), no padding"),
    "B1": Workload("B1", _cfg(4, 16, 128, 4, 128, 4), 1.0, 0.0,
                   "d128 h4 ffn128 L4 causal, batch 4 x seq 16, x~N(0,1)"),
    "B2": Workload("B2", _cfg(32, 1, 128, 4, 128, 4), 1.0, 0.0,
                   "d128 h4 ffn128 L4 causal, batch 32 x seq 1 (single token), x~N(0,1)"),
    "C": Workload("C", _cfg(32, 512, 128, 4, 128, 4), 8.0, 0.5,
                  "d128 h4 ffn128 L4 causal + key padding, batch 32 x seq 512, "
                  "lengths U[256,512], x=8*N(0,1)"),
    "D": Workload("D", _cfg(16, 1024, 512, 8, 2048, 6), 0.05, 0.0,
                  "d512 h8 ffn2048 L6 causal, batch 16 x seq 1024, x=0.05*N(0,1)"),
    "E": Workload("E", _cfg(64, 2048, 1024, 16, 4096, 12), 1.0, 0.5,
                  "d1024 h16 ffn4096 L12 causal + key padding, batch 64 x seq 2048, "
                  "lengths U[1024,2048], x~N(0,1)"),
}

# The reference's official evaluation table (tools/shapes.py:9-24): case, batch,
# d_model, heads, seq_len, layers, ffn_dim; every case causal, timed with the
# benchmark's defaults (no padding, x ~ N(0,1); torch_transformer_benchmark.py:
# 614-615). Case 14 (batch 32 x seq 100000, d_model 1024) is listed for
# completeness; its reference-side forward does not fit a host (the reference
# publishes no number for it, README.md:263-270).
OFFICIAL_TABLE = [
    (1, 64, 128, 4, 128, 4, 128),
    (2, 1, 128, 4, 128, 4, 128),
    (3, 4, 128, 4, 128, 4, 128),
    (4, 16, 128, 4, 128, 4, 128),
    (5, 128, 128, 4, 128, 4, 128),
    (6, 10000, 128, 4, 128, 4, 128),
    (7, 64, 32, 4, 128, 4, 32),
    (8, 64, 1024, 4, 128, 4, 1024),
    (9, 64, 128, 1, 128, 4, 128),
    (10, 64, 128, 2, 128, 4, 128),
    (11, 64, 128, 16, 128, 4, 128),
    (12, 64, 128, 4, 32, 4, 128),
    (13, 64, 128, 4, 1024, 4, 128),
    (14, 32, 1024, 16, 100000, 2, 1024),
]

OFFICIAL: Dict[str, Workload] = {
    f"case{c}": Workload(f"case{c}", _cfg(b, s, d, h, f, l), 1.0, 0.0,
                         f"official case {c}: d{d} h{h} ffn{f} L{l} causal, "
                         f"batch {b} x seq {s}, x~N(0,1), no padding")
    for (c, b, d, h, s, l, f) in OFFICIAL_TABLE
}

# Everything bench.py can run: the five workloads plus the official cases
# (case 14: about 105 GB of device memory, seconds per forward).
BENCH_WORKLOADS: Dict[str, Workload] = {**WORKLOADS, **OFFICIAL}

# Seeds used by the contract: model weights from torch.manual_seed(1234)
# (torch_transformer_benchmark.py:683), timing input from seed + 100000 (:533).
MODEL_SEED = 1234
TIMING_DATA_SEED = 1234 + 100000
