"""ORACLE -- test infrastructure only.

A restatement of the reference forward pass (`BaselineTransformer.forward`,
torch_transformer_benchmark.py:59-172) as plain functions over a state dict,
op for op in the reference's order, in fp32 torch eager. It is the checker for
the CUDA path and the timed CPU baseline, and nothing else: only `tests/`,
`__graft_entry__.smoke()` and `bench.py` (its `cpu_baseline` leg and its
`--impl reference` arm) may import it. The product path never calls it.

Parity pin: `tests/golden/*.npz` hold outputs of the reference module itself
(imported from the reference source tree by `tests/golden/make_golden.py`) on
seeded inputs; `tests/test_oracle_golden.py` checks this restatement against
them. The restatement keeps the reference's arithmetic exactly (explicit
[B,H,S,S] scores, scale applied after the matmul, -inf masks, fp32 softmax), so
on CPU it reproduces the goldens to rounding.

`batch_chunk` runs the batch in slices (sequences are independent), which
bounds the [B,H,S,S] score tensor at large sizes without changing any value;
`query_chunk` runs each attention in blocks of query rows (every row's softmax
is its own), which bounds it for sequences too long for one [S,S] tensor.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn.functional as F


def layer_norm(x, weight, bias, eps: float = 1e-5):
    """nn.LayerNorm(d_model) with default eps=1e-5, biased variance
    (torch_transformer_benchmark.py:128,130,160)."""
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def _attention_query_chunks(q, k, v, mask, causal: bool, scale: float, chunk: int):
    """The same scores / masks / softmax / P.V as the full [B,H,S,S] form
    (torch_transformer_benchmark.py:97-112), one block of `chunk` query rows
    at a time. Each query row's softmax depends only on its own scores, so the
    values are those of the full form; under the causal mask a block's keys
    stop at its last query (later keys get -inf, hence probability 0). Only
    the [B,H,chunk,S] scores of one block are held, which is what makes
    sequences of 1e5 tokens checkable."""
    s = q.shape[2]
    out = []
    for q0 in range(0, s, chunk):
        q1 = min(s, q0 + chunk)
        kend = q1 if causal else s
        scores = torch.matmul(q[:, :, q0:q1], k[:, :, :kend].transpose(-2, -1)) * scale
        if causal:
            qi = torch.arange(q0, q1, device=q.device)[:, None]
            kj = torch.arange(kend, device=q.device)[None, :]
            scores = scores.masked_fill(kj > qi, float("-inf"))
        if mask is not None:
            scores = scores.masked_fill(~mask[:, None, None, :kend], float("-inf"))
        probs = torch.softmax(scores.float(), dim=-1).to(dtype=q.dtype)
        del scores
        out.append(torch.matmul(probs, v[:, :, :kend]))
        del probs
    return torch.cat(out, 2)


def self_attention(p: Dict[str, torch.Tensor], prefix: str, x, mask, causal: bool,
                   num_heads: int, query_chunk: Optional[int] = None):
    """BaselineSelfAttention.forward, torch_transformer_benchmark.py:85-122.
    With `query_chunk`, the attention core runs in blocks of query rows
    (_attention_query_chunks); everything else is unchanged."""
    b, s, d = x.shape
    hd = d // num_heads
    scale = hd ** -0.5                                         # :70

    def split(t):                                              # :77-83
        return t.view(b, s, num_heads, hd).transpose(1, 2).contiguous()

    q = split(F.linear(x, p[prefix + "q_proj.weight"], p[prefix + "q_proj.bias"]))
    k = split(F.linear(x, p[prefix + "k_proj.weight"], p[prefix + "k_proj.bias"]))
    v = split(F.linear(x, p[prefix + "v_proj.weight"], p[prefix + "v_proj.bias"]))
    if query_chunk is None or query_chunk >= s:
        scores = torch.matmul(q, k.transpose(-2, -1)) * scale      # :97
        if causal:                                                 # :99-103
            cm = torch.ones((s, s), device=x.device, dtype=torch.bool).triu(diagonal=1)
            scores = scores.masked_fill(cm, float("-inf"))
        if mask is not None:                                       # :105-108
            scores = scores.masked_fill(~mask[:, None, None, :], float("-inf"))
        probs = torch.softmax(scores.float(), dim=-1).to(dtype=x.dtype)   # :111
        ctx = torch.matmul(probs, v)                               # :112
    else:
        ctx = _attention_query_chunks(q, k, v, mask, causal, scale, query_chunk)
    ctx = ctx.transpose(1, 2).contiguous().view(b, s, d)       # :113-117
    out = F.linear(ctx, p[prefix + "out_proj.weight"], p[prefix + "out_proj.bias"])
    if mask is not None:                                       # :120-121
        out = out.masked_fill(~mask[..., None], 0)
    return out


def block(p, prefix: str, x, mask, causal: bool, num_heads: int,
          query_chunk: Optional[int] = None):
    """BaselineTransformerBlock.forward, torch_transformer_benchmark.py:134-145."""
    n1 = layer_norm(x, p[prefix + "norm1.weight"], p[prefix + "norm1.bias"])
    x = x + self_attention(p, prefix + "attention.", n1, mask, causal, num_heads, query_chunk)
    n2 = layer_norm(x, p[prefix + "norm2.weight"], p[prefix + "norm2.bias"])
    h = F.gelu(F.linear(n2, p[prefix + "ffn_in.weight"], p[prefix + "ffn_in.bias"]),
               approximate="none")
    x = x + F.linear(h, p[prefix + "ffn_out.weight"], p[prefix + "ffn_out.bias"])
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
    return x


def _forward(p, cfg, x, mask, query_chunk=None):
    for i in range(cfg.num_layers):                            # :167-168
        x = block(p, f"layers.{i}.", x, mask, cfg.causal, cfg.num_heads, query_chunk)
    x = layer_norm(x, p["final_norm.weight"], p["final_norm.bias"])   # :169
    if mask is not None:                                       # :170-171
        x = x.masked_fill(~mask[..., None], 0)
    return x


@torch.inference_mode()
def forward(params: Dict[str, torch.Tensor], cfg, x: torch.Tensor,
            mask: Optional[torch.Tensor] = None, batch_chunk: Optional[int] = None,
            query_chunk: Optional[int] = None):
    """BaselineTransformer.forward (torch_transformer_benchmark.py:162-172) over a
    state dict with the reference's parameter names. `batch_chunk` slices the
    batch, `query_chunk` the query rows of each attention."""
    if batch_chunk is None or batch_chunk >= x.shape[0]:
        return _forward(params, cfg, x, mask, query_chunk)
    outs = []
    for b0 in range(0, x.shape[0], batch_chunk):
        m = None if mask is None else mask[b0:b0 + batch_chunk]
        outs.append(_forward(params, cfg, x[b0:b0 + batch_chunk], m, query_chunk))
    return torch.cat(outs, 0)


def init_params(cfg, seed: int = 1234, device="cpu") -> Dict[str, torch.Tensor]:
    """Weights exactly as `torch.manual_seed(seed); BaselineTransformer(cfg)` draws
    them (torch_transformer_benchmark.py:683,690): nn.Linear default init
    (kaiming-uniform weight, U(+-1/sqrt(fan_in)) bias) in module-construction
    order, LayerNorm weight 1 / bias 0."""
    torch.manual_seed(seed)
    d, f = cfg.d_model, cfg.ffn_dim
    p: Dict[str, torch.Tensor] = {}

    def lin(name, fan_in, fan_out):
        m = torch.nn.Linear(fan_in, fan_out)
        p[name + ".weight"] = m.weight.detach()
        p[name + ".bias"] = m.bias.detach()

    for i in range(cfg.num_layers):
        pre = f"layers.{i}."
        p[pre + "norm1.weight"] = torch.ones(d)
        p[pre + "norm1.bias"] = torch.zeros(d)
        for name in ("q_proj", "k_proj", "v_proj", "out_proj"):
            lin(pre + "attention." + name, d, d)
        p[pre + "norm2.weight"] = torch.ones(d)
        p[pre + "norm2.bias"] = torch.zeros(d)
        lin(pre + "ffn_in", d, f)
        lin(pre + "ffn_out", f, d)
    p["final_norm.weight"] = torch.ones(d)
    p["final_norm.bias"] = torch.zeros(d)
    return {k: v.to(device) for k, v in p.items()}
