"""Official case 14 of the reference's shape table (tools/shapes.py:23):
batch 32 x seq 100000, d_model 1024, 16 heads, ffn 1024, 2 layers, causal --
3.2M tokens, the outlier of the table -- at full size through the default
schedule.

The oracle checks the first and the last sequence over all 100000 rows, on the
GPU in strict fp32, with its attention in blocks of query rows (one head's full
[S, S] score tensor would be 40 GB). Sequences are independent, so two whole
sequences check every row position, and the last one the largest offsets into
every activation buffer (x, q|k, v^T, the context, the FFN hidden state, y).

Device memory: x and y 13.1 GB each, the forward's scratch 78.6 GB, the oracle
about 30 GB afterwards.

Tolerance: the reference's accuracy gate, element-wise
abs(opt - ref) <= 0.002 OR abs(opt - ref) <= 0.02 * abs(ref), all finite
(torch_transformer_benchmark.py:309-316, defaults :618-619).
"""
import pytest
import torch

from oracle import reference_model as oracle
from ttjam_gottagofast_b200 import UserOptimizedTransformer, compare_outputs, generate_random_case
from ttjam_gottagofast_b200.config import OFFICIAL
from ttjam_gottagofast_b200.contract import ATOL, RTOL

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
NEEDED_BYTES = 120 * 10**9


def test_official_case14_full_size_two_whole_sequences():
    w = OFFICIAL["case14"]
    cfg = w.config
    assert (cfg.batch_size, cfg.seq_len, cfg.d_model, cfg.num_heads, cfg.ffn_dim,
            cfg.num_layers) == (32, 100000, 1024, 16, 1024, 2)
    torch.cuda.empty_cache()
    free, _ = torch.cuda.mem_get_info(DEV)
    if free < NEEDED_BYTES:
        pytest.skip(f"needs {NEEDED_BYTES / 1e9:.0f} GB of free device memory, "
                    f"{free / 1e9:.0f} GB free")
    old = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    try:
        params = oracle.init_params(cfg, seed=1234, device=DEV)
        model = UserOptimizedTransformer(cfg).to(DEV).eval()
        model.load_state_dict(params, strict=True)
        # generated on the device: 13 GB of input never passes through the host
        x, mask = generate_random_case(cfg, DEV, torch.float32, 101234, w.padding_ratio,
                                       w.input_scale)
        assert model.forward_plan(cfg.batch_size, cfg.seq_len) == "ops_tc"
        with torch.inference_mode():
            y = model(x, mask)
        torch.cuda.synchronize()
        assert model.read_device_status() == (0, 0)
        assert bool(torch.isfinite(y).all())
        torch.cuda.empty_cache()
        for idx in (0, cfg.batch_size - 1):
            ref = oracle.forward(params, cfg, x[idx:idx + 1], mask[idx:idx + 1],
                                 query_chunk=1024)
            res = compare_outputs(ref, y[idx:idx + 1], rtol=RTOL, atol=ATOL)
            print(f"case14/seq{idx}: max_abs={res.max_abs_error:.3e} "
                  f"max_rel={res.max_relative_error:.3e} "
                  f"failed={res.failed_elements}/{res.total_elements}")
            assert res.passed, (idx, res)
            del ref
            torch.cuda.empty_cache()
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = old
        torch.cuda.empty_cache()
