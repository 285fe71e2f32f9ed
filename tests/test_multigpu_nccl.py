"""The batch-sharded forward on 2 GPUs over NCCL, checked against the oracle.

Each rank runs `UserOptimizedTransformer` on its sequences of a padded batch
(the length-balanced assignment), the outputs are gathered with
`all_gather_into_tensor` over NCCL, and rank 0 checks sampled sequences of the
gathered batch against the oracle with the contract's accuracy gate
(abs <= 0.002 OR abs <= 0.02*|ref|). Skipped with fewer than 2 GPUs.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from oracle import reference_model as oracle
        from ttjam_gottagofast_b200 import UserOptimizedTransformer, compare_outputs
        from ttjam_gottagofast_b200 import generate_random_case
        from ttjam_gottagofast_b200.config import TransformerConfig
        from ttjam_gottagofast_b200.shard import balanced_assignment, sharded_forward
        cfg = TransformerConfig(batch_size=6, seq_len=256, d_model=256, num_heads=4,
                                ffn_dim=512, num_layers=2, causal=True)
        params = oracle.init_params(cfg, seed=99, device=dev)
        model = UserOptimizedTransformer(cfg).to(dev).eval()
        model.load_state_dict(params, strict=True)
        x, mask = generate_random_case(cfg, "cpu", torch.float32, 5, 0.5, 1.0)
        x, mask = x.to(dev), mask.to(dev)
        assignment = balanced_assignment(mask.sum(1).tolist(), world, cfg.seq_len)
        with torch.inference_mode():
            y = sharded_forward(model, x, mask, assignment=assignment)
        torch.cuda.synchronize(dev)
        msg = "ok"
        if rank == 0:
            picks = [0, 2, 5]
            idx = torch.tensor(picks, device=dev)
            with torch.inference_mode():
                ref = oracle.forward(params, cfg, x[idx], mask[idx])
            res = compare_outputs(ref, y[idx])
            if not res.passed or not bool((y[~mask] == 0).all()):
                msg = f"mismatch: {res}"
        q.put((rank, msg, assignment))
    except Exception as e:  # noqa: BLE001 - reported to the parent
        q.put((rank, f"error: {type(e).__name__}: {e}", None))
    finally:
        dist.destroy_process_group()


def test_sharded_forward_nccl_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    out = {}
    while not q.empty():
        r, msg, assignment = q.get()
        out[r] = msg
    assert out == {0: "ok", 1: "ok"}, out
