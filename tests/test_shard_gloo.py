"""Batch sharding and the output gather on 2 CPU ranks (gloo), plus failure
handling: a rank that raises makes its peer fail with a timeout error instead
of hanging."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ttjam_gottagofast_b200.shard import (balanced_assignment, sequence_cost, shard_range,
                                          sharded_forward)


def test_shard_ranges_cover_batch_exactly():
    for batch in (0, 1, 7, 8, 64, 65):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for rank in range(world):
                s, c = shard_range(batch, world, rank)
                seen.extend(range(s, s + c))
            assert seen == list(range(batch))
            sizes = [shard_range(batch, world, r)[1] for r in range(world)]
            assert max(sizes) - min(sizes) <= (1 if batch else 0)
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def test_balanced_assignment_partitions_and_evens_attention_work():
    g = torch.Generator().manual_seed(3)
    for n, world in ((64, 8), (64, 2), (7, 3), (3, 4), (0, 2)):
        lengths = torch.randint(1024, 2049, (n,), generator=g).tolist()
        a = balanced_assignment(lengths, world, 2048)
        assert sorted(i for ix in a for i in ix) == list(range(n))
        assert [len(ix) for ix in a] == [shard_range(n, world, r)[1] for r in range(world)]
        assert all(ix == sorted(ix) for ix in a)
        assert a == balanced_assignment(lengths, world, 2048)  # deterministic
    lengths = torch.randint(1024, 2049, (64,), generator=g).tolist()
    work = lambda ix: sum(lengths[i] ** 2 for i in ix)  # noqa: E731
    bal = [work(ix) for ix in balanced_assignment(lengths, 8, 2048)]
    cont = [work(range(r * 8, r * 8 + 8)) for r in range(8)]
    assert max(bal) / min(bal) < 1.05
    assert max(bal) <= max(cont)


def test_sequence_cost_counts_live_row_tiles():
    # all rows without row_tile; with it, the 256-row tiles up to the last
    # valid key rounded up to 64 (1000 -> 1024 -> 4 tiles; 1025 -> 1088 -> 5)
    assert sequence_cost(1000, 2048, 0.0) == 2048
    assert sequence_cost(1000, 2048, 0.0, row_tile=256) == 1024
    assert sequence_cost(1025, 2048, 0.0, row_tile=256) == 1280
    assert sequence_cost(2048, 2048, 0.0, row_tile=256) == 2048
    assert sequence_cost(0, 2048, 0.0, row_tile=256) == 0
    # a tile size that does not divide seq_len falls back to all rows
    assert sequence_cost(100, 1000, 0.0, row_tile=256) == 1000
    assert sequence_cost(64, 128, 2.0) == 128 + 2.0 * 64 * 65 / 256


def test_balanced_assignment_with_live_rows_evens_estimated_work():
    g = torch.Generator().manual_seed(11)
    lengths = torch.randint(1024, 2049, (64,), generator=g).tolist()
    for world in (2, 4, 8):
        a = balanced_assignment(lengths, world, 2048, attn_weight=0.72, row_tile=256)
        assert sorted(i for ix in a for i in ix) == list(range(64))
        assert [len(ix) for ix in a] == [64 // world] * world
        load = [sum(sequence_cost(lengths[i], 2048, 0.72, 256) for i in ix) for ix in a]
        cont = [sum(sequence_cost(lengths[i], 2048, 0.72, 256)
                    for i in range(r * 64 // world, (r + 1) * 64 // world)) for r in range(world)]
        assert max(load) <= max(cont)
        assert max(load) / min(load) < 1.03


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _stand_in_forward(x, mask):
    # any per-sequence function stands in for the GPU forward on CPU ranks
    out = x * 2 + torch.arange(x.shape[1], dtype=x.dtype)[None, :, None]
    if mask is not None:
        out = out.masked_fill(~mask[..., None], 0)
    return out


def _worker(rank, world, port, batch, result_q, fail_rank, balanced=False):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(batch, 5, 3, generator=g)
        mask = torch.rand(batch, 5, generator=g) > 0.3
        if rank == fail_rank:
            raise RuntimeError("injected failure on the host before the gather")
        assignment = (balanced_assignment(mask.sum(1).tolist(), world, x.shape[1])
                      if balanced else None)
        y = sharded_forward(_stand_in_forward, x, mask, assignment=assignment)
        ok = torch.equal(y, _stand_in_forward(x, mask))
        result_q.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:  # noqa: BLE001 - report any failure to the parent
        result_q.put((rank, f"error: {type(e).__name__}: {e}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, batch, fail_rank=-1, timeout=60, balanced=False):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batch, q, fail_rank, balanced))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    out = {}
    while not q.empty():
        r, msg = q.get()
        out[r] = msg
    return out


@pytest.mark.parametrize("batch", [8, 7, 1])
def test_gather_reassembles_batch_on_two_ranks(batch):
    out = _run(2, batch)
    assert out == {0: "ok", 1: "ok"}, out


@pytest.mark.parametrize("batch", [8, 5])
def test_gather_undoes_balanced_assignment_on_two_ranks(batch):
    out = _run(2, batch, balanced=True)
    assert out == {0: "ok", 1: "ok"}, out


def test_failed_rank_makes_peer_error_not_hang():
    out = _run(2, 8, fail_rank=1)
    assert out[1].startswith("error: RuntimeError")
    assert 0 in out and out[0].startswith("error"), out
