"""Doc-sharded multi-rank logic on CPU with the gloo backend (world size 2):
shard ranges, the score all-gather and the per-rank top-k merge give the
same result as one rank over the whole corpus. A rank that fails makes the
others fail fast instead of hanging."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from flash_maxsim_b200 import sharded
        B, Nq = 11, 3
        g = torch.Generator().manual_seed(0)
        full = torch.randn(Nq, B, generator=g)
        full[:, 4] = full[:, 7]  # a tie across shards
        lo, hi = sharded.shard_range(B, rank, world)
        got = sharded.all_gather_scores(full[:, lo:hi].contiguous(), B)
        v, i = sharded.topk_merge(full[:, lo:hi].contiguous(), 4, B)
        q.put((rank, torch.equal(got, full), v, i, full))
    finally:
        dist.destroy_process_group()


def test_all_gather_and_topk_merge_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same, v, i, full in res:
        assert same
        # reference: stable top-k by (score desc, doc id asc)
        order = sorted(range(full.shape[1]), key=lambda b: (-float(full[0, b]), b))[:4]
        assert i[0].tolist() == order
        assert torch.equal(v[0], full[0, order])


def test_shard_ranges_cover_corpus():
    from flash_maxsim_b200.sharded import shard_range
    for B in (0, 1, 7, 100000):
        for world in (1, 2, 3, 8):
            spans = [shard_range(B, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == B
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _failing_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from flash_maxsim_b200 import sharded
    if rank == 1:
        # this rank fails before the exchange (host-side fault injection)
        q.put((rank, "raised"))
        raise SystemExit(3)
    try:
        sharded.all_gather_scores(torch.zeros(2, 5), 10)
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "error:" + type(e).__name__))


def test_failed_rank_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "raised"
    assert res[0].startswith("error:")


def _grad_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from flash_maxsim_b200 import sharded
        x = torch.arange(6, dtype=torch.float32).reshape(2, 3).requires_grad_(True)
        y = sharded.sum_grad_across_ranks(x)
        (y * (rank + 1)).sum().backward()
        q.put((rank, x.grad.clone()))
    finally:
        dist.destroy_process_group()


def test_query_gradient_summed_over_ranks():
    # the doc-sharded training path sums dQ over ranks: rank r contributes r + 1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_grad_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, g in res:
        assert torch.equal(g, torch.full((2, 3), 3.0))
