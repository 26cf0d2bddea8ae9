"""Doc-sharded scoring and training over NCCL on two GPUs (skipped with one):
gathered scores and merged top-k are bit-identical to one GPU over the whole
corpus; the sharded training step gives every rank the single-GPU dQ (up to
fp32 summation order) and the local dD rows."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs(dev):
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(0)
    Q = F.normalize(torch.randn(8, 32, 128, generator=g), dim=-1).half()
    D = F.normalize(torch.randn(1001, 300, 128, generator=g), dim=-1).half()
    lens = torch.randint(1, 301, (1001,), generator=g, dtype=torch.int32)
    gr = torch.randn(8, 1001, generator=g)
    return Q.to(dev), D.to(dev), lens.to(dev), gr.to(dev)


def _worker(rank, world, port, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        from flash_maxsim_b200 import sharded
        Q, D, lens, gr = _inputs(dev)
        B = D.shape[0]
        lo, hi = sharded.shard_range(B, rank, world)
        full = sharded.sharded_maxsim_batched(Q, D[lo:hi].contiguous(), B, lens[lo:hi])
        v, i = sharded.sharded_maxsim_batched(Q, D[lo:hi].contiguous(), B, lens[lo:hi], topk=10)
        q_ = Q.clone().requires_grad_(True)
        d_ = D[lo:hi].clone().requires_grad_(True)
        s = sharded.sharded_maxsim_train(q_, d_, lens[lo:hi])
        s.backward(gr[:, lo:hi])
        torch.cuda.synchronize()
        q.put((rank, full.cpu(), v.cpu(), i.cpu(), q_.grad.float().cpu(), d_.grad.float().cpu(), lo, hi))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_sharded_two_gpus_match_one_gpu():
    import flash_maxsim_b200 as fm
    dev = torch.device("cuda", 0)
    Q, D, lens, gr = _inputs(dev)
    want = fm.flash_maxsim_batched(Q, D, lens).cpu()
    wv, wi = fm.flash_maxsim_batched_topk(Q, D, 10, lens)
    q_ = Q.clone().requires_grad_(True)
    d_ = D.clone().requires_grad_(True)
    fm.flash_maxsim_train(q_, d_, lens).backward(gr)
    ctx = mp.get_context("spawn")
    qq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, qq)) for r in range(2)]
    for p in procs:
        p.start()
    res = [qq.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, full, v, i, dq, dd, lo, hi in res:
        assert torch.equal(full, want)
        assert torch.equal(v, wv.cpu()) and torch.equal(i, wi.cpu())
        np.testing.assert_allclose(dq.numpy(), q_.grad.float().cpu().numpy(), atol=1e-2, rtol=1e-3)
        assert torch.equal(dd, d_.grad.float().cpu()[lo:hi])
