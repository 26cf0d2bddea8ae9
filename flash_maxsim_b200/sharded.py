"""Doc-sharded multi-GPU scoring: one process per GPU, every rank scores its
own contiguous document shard with the local kernel, and the per-rank score
blocks are combined either with one all-gather or with a per-rank top-k and a
merge. Over NCCL the gather runs on NVLink / NVSwitch.

Scores of a document do not depend on which rank holds it, so the gathered
[Nq, B] matrix is bit-identical to a single-GPU run on the whole corpus.
The reference library has no multi-GPU path; this layer sits above its API.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .api import flash_maxsim_batched, flash_maxsim_batched_topk, topk_merge_candidates


def shard_range(B: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous document range [lo, hi) of `rank`; sizes differ by at most one."""
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"rank {rank} outside world of {world}")
    return B * rank // world, B * (rank + 1) // world


def _world(group):
    return dist.get_world_size(group), dist.get_rank(group)


def _gather_padded(x: torch.Tensor, group) -> list[torch.Tensor]:
    """All-gather equal-shaped tensors; NCCL uses the single-buffer collective."""
    world, _ = _world(group)
    if dist.get_backend(group) == "nccl":
        out = torch.empty((world,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return list(out.unbind(0))
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return parts


def all_gather_scores(local: torch.Tensor, B: int, group=None) -> torch.Tensor:
    """[Nq, B_rank] per-rank scores -> [Nq, B] on every rank (shard order)."""
    world, rank = _world(group)
    lo, hi = shard_range(B, rank, world)
    if local.dim() != 2 or local.shape[1] != hi - lo:
        raise ValueError(f"rank {rank}: expected scores [Nq, {hi - lo}], got {tuple(local.shape)}")
    width = -(-B // world)  # largest shard
    if local.shape[1] < width:
        local = torch.nn.functional.pad(local, (0, width - local.shape[1]))
    parts = _gather_padded(local, group)
    cols = []
    for r, p in enumerate(parts):
        a, b = shard_range(B, r, world)
        cols.append(p[:, : b - a])
    return torch.cat(cols, dim=1)


def topk_merge(local: torch.Tensor, k: int, B: int, group=None):
    """Global top-k per query from per-rank scores [Nq, B_rank].

    Each rank keeps its own top-min(k, B_rank), the candidates (score, global
    doc id) of all ranks are all-gathered, and the merge takes the top-k of
    the world * k candidates. Ties are broken towards the lower document id.
    CUDA scores are selected and merged by the library's top-k kernels.
    Returns (values [Nq, k], doc ids int64 [Nq, k]) on every rank.
    """
    world, rank = _world(group)
    lo, hi = shard_range(B, rank, world)
    if local.dim() != 2 or local.shape[1] != hi - lo:
        raise ValueError(f"rank {rank}: expected scores [Nq, {hi - lo}], got {tuple(local.shape)}")
    if not (1 <= k <= B):
        raise ValueError(f"k={k} outside [1, {B}]")
    Nq = local.shape[0]
    kk = min(k, local.shape[1])
    if local.is_cuda:
        # per-rank selection and the final merge run as GPU kernels
        from .api import topk_merge_candidates, topk_scores
        vals = torch.full((Nq, k), float("-inf"), dtype=torch.float32, device=local.device)
        ids = torch.full((Nq, k), -1, dtype=torch.int32, device=local.device)
        if kk > 0:
            v, i = topk_scores(local, kk, id_offset=lo)
            vals[:, :kk] = v
            ids[:, :kk] = i.to(torch.int32)
        cand_v = torch.stack(_gather_padded(vals, group), dim=1)  # [Nq, world, k]
        cand_i = torch.stack(_gather_padded(ids, group), dim=1)
        return topk_merge_candidates(cand_v, cand_i, k)
    # CPU-resident scores (host-side logic, e.g. gloo ranks): the same order
    # with torch sorts
    vals = torch.full((Nq, k), float("-inf"), dtype=torch.float32, device=local.device)
    ids = torch.full((Nq, k), torch.iinfo(torch.int64).max, dtype=torch.int64, device=local.device)
    if kk > 0:
        v, i = _stable_topk(local.float(), torch.arange(lo, hi, device=local.device), kk)
        vals[:, :kk] = v
        ids[:, :kk] = i
    all_v = torch.cat(_gather_padded(vals, group), dim=1)
    all_i = torch.cat(_gather_padded(ids, group), dim=1)
    v, order = _stable_topk_idx(all_v, all_i, k)
    return v, order


def _stable_topk(scores: torch.Tensor, doc_ids: torch.Tensor, k: int):
    """Top-k by (score desc, doc id asc)."""
    return _stable_topk_idx(scores, doc_ids.expand_as(scores), k)


def _stable_topk_idx(vals: torch.Tensor, ids: torch.Tensor, k: int):
    # sort by id first, then a stable sort by score keeps ascending ids on ties
    o1 = torch.argsort(ids, dim=1, stable=True)
    v1 = torch.gather(vals, 1, o1)
    i1 = torch.gather(ids, 1, o1)
    o2 = torch.argsort(v1, dim=1, descending=True, stable=True)[:, :k]
    return torch.gather(v1, 1, o2), torch.gather(i1, 1, o2)


def sharded_maxsim_batched(Q: torch.Tensor, D_local: torch.Tensor, B: int, doc_lengths_local=None,
                           group=None, topk: int | None = None):
    """Score a doc-sharded corpus: this rank holds documents shard_range(B, ...)
    as D_local [B_rank, Ld, d]. Returns the gathered [Nq, B] scores, or the
    merged (values, doc ids) top-k when `topk` is given."""
    if topk is not None:
        world, rank = _world(group)
        lo, hi = shard_range(B, rank, world)
        Nq = Q.shape[0]
        k = int(topk)
        if not (1 <= k <= B):
            raise ValueError(f"k={k} outside [1, {B}]")
        vals = torch.full((Nq, k), float("-inf"), dtype=torch.float32, device=Q.device)
        ids = torch.full((Nq, k), -1, dtype=torch.int32, device=Q.device)
        kk = min(k, hi - lo)
        if kk > 0:
            # the scoring kernel keeps this rank's top-k itself
            v, i = flash_maxsim_batched_topk(Q, D_local, kk, doc_lengths_local)
            vals[:, :kk] = v
            ids[:, :kk] = (i + lo).to(torch.int32)
        cand_v = torch.stack(_gather_padded(vals, group), dim=1)
        cand_i = torch.stack(_gather_padded(ids, group), dim=1)
        return topk_merge_candidates(cand_v, cand_i, k)
    local = flash_maxsim_batched(Q, D_local, doc_lengths_local)
    return all_gather_scores(local, B, group)


class _SumGradAcrossRanks(torch.autograd.Function):
    """Identity forward; the backward all-reduces (sums) the gradient over the
    group, so a query shared by every rank receives the gradient of the
    scores of all shards."""

    @staticmethod
    def forward(ctx, x, group):
        ctx.group = group
        return x.view_as(x)

    @staticmethod
    def backward(ctx, grad):
        grad = grad.contiguous()
        dist.all_reduce(grad, op=dist.ReduceOp.SUM, group=ctx.group)
        return grad, None


def sum_grad_across_ranks(x: torch.Tensor, group=None) -> torch.Tensor:
    return _SumGradAcrossRanks.apply(x, group)


def sharded_maxsim_train(Q: torch.Tensor, D_local: torch.Tensor, doc_lengths_local=None, group=None):
    """Doc-sharded training forward: this rank's scores [Nq, B_rank] (or
    [B_rank] for Q [Lq, d]) of its document shard, with autograd. The
    backward gives dD for the local documents and dQ summed over all ranks
    (one NCCL all-reduce of Nq * Lq * d values), so every rank holds the same
    query gradient as a single-GPU run over the whole corpus (up to the
    order of the fp32 sums). The caller's loss must be computed on the local
    scores (or on scores gathered with torch.distributed.nn)."""
    from .api import flash_maxsim_train
    return flash_maxsim_train(sum_grad_across_ranks(Q, group), D_local, doc_lengths_local)
