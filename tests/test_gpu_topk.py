"""Top-k selection on the GPU (csrc/fm_topk.cuh and the top-k tails of the
scoring kernels). The selected ids must be exactly the stable top-k (score
descending, ties by the lower id) of the full score matrix the same kernel
writes, and those scores match the oracle within abs 1e-2 / rel 1e-3."""
import numpy as np
import pytest
import torch

from oracle import maxsim_oracle as O

pytestmark = pytest.mark.gpu


def stable_topk(scores: np.ndarray, k: int, offset: int = 0):
    order = np.lexsort((np.arange(scores.shape[-1])[None, :].repeat(scores.shape[0], 0), -scores), axis=-1)
    ids = order[:, :k]
    return np.take_along_axis(scores, ids, axis=1), ids + offset


def check(vals, ids, full, k, offset=0):
    wv, wi = stable_topk(full, k, offset)
    np.testing.assert_array_equal(ids, wi)
    np.testing.assert_array_equal(vals, wv)


def dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


@pytest.mark.parametrize("Nq,Lq,B,Ld,d,k,varlen", [
    (100, 32, 20000, 300, 128, 10, False),   # config 2 per-document shapes
    (100, 32, 3001, 300, 128, 100, True),    # B not a multiple of the document group
    (8, 32, 500, 300, 128, 500, False),      # k = B
    (3, 64, 777, 200, 96, 1, True),
    (16, 1024, 200, 1024, 128, 7, False),    # long queries and documents
    (2, 32, 5000, 64, 128, 1024, False),     # largest k
])
def test_batched_topk_exact(cuda, Nq, Lq, B, Ld, d, k, varlen):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(Nq + B, (Nq, Lq, d), (B, Ld, d))
    lens = None
    if varlen:
        lens = np.random.default_rng(1).integers(0, Ld + 1, B).astype(np.int32)
        lens[3] = 0
        lens = dev(lens, cuda)
    q, dd = dev(Q, cuda), dev(D, cuda)
    vals, ids = fm.flash_maxsim_batched_topk(q, dd, k, lens)
    full = fm.flash_maxsim_batched(q, dd, lens)
    fm.check_status(cuda)
    assert vals.shape == (Nq, k) and ids.dtype == torch.int64
    check(vals.cpu().numpy(), ids.cpu().numpy(), full.cpu().numpy(), k)


def test_topk_ties_go_to_lower_ids(cuda):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(3, (4, 32, 128), (50, 300, 128))
    D = np.concatenate([D] * 40)  # every score appears 40 times
    q, dd = dev(Q, cuda), dev(D, cuda)
    vals, ids = fm.flash_maxsim_batched_topk(q, dd, 100)
    full = fm.flash_maxsim_batched(q, dd)
    check(vals.cpu().numpy(), ids.cpu().numpy(), full.cpu().numpy(), 100)
    i = ids.cpu().numpy()
    assert (i[:, :40] % 50 == i[:, :1] % 50).all()  # the 40 copies of the best document come first


@pytest.mark.parametrize("B,k,varlen", [(1000, 10, False), (30000, 64, True), (5, 5, True)])
def test_single_query_topk(cuda, B, k, varlen):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(B, (32, 128), (B, 300, 128))
    lens = None
    if varlen:
        lens = np.random.default_rng(2).integers(0, 301, B).astype(np.int32)
        lens[0] = 0
    q, dd = dev(Q, cuda), dev(D, cuda)
    ln = None if lens is None else dev(lens, cuda)
    vals, ids = fm.flash_maxsim_topk(q, dd, k, ln)
    full = fm.flash_maxsim(q, dd, ln)
    fm.check_status(cuda)
    assert vals.shape == (k,)
    check(vals.cpu().numpy()[None], ids.cpu().numpy()[None], full.cpu().numpy()[None], k)
    want = O.maxsim(Q, D, lens)
    np.testing.assert_allclose(vals.cpu().numpy(), want[ids.cpu().numpy()], atol=1e-2, rtol=1e-3)


def test_topk_scores_of_any_matrix(cuda):
    import flash_maxsim_b200 as fm
    g = torch.Generator(device=cuda).manual_seed(0)
    s = torch.randn(7, 100000, device=cuda, generator=g)
    s[:, 500:600] = s[:, 100:200]  # ties
    s[2, 7] = float("-inf")
    for k in (1, 10, 333):
        v, i = fm.topk_scores(s, k, id_offset=1000)
        check(v.cpu().numpy(), i.cpu().numpy(), s.cpu().numpy(), k, offset=1000)
    # INT8 scores
    Q, D = O.seeded_inputs(4, (32, 128), (2000, 300, 128))
    u8, sc, mn = fm.quantize_int8(dev(D, cuda))
    s8 = fm.flash_maxsim_int8(dev(Q, cuda), u8, sc, mn)
    v, i = fm.topk_scores(s8, 25)
    check(v.cpu().numpy()[None], i.cpu().numpy()[None], s8.cpu().numpy()[None], 25)


def test_merge_candidates(cuda):
    from flash_maxsim_b200.api import topk_merge_candidates
    rng = np.random.default_rng(5)
    Nq, P, k = 5, 8, 16
    full = rng.standard_normal((Nq, P * 100)).astype(np.float32)
    full[:, 50] = full[:, 750]
    cv, ci = [], []
    for p in range(P):
        v, i = stable_topk(full[:, p * 100:(p + 1) * 100], k, offset=p * 100)
        cv.append(v)
        ci.append(i)
    cv = np.stack(cv, 1)
    ci = np.stack(ci, 1)
    v, i = topk_merge_candidates(dev(cv, cuda), dev(ci.astype(np.int32), cuda), k)
    check(v.cpu().numpy(), i.cpu().numpy(), full, k)
