"""INT8, sparse, training and failure-detection parity on the GPU.
Scores: abs 1e-2 / rel 1e-3; quantize_int8: bit-exact; gradients: tie-aware,
abs 1e-2 / rel 1e-3."""
import numpy as np
import pytest
import torch

from oracle import maxsim_oracle as O
from tests.conftest import golden
from tests.test_gpu_fwd import close, dev

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-2, 1e-3


# ---------------------------------------------------------------- INT8
def test_quantize_bit_exact_golden(cuda):
    import flash_maxsim_b200 as fm
    g = golden("int8")
    u8, sc, mn = fm.quantize_int8(dev(g["D"], cuda))
    assert torch.equal(u8.cpu(), torch.from_numpy(g["u8"]))
    assert torch.equal(sc.cpu().view(torch.int16), torch.from_numpy(g["scales"]).view(torch.int16))
    assert torch.equal(mn.cpu().view(torch.int16), torch.from_numpy(g["mins"]).view(torch.int16))
    # fp32 input path, d=64... and odd Ld
    u8, sc, mn = fm.quantize_int8(dev(g["D32"], cuda))
    assert torch.equal(u8.cpu(), torch.from_numpy(g["u8_32"]))
    assert torch.equal(sc.cpu().view(torch.int16), torch.from_numpy(g["scales_32"]).view(torch.int16))
    assert torch.equal(mn.cpu().view(torch.int16), torch.from_numpy(g["mins_32"]).view(torch.int16))


@pytest.mark.parametrize("shape,dtype", [((37, 300, 128), np.float16), ((5, 17, 256), np.float32),
                                         ((3, 8, 40), np.float16), ((2, 9, 2048), np.float32)])
def test_quantize_bit_exact_vs_oracle(cuda, shape, dtype):
    import flash_maxsim_b200 as fm
    (D,) = O.seeded_inputs(sum(shape), shape, dtype=dtype)
    D[0, 0] = 0.5  # constant row: scale clamps to 1e-8
    u8, sc, mn = fm.quantize_int8(dev(D, cuda))
    ou, osc, omn = O.quantize_int8(D)
    np.testing.assert_array_equal(u8.cpu().numpy(), ou)
    np.testing.assert_array_equal(sc.cpu().numpy().view(np.uint16), osc.view(np.uint16))
    np.testing.assert_array_equal(mn.cpu().numpy().view(np.uint16), omn.view(np.uint16))


@pytest.mark.parametrize("dtype", [np.float16, np.float32])
def test_quantize_bit_exact_many_rows_and_ties(cuda, dtype):
    """Many rows plus rows whose exact quotients (x - min) / scale are
    half-integers (rint ties to even): the kernel's codes must equal the IEEE
    division's everywhere."""
    import flash_maxsim_b200 as fm
    (D,) = O.seeded_inputs(11, (2048, 128, 128), dtype=dtype)
    ties = np.zeros((4, 128), dtype=np.float32)
    ties[0] = np.arange(128) + 0.5           # min 0.5, max 127.5: scale 0.5
    ties[0, 0], ties[0, 1] = 0.0, 255.0      # min 0, max 255: scale 1, quotients k + 0.5
    ties[1] = 2 * np.arange(128) + 1.0       # scale 2 (max 510): odd values -> k + 0.5
    ties[1, 0], ties[1, 1] = 0.0, 510.0
    ties[2] = np.linspace(-3, 5, 128)
    ties[3] = -ties[0]
    D[0, :4] = ties.astype(dtype)
    u8, sc, mn = fm.quantize_int8(dev(D, cuda))
    ou, osc, omn = O.quantize_int8(D)
    np.testing.assert_array_equal(u8.cpu().numpy(), ou)
    np.testing.assert_array_equal(sc.cpu().numpy().view(np.uint16), osc.view(np.uint16))
    np.testing.assert_array_equal(mn.cpu().numpy().view(np.uint16), omn.view(np.uint16))


def test_quantize_bf16(cuda):
    import flash_maxsim_b200 as fm
    (D,) = O.seeded_inputs(3, (4, 50, 128), dtype=np.float32)
    Db = torch.from_numpy(D).to(torch.bfloat16)
    u8, sc, mn = fm.quantize_int8(Db.to(cuda))
    ou, osc, omn = O.quantize_int8(Db.float().numpy())
    np.testing.assert_array_equal(u8.cpu().numpy(), ou)
    np.testing.assert_array_equal(sc.cpu().numpy().view(np.uint16), osc.view(np.uint16))


def test_int8_golden(cuda):
    import flash_maxsim_b200 as fm
    g = golden("int8")
    got = fm.flash_maxsim_int8(dev(g["Q"], cuda), dev(g["u8"], cuda), dev(g["scales"], cuda),
                               dev(g["mins"], cuda))
    close(got.cpu(), g["scores"])


@pytest.mark.parametrize("Lq,B,Ld,d,varlen", [(32, 500, 300, 128, True), (64, 33, 1024, 128, False),
                                              (200, 20, 77, 256, True), (7, 10, 40, 48, False)])
def test_int8_vs_oracle(cuda, Lq, B, Ld, d, varlen):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(Lq + B, (Lq, d), (B, Ld, d))
    u8, sc, mn = O.quantize_int8(D)
    lens = None
    if varlen:
        lens = np.random.default_rng(1).integers(0, Ld + 1, B).astype(np.int32)
    want = O.maxsim(Q, O.dequantize_int8(u8, sc, mn), lens)
    got = fm.flash_maxsim_int8(dev(Q, cuda), dev(u8, cuda), dev(sc, cuda), dev(mn, cuda),
                               None if lens is None else dev(lens, cuda))
    close(got.cpu(), want)
    # scales / mins given as [B, Ld]
    got2 = fm.flash_maxsim_int8(dev(Q, cuda), dev(u8, cuda), dev(sc[..., 0], cuda), dev(mn[..., 0], cuda),
                                None if lens is None else dev(lens, cuda))
    assert torch.equal(got, got2)


def test_int8_ranking_like_reference_test(cuda):
    # the reference's test_large_dim_int8: top-3 of fp16 and INT8 agree
    import flash_maxsim_b200 as fm
    for d in (256, 512, 1024):
        Q, D = O.seeded_inputs(d, (32, d), (20, 128, d))
        q, dd = dev(Q, cuda), dev(D, cuda)
        u8, sc, mn = fm.quantize_int8(dd)
        a = fm.flash_maxsim(q, dd).argsort(descending=True)[:3]
        b = fm.flash_maxsim_int8(q, u8, sc, mn).argsort(descending=True)[:3]
        assert torch.equal(a, b)


# ---------------------------------------------------------------- sparse
def test_sparse_golden(cuda):
    import flash_maxsim_b200 as fm
    g = golden("sparse")
    got = fm.flash_maxsim_sparse(dev(g["Q"], cuda), dev(g["D"], cuda), dev(g["indices"], cuda))
    close(got.cpu(), g["scores"])


@pytest.mark.parametrize("Lq,K,B,Ld", [(32, 8, 100, 300), (32, 32, 50, 64), (100, 37, 20, 500), (64, 70, 30, 129), (32, 0, 12, 40),
                                       (16, 3, 40, 17)])
def test_sparse_vs_oracle(cuda, Lq, K, B, Ld):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(K + Ld, (Lq, 128), (B, Ld, 128))
    rng = np.random.default_rng(K)
    idx = rng.integers(-Lq, Lq, (B, K)).astype(np.int32)  # negative ids wrap, duplicates allowed
    lens = rng.integers(0, Ld + 1, B).astype(np.int32)
    want = O.maxsim_sparse(Q, D, np.where(idx < 0, idx + Lq, idx), lens)
    got = fm.flash_maxsim_sparse(dev(Q, cuda), dev(D, cuda), dev(idx, cuda), dev(lens, cuda))
    close(got.cpu(), want)
    # the reference's own naive function on the same indices (no lengths)
    want2 = fm.maxsim_sparse_naive(dev(Q, cuda), dev(D, cuda), dev(np.where(idx < 0, idx + Lq, idx), cuda))
    got2 = fm.flash_maxsim_sparse(dev(Q, cuda), dev(D, cuda), dev(idx, cuda))
    close(got2.cpu(), want2.cpu())


def test_sparse_bad_index_reported(cuda):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(5, (8, 128), (4, 16, 128))
    idx = torch.tensor([[0, 1], [2, 99], [3, 4], [5, 6]], dtype=torch.int32, device=cuda)
    with pytest.raises(RuntimeError, match="index"):
        fm.flash_maxsim_sparse(dev(Q, cuda), dev(D, cuda), idx)
        fm.check_status(cuda)


def test_device_error_raised_on_next_call_without_sync_check(cuda, monkeypatch):
    # default behaviour: no synchronisation after the call, but the recorded
    # error reaches the host asynchronously and the next call raises
    import flash_maxsim_b200 as fm
    monkeypatch.setenv("FLASH_MAXSIM_SYNC_CHECK", "0")
    Q, D = O.seeded_inputs(5, (8, 128), (4, 16, 128))
    idx = torch.tensor([[0, 1], [2, 99], [3, 4], [5, 6]], dtype=torch.int32, device=cuda)
    fm.flash_maxsim_sparse(dev(Q, cuda), dev(D, cuda), idx)   # returns without raising
    torch.cuda.synchronize(cuda)
    with pytest.raises(RuntimeError, match="index"):
        fm.flash_maxsim(dev(Q, cuda), dev(D, cuda))
    # the word was cleared: the following calls are clean
    fm.flash_maxsim(dev(Q, cuda), dev(D, cuda))
    torch.cuda.synchronize(cuda)
    fm.flash_maxsim(dev(Q, cuda), dev(D, cuda))
    fm.check_status(cuda)


# ---------------------------------------------------------------- training
def _check_grads(Q, D, lens, g, dQ, dD, s):
    """Tie-aware gradient check: the GPU argmax must be an eps-argmax of the
    oracle scores, and the gradients must equal the closed form for the
    oracle's argmax up to rows whose top-2 gap is below eps."""
    Nq = Q.shape[0]
    am, gaps, scores = [], [], []
    for n in range(Nq):
        sc, a, gap = O.maxsim_argmax(Q[n], D, lens)
        am.append(a); gaps.append(gap); scores.append(sc)
    am = np.stack(am)          # [Nq, B, Lq]
    gaps = np.stack(gaps)
    close(s, np.stack(scores))
    if lens is not None:
        am = np.where((np.asarray(lens) == 0)[None, :, None], -1, am)
    tied = (gaps < 1e-5) & (am >= 0)
    wQ, wD = O.maxsim_grads(Q, D, am, g)
    okQ = ~tied.any(axis=1)    # [Nq, Lq] rows without near-ties in any doc
    np.testing.assert_allclose(dQ[okQ], wQ[okQ], atol=ATOL, rtol=RTOL)
    okD = np.ones(D.shape[:2], bool)
    for n, b, q in zip(*np.nonzero(tied)):
        okD[b] = False
    np.testing.assert_allclose(dD[okD], wD[okD], atol=ATOL, rtol=RTOL)


def test_train_golden(cuda):
    import flash_maxsim_b200 as fm
    gd = golden("train")
    q = dev(gd["Q"], cuda).float().requires_grad_(True)
    d = dev(gd["D"], cuda).float().requires_grad_(True)
    s = fm.flash_maxsim_train(q, d)
    (s * dev(gd["grad_scores"], cuda)).sum().backward()
    close(s.detach().cpu(), gd["scores"])
    assert q.grad.dtype == torch.float32 and d.grad.dtype == torch.float32
    np.testing.assert_allclose(q.grad.cpu().numpy(), gd["dQ"], atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(d.grad.cpu().numpy(), gd["dD"], atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("Nq,Lq,B,Ld,d,varlen", [(1, 32, 60, 300, 128, False), (3, 64, 40, 200, 128, True),
                                                 (2, 40, 16, 520, 256, True), (4, 128, 12, 96, 64, False)])
def test_train_vs_oracle(cuda, Nq, Lq, B, Ld, d, varlen):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(Nq * Lq + Ld, (Nq, Lq, d), (B, Ld, d))
    lens = None
    if varlen:
        lens = np.random.default_rng(2).integers(0, Ld + 1, B).astype(np.int32)
        lens[0] = 0
    g = np.random.default_rng(3).standard_normal((Nq, B)).astype(np.float32)
    q = dev(Q, cuda).requires_grad_(True)
    dd = dev(D, cuda).requires_grad_(True)
    s = fm.flash_maxsim_train(q, dd, None if lens is None else dev(lens, cuda))
    s.backward(dev(g, cuda))
    gg = np.where(np.isfinite(s.detach().cpu().numpy()), g, 0.0).astype(np.float32)
    if lens is not None:
        # an empty document scores -inf: no gradient flows to it
        g = gg
    _check_grads(Q, D, lens, g, q.grad.float().cpu().numpy(), dd.grad.float().cpu().numpy(),
                 s.detach().cpu().numpy())


def test_train_deterministic(cuda):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(9, (2, 32, 128), (50, 100, 128))
    outs = []
    for _ in range(2):
        q = dev(Q, cuda).requires_grad_(True)
        dd = dev(D, cuda).requires_grad_(True)
        fm.flash_maxsim_train(q, dd).sum().backward()
        outs.append((q.grad.clone(), dd.grad.clone()))
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


# ---------------------------------------------------------------- failure detection
def test_bounded_wait_reports_timeout(cuda):
    """A device wait that nothing satisfies gives up after its limit and
    reports through the status word; the context stays usable."""
    import flash_maxsim_b200 as fm
    from flash_maxsim_b200 import _lib
    st = torch.zeros(1, dtype=torch.int32, device=cuda)
    rc = _lib.lib.fm_wait_selftest(st.data_ptr(), 2_000_000, _lib.stream_of(cuda))  # 2 ms
    assert rc == 0
    torch.cuda.synchronize(cuda)
    assert int(st.item()) == _lib.FM_ERR_TIMEOUT_SELFTEST
    # still usable afterwards
    Q, D = O.seeded_inputs(1, (32, 128), (4, 20, 128))
    close(fm.flash_maxsim(dev(Q, cuda), dev(D, cuda)).cpu(), O.maxsim(Q, D))


def test_backward_ignores_out_of_range_argmax(cuda):
    # argmax entries outside [0, Ld) (here Ld and Ld + 7) contribute nothing to
    # dQ or dD, and are never read: the C entry point takes argmax from callers
    from flash_maxsim_b200 import _lib
    Nq, Lq, B, Ld, d = 2, 32, 40, 100, 128
    Q, D = O.seeded_inputs(31, (Nq, Lq, d), (B, Ld, d))
    am = np.random.default_rng(5).integers(0, Ld, (Nq, B, Lq)).astype(np.int32)
    am[0, 3, 5] = Ld
    am[1, B - 1, 0] = Ld + 7
    am[1, 7, 9] = -1
    g = np.random.default_rng(6).standard_normal((Nq, B)).astype(np.float32)
    dQ = torch.empty(Nq, Lq, d, device=cuda, dtype=torch.float16)
    dD = torch.empty(B, Ld, d, device=cuda, dtype=torch.float16)
    q, dd, a, gg = dev(Q, cuda), dev(D, cuda), dev(am, cuda), dev(g, cuda)
    need = int(_lib.lib.fm_maxsim_bwd_workspace_size(Nq, B, Lq, Ld, d))
    ws = torch.empty(max(need, 16) // 4, device=cuda, dtype=torch.float32)
    rc = _lib.lib.fm_maxsim_bwd(q.data_ptr(), dd.data_ptr(), a.data_ptr(), gg.data_ptr(), dQ.data_ptr(),
                                dD.data_ptr(), Nq, B, Lq, Ld, d, ws.data_ptr(), max(need, 16), _lib.stream_of(cuda))
    assert rc == 0
    torch.cuda.synchronize(cuda)
    am_ok = np.where((am >= 0) & (am < Ld), am, -1)
    wQ, wD = O.maxsim_grads(Q, D, am_ok, g)
    np.testing.assert_allclose(dQ.float().cpu().numpy(), wQ, atol=ATOL, rtol=RTOL)
    np.testing.assert_allclose(dD.float().cpu().numpy(), wD, atol=ATOL, rtol=RTOL)
