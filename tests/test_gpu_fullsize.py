"""Parity at the BASELINE configurations' own per-document shapes, with
enough documents that every persistent CTA loops over many work items (ring
phases wrap many times): each launch covers the whole batch, and a seeded
sample of its documents is checked against the CPU oracle
(oracle/sampled_check.py). Tolerance: abs 1e-2 / rel 1e-3 on scores and
gradients; the training check is tie-aware."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import sampled_check as SC

pytestmark = pytest.mark.gpu


def synth(shape, seed, dev):
    """N(0, 1) rows, L2-normalised, fp16, from a seeded device generator."""
    g = torch.Generator(device=dev).manual_seed(seed)
    out = torch.empty(shape, dtype=torch.float16, device=dev)
    flat = out.view(-1, shape[-1])
    step = 1 << 20
    for r0 in range(0, flat.shape[0], step):
        n = min(step, flat.shape[0] - r0)
        flat[r0:r0 + n] = F.normalize(torch.randn(n, shape[-1], generator=g, device=dev), dim=-1).half()
    return out


def _np(t):
    return t.detach().cpu().numpy()


def _assert_ok(res):
    assert res["ok"], res


@pytest.mark.parametrize("Nq,Lq,B,Ld,d,varlen", [
    (100, 32, 20000, 300, 128, False),   # config 2 per-document shapes
    (100, 32, 20000, 300, 128, True),
    (1, 32, 30000, 300, 128, False),     # config 1 shapes, many docs per CTA
    (1, 32, 30000, 300, 128, True),
])
def test_fullsize_batched(cuda, Nq, Lq, B, Ld, d, varlen):
    import flash_maxsim_b200 as fm
    Q = synth((Nq, Lq, d), 1, cuda)
    D = synth((B, Ld, d), 2, cuda)
    lens = None
    if varlen:
        gl = torch.Generator(device=cuda).manual_seed(3)
        lens = torch.randint(0, Ld + 1, (B,), generator=gl, device=cuda, dtype=torch.int32)
    if Nq == 1:
        got = fm.flash_maxsim(Q[0], D, lens).unsqueeze(0)
    else:
        got = fm.flash_maxsim_batched(Q, D, lens)
    fm.check_status(cuda)
    idx = SC.sample_docs(B, 256, seed=B + Nq)
    it = torch.from_numpy(idx).to(cuda)
    res = SC.check_scores(_np(Q), _np(D[it]), _np(got[:, it]), None if lens is None else _np(lens[it]))
    _assert_ok(res)


def test_fullsize_visual(cuda):
    # config 3 per-document shapes (Lq = Ld = 1024), 1200 documents
    import flash_maxsim_b200 as fm
    Nq, Lq, B, Ld, d = 16, 1024, 1200, 1024, 128
    Q = synth((Nq, Lq, d), 4, cuda)
    D = synth((B, Ld, d), 5, cuda)
    got = fm.flash_maxsim_batched(Q, D)
    fm.check_status(cuda)
    idx = SC.sample_docs(B, 24, seed=7)
    it = torch.from_numpy(idx).to(cuda)
    _assert_ok(SC.check_scores(_np(Q), _np(D[it]), _np(got[:, it])))


def test_fullsize_int8(cuda):
    # config 4 per-document shapes, 50000 documents
    import flash_maxsim_b200 as fm
    Lq, B, Ld, d = 32, 50000, 300, 128
    Q = synth((Lq, d), 6, cuda)
    D = synth((B, Ld, d), 7, cuda)
    u8, sc, mn = fm.quantize_int8(D)
    del D
    got = fm.flash_maxsim_int8(Q, u8, sc, mn)
    fm.check_status(cuda)
    idx = SC.sample_docs(B, 256, seed=8)
    it = torch.from_numpy(idx).to(cuda)
    _assert_ok(SC.check_int8(_np(Q), _np(u8[it]), _np(sc[it]), _np(mn[it]), _np(got[it])))


@pytest.mark.parametrize("Lq", [32, 64])
def test_int8_many_docs_per_cta_varlen(cuda, Lq):
    # the short-query INT8 kernel's per-document exchange slots (8 per CTA)
    # wrap many times: 3000 documents over 148 CTAs, ragged lengths with
    # empty documents, for both epilogue layouts (8 warps for 32 query rows,
    # 4 warps for 64)
    import flash_maxsim_b200 as fm
    B, Ld, d = 3000, 300, 128
    Q = synth((Lq, d), 16 + Lq, cuda)
    D = synth((B, Ld, d), 17, cuda)
    u8, sc, mn = fm.quantize_int8(D)
    del D
    lens = np.random.default_rng(Lq).integers(0, Ld + 1, B).astype(np.int32)
    idx = SC.sample_docs(B, 256, seed=9)
    lens[idx[::5]] = 0
    lens[idx[1::5]] = 44  # as long as the tail chunk of a 300-token document
    got = fm.flash_maxsim_int8(Q, u8, sc, mn, torch.from_numpy(lens).to(cuda))
    fm.check_status(cuda)
    it = torch.from_numpy(idx).to(cuda)
    _assert_ok(SC.check_int8(_np(Q), _np(u8[it]), _np(sc[it]), _np(mn[it]), _np(got[it]), lens[idx]))


def test_fullsize_train(cuda):
    # config 5 shapes: Nq=64, Lq=64, d=256, Ld=1024, lengths U[32, 1024], 600 docs
    import flash_maxsim_b200 as fm
    from flash_maxsim_b200 import api
    Nq, Lq, B, Ld, d = 64, 64, 600, 1024, 256
    Q = synth((Nq, Lq, d), 9, cuda)
    D = synth((B, Ld, d), 10, cuda)
    gl = torch.Generator(device=cuda).manual_seed(11)
    lens = torch.randint(32, Ld + 1, (B,), generator=gl, device=cuda, dtype=torch.int32)
    lens[5] = 0  # one empty document
    g = torch.randn(Nq, B, device=cuda, generator=torch.Generator(device=cuda).manual_seed(12))
    q = Q.clone().requires_grad_(True)
    dd = D.clone().requires_grad_(True)
    s = fm.flash_maxsim_train(q, dd, lens)
    s.backward(g)
    fm.check_status(cuda)
    # the same forward with the argmax exposed (deterministic: identical launch)
    s2, am = api._fwd(Q, D, lens, Nq, B, Lq, Ld, True, True)
    assert torch.equal(s.detach(), s2)
    am = am.view(Nq, B, Lq)
    idx = SC.sample_docs(B, 32, seed=13)
    idx = np.union1d(idx, [5])
    it = torch.from_numpy(idx).to(cuda)
    rows = [(0, 0), (7, 63), (31, 17), (63, 40)]
    Dsel = []
    for n, qq in rows:
        a = am[n, :, qq].long()
        sel = D[torch.arange(B, device=cuda), a.clamp(min=0)].float()
        Dsel.append(_np(torch.where((a >= 0)[:, None], sel, torch.zeros_like(sel))))
    g_eff = torch.where(torch.isfinite(s.detach()), g, torch.zeros_like(g))
    res = SC.check_train(_np(Q), _np(D[it]), _np(lens[it]), _np(g[:, it]), _np(s.detach()[:, it]),
                         _np(am[:, it]), _np(dd.grad[it].float()), rows,
                         np.stack([_np(q.grad[n, qq].float()) for n, qq in rows]),
                         (_np(g_eff), Dsel))
    _assert_ok(res)
