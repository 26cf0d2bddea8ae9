"""Forward parity on the GPU: sm_100a kernels vs the oracle and the
reference's golden vectors. Tolerance (north star): abs 1e-2, rel 1e-3."""
import numpy as np
import pytest
import torch

from oracle import maxsim_oracle as O
from tests.conftest import golden

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-2, 1e-3


def close(got, want):
    got = np.asarray(got, dtype=np.float32)
    want = np.asarray(want, dtype=np.float32)
    assert got.shape == want.shape
    ninf = np.isneginf(want)
    np.testing.assert_array_equal(np.isneginf(got), ninf)
    np.testing.assert_allclose(got[~ninf], want[~ninf], atol=ATOL, rtol=RTOL)


def dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


def test_golden_textual(cuda):
    import flash_maxsim_b200 as fm
    g = golden("textual")
    Q, D = dev(g["Q"], cuda), dev(g["D"], cuda)
    close(fm.flash_maxsim(Q, D).cpu(), g["scores"])
    close(fm.flash_maxsim(Q, D, doc_lengths=dev(g["lengths"], cuda)).cpu(), g["scores_len"])


def test_golden_batched(cuda):
    import flash_maxsim_b200 as fm
    g = golden("batched")
    Q, D = dev(g["Q"], cuda), dev(g["D"], cuda)
    close(fm.flash_maxsim_batched(Q, D).cpu(), g["scores"])
    Dq = D.unsqueeze(0).expand(5, -1, -1, -1).contiguous()
    close(fm.flash_maxsim_batched(Q, Dq, shared_docs=False).cpu(), g["scores"])


def test_golden_large_d(cuda):
    import flash_maxsim_b200 as fm
    g = golden("large_d")
    for d in (256, 512, 1024, 2048):
        close(fm.flash_maxsim(dev(g[f"Q{d}"], cuda), dev(g[f"D{d}"], cuda)).cpu(), g[f"s{d}"])


@pytest.mark.parametrize("Nq,Lq,B,Ld,d,varlen", [
    (1, 32, 1000, 300, 128, False),   # BASELINE config 1 shape
    (1, 32, 333, 300, 128, True),
    (1, 1, 7, 5, 128, False),         # tiny
    (1, 17, 50, 33, 64, True),        # odd Lq / Ld, one K atom
    (1, 64, 40, 1024, 128, True),     # long docs, 4 chunks
    (1, 128, 30, 512, 128, False),
    (3, 32, 77, 300, 128, True),      # 3 row groups (no replication)
    (2, 48, 64, 200, 96, True),       # d=96: padded K atom
    (8, 32, 100, 300, 128, True),     # 2 M-blocks
    (5, 100, 40, 260, 128, True),     # ragged row groups
    (2, 256, 24, 300, 128, False),    # Lq > 128
    (4, 1024, 6, 1024, 128, False),   # visual-like, chunk groups + state
    (3, 64, 20, 700, 256, True),      # d=256: K split over two Q stages
    (2, 40, 10, 129, 320, True),      # d=320: odd atom count
    # single short query (document chunk as the M operand)
    (1, 40, 50, 513, 128, True),      # 64-column query, 3 chunks, ragged last chunk
    (1, 8, 20, 1, 32, False),         # d=32 (half atom), one-token documents
    (1, 64, 600, 256, 128, True),     # chunk-sized documents, many docs per CTA
    (1, 33, 20, 257, 120, True),      # d=120, one token past a chunk
    (1, 32, 2000, 77, 128, True),     # short documents, > 8 documents per exchange slot cycle
    # flat token stream (no lengths, whole row groups, >= 128 query rows)
    (4, 32, 300, 300, 128, False),    # documents straddle 224-token chunks
    (5, 64, 77, 150, 128, False),     # several documents end in one item
    (4, 32, 97, 128, 128, False),     # shortest flat documents: two ends in one chunk
    (4, 32, 61, 130, 128, False),
    (2, 96, 200, 257, 96, False),     # d=96, odd Ld
    (3, 64, 50, 200, 64, False),      # one K atom, 256-token chunks
    (40, 128, 20, 300, 128, False),   # 160 row groups: two query spans
    (16, 1024, 7, 1024, 128, False),  # long queries, spans of 4 queries
    (100, 32, 1000, 300, 128, False), # config-2 shapes, few documents per CTA
])
def test_batched_vs_oracle(cuda, Nq, Lq, B, Ld, d, varlen):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(100 + Nq * Lq + Ld, (Nq, Lq, d), (B, Ld, d))
    lens = None
    if varlen:
        lens = np.random.default_rng(B).integers(0, Ld + 1, B).astype(np.int32)
        lens[0] = 0
        lens[-1] = Ld
    want = O.maxsim_batched(Q, D, lens)
    got = fm.flash_maxsim_batched(dev(Q, cuda), dev(D, cuda),
                                  None if lens is None else dev(lens, cuda)).cpu()
    close(got, want)
    if Nq == 1:
        got1 = fm.flash_maxsim(dev(Q[0], cuda), dev(D, cuda),
                               None if lens is None else dev(lens, cuda)).cpu()
        close(got1, want[0])


@pytest.mark.parametrize("Nq,Lq,B,Ld,d", [(4, 32, 30, 300, 128), (3, 70, 11, 500, 128)])
def test_per_query_docs(cuda, Nq, Lq, B, Ld, d):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(7, (Nq, Lq, d), (Nq, B, Ld, d))
    lens = np.random.default_rng(3).integers(1, Ld + 1, Nq * B).astype(np.int32)
    want = O.maxsim_batched(Q, D, lens, shared_docs=False)
    got = fm.flash_maxsim_batched(dev(Q, cuda), dev(D, cuda), dev(lens, cuda), shared_docs=False)
    close(got.cpu(), want)


def test_lengths_clamped_and_negative(cuda):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(11, (32, 128), (6, 100, 128))
    lens = np.array([-5, 0, 1, 100, 1000, 50], dtype=np.int32)
    want = O.maxsim(Q, D, np.clip(lens, 0, 100))
    close(fm.flash_maxsim(dev(Q, cuda), dev(D, cuda), dev(lens, cuda)).cpu(), want)


def test_fp32_and_bf16_inputs_cast_like_reference(cuda):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(12, (32, 128), (20, 64, 128), dtype=np.float32)
    want = O.maxsim(Q.astype(np.float16), D.astype(np.float16))
    close(fm.flash_maxsim(dev(Q, cuda), dev(D, cuda)).cpu(), want)


def test_noncontiguous_and_offset_views(cuda):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(13, (32, 128), (21, 64, 128))
    Dt = dev(D, cuda)
    view = Dt[1:]                        # storage offset 64*128*2 bytes
    tview = dev(Q, cuda).t().contiguous().t()  # non-contiguous
    close(fm.flash_maxsim(tview, view).cpu(), O.maxsim(Q, D[1:]))


def test_determinism(cuda):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(14, (8, 64, 128), (200, 300, 128))
    q, d_ = dev(Q, cuda), dev(D, cuda)
    a = fm.flash_maxsim_batched(q, d_)
    b = fm.flash_maxsim_batched(q, d_)
    assert torch.equal(a, b)


def test_empty_batch(cuda):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(15, (32, 128), (1, 8, 128))
    out = fm.flash_maxsim(dev(Q, cuda), dev(D, cuda)[:0])
    assert out.shape == (0,)


@pytest.mark.parametrize("pinned,lengths", [(True, True), (True, False), (False, True)])
def test_batched_from_host_streams_pieces(cuda, pinned, lengths):
    # documents in host memory, copied in ~23 pieces through two device
    # buffers while earlier pieces are scored: the same scores as one call on
    # the whole device-resident corpus, and the oracle agrees
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(31, (3, 32, 128), (3000, 300, 128))
    lens = np.random.default_rng(5).integers(0, 301, 3000).astype(np.int32) if lengths else None
    hD = torch.from_numpy(D).half()
    if pinned:
        hD = hD.pin_memory()
    hQ = torch.from_numpy(Q).half()
    want = fm.flash_maxsim_batched(hQ.to(cuda), hD.to(cuda), None if lens is None else dev(lens, cuda))
    got = fm.flash_maxsim_batched_from_host(hQ, hD, None if lens is None else torch.from_numpy(lens),
                                            piece_bytes=10 << 20, nbuf=2, device=cuda)
    assert got.device == want.device
    assert torch.equal(got, want)
    close(got[:, :200].cpu(), O.maxsim_batched(Q, D[:200], None if lens is None else lens[:200]))
