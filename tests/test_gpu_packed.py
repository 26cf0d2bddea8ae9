"""Packed (unpadded) documents: flash_maxsim_packed over D_tokens [T, d] +
cu_seqlens must equal the padded path and the oracle (abs 1e-2 / rel 1e-3);
bit-identical to the padded path, since the same kernels see the same rows."""
import numpy as np
import pytest
import torch

from oracle import maxsim_oracle as O

pytestmark = pytest.mark.gpu


def dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


@pytest.mark.parametrize("Nq,Lq,B,Ld,d", [
    (1, 32, 1000, 300, 128),     # config 1 shapes (short-query kernel)
    (1, 32, 333, 520, 128),
    (100, 32, 2000, 300, 128),   # config 2 shapes (grouped documents)
    (64, 64, 120, 1024, 256),    # config 5 shapes: lengths U[32, 1024]
    (3, 17, 50, 33, 64),
    (16, 1024, 12, 1024, 128),
])
def test_packed_equals_padded_and_oracle(cuda, Nq, Lq, B, Ld, d):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(B + Ld, (Nq, Lq, d), (B, Ld, d))
    lens = np.random.default_rng(B).integers(32 if Ld >= 1024 else 0, Ld + 1, B).astype(np.int32)
    lens[1] = 0
    lens[2] = Ld
    q, dd, ln = dev(Q, cuda), dev(D, cuda), dev(lens, cuda)
    tok, cu = fm.pack_documents(dd, ln)
    assert tok.shape[0] == int(lens.sum())
    if Nq == 1:
        got = fm.flash_maxsim_packed(q[0], tok, cu)
        pad = fm.flash_maxsim(q[0], dd, ln)
        want = O.maxsim(Q[0], D, lens)
    else:
        got = fm.flash_maxsim_packed(q, tok, cu, max_len=Ld)
        pad = fm.flash_maxsim_batched(q, dd, ln)
        want = O.maxsim_batched(Q, D, lens)
    fm.check_status(cuda)
    assert torch.equal(got, pad)
    g = got.cpu().numpy()
    ninf = np.isneginf(want)
    np.testing.assert_array_equal(np.isneginf(g), ninf)
    np.testing.assert_allclose(g[~ninf], want[~ninf], atol=1e-2, rtol=1e-3)


def test_packed_offsets_not_from_zero(cuda):
    # cu_seqlens may start past row 0 and leave gaps between documents
    import flash_maxsim_b200 as fm
    Q, T = O.seeded_inputs(9, (32, 128), (5000, 128))
    cu = np.array([7, 307, 307, 1000, 1001, 4321, 4999], dtype=np.int32)
    got = fm.flash_maxsim_packed(dev(Q, cuda), dev(T, cuda), dev(cu, cuda))
    fm.check_status(cuda)
    want = np.array([O.maxsim(Q, T[None, cu[b]:cu[b + 1]])[0] if cu[b + 1] > cu[b] else -np.inf
                     for b in range(len(cu) - 1)], dtype=np.float32)
    g = got.cpu().numpy()
    np.testing.assert_array_equal(np.isneginf(g), np.isneginf(want))
    np.testing.assert_allclose(g[np.isfinite(want)], want[np.isfinite(want)], atol=1e-2, rtol=1e-3)
