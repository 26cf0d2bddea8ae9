"""fm_maxsim_bwd_noalloc: the training backward for callers that cannot
allocate device memory (they pass only the tensors they own; the library uses
its built-in 16 MiB scratch for the dQ partial sums). Where it uses the same
document ranges as the regular entry point, fm_maxsim_bwd (which takes a
caller-allocated workspace), its gradients must be bit-identical to it on two
calls in a row (the scratch is shared and keeps the previous call's contents);
where the scratch forces fewer ranges, they must match within the gradient
tolerance of the other tests.

Kept in a file of its own that pytest collects last."""
import numpy as np
import pytest
import torch

from oracle import maxsim_oracle as O

pytestmark = pytest.mark.gpu
ATOL, RTOL = 1e-2, 1e-3


def _fwd_argmax(lib, _lib, Q, D, Nq, B, Lq, Ld, d, dev):
    scores = torch.empty(Nq, B, device=dev, dtype=torch.float32)
    am = torch.empty(Nq * B, Lq, device=dev, dtype=torch.int32)
    st = torch.zeros(1, device=dev, dtype=torch.int32)
    rc = lib.fm_maxsim_fwd(Q.data_ptr(), D.data_ptr(), None, scores.data_ptr(), am.data_ptr(),
                           Nq, B, Lq, Ld, d, 1, st.data_ptr(), _lib.stream_of(dev))
    assert rc == 0
    return am


def _run(cuda, Nq, Lq, B, Ld, d, exact):
    from flash_maxsim_b200 import _lib
    lib = _lib.lib
    Qn, Dn = O.seeded_inputs(21 + Nq, (Nq, Lq, d), (B, Ld, d))
    Q = torch.from_numpy(Qn).to(cuda)
    D = torch.from_numpy(Dn).to(cuda)
    g = torch.from_numpy(np.random.default_rng(4).standard_normal((Nq, B)).astype(np.float32)).to(cuda)
    am = _fwd_argmax(lib, _lib, Q, D, Nq, B, Lq, Ld, d, cuda)
    stream = _lib.stream_of(cuda)

    need = int(lib.fm_maxsim_bwd_workspace_size(Nq, B, Lq, Ld, d))
    assert need > 0  # this shape goes through the scratch
    ws = torch.empty(need // 4, device=cuda, dtype=torch.float32)
    dQ_ref = torch.empty(Nq, Lq, d, device=cuda, dtype=torch.float16)
    dD_ref = torch.empty(B, Ld, d, device=cuda, dtype=torch.float16)
    assert lib.fm_maxsim_bwd(Q.data_ptr(), D.data_ptr(), am.data_ptr(), g.data_ptr(), dQ_ref.data_ptr(),
                             dD_ref.data_ptr(), Nq, B, Lq, Ld, d, ws.data_ptr(), need, stream) == 0

    for call in range(2):
        dQ = torch.full((Nq, Lq, d), float("nan"), device=cuda, dtype=torch.float16)
        dD = torch.full((B, Ld, d), float("nan"), device=cuda, dtype=torch.float16)
        rc = lib.fm_maxsim_bwd_noalloc(Q.data_ptr(), D.data_ptr(), am.data_ptr(), g.data_ptr(),
                                       dQ.data_ptr(), dD.data_ptr(), Nq, B, Lq, Ld, d, stream)
        assert rc == 0, _lib.status_string(rc)
        torch.cuda.synchronize(cuda)
        assert torch.equal(dD, dD_ref), f"dD, call {call}"
        if exact:
            assert torch.equal(dQ, dQ_ref), f"dQ, call {call}"
        else:
            np.testing.assert_allclose(dQ.float().cpu().numpy(), dQ_ref.float().cpu().numpy(), atol=ATOL,
                                       rtol=RTOL, err_msg=f"dQ, call {call}")


def test_noalloc_backward_matches_workspace_backward(cuda):
    # workspace of this shape fits the scratch: the same ranges, bit-identical
    _run(cuda, 2, 32, 400, 300, 128, exact=True)


def test_noalloc_backward_with_fewer_ranges(cuda):
    # the usual 5 ranges of 4 MiB partial sums do not fit 16 MiB: 4 ranges
    from flash_maxsim_b200 import _lib
    assert _lib.lib.fm_maxsim_bwd_workspace_size(64, 600, 64, 1024, 256) > 16 << 20
    _run(cuda, 64, 64, 600, 1024, 256, exact=False)


def test_noalloc_rejects_shapes_beyond_scratch(cuda):
    from flash_maxsim_b200 import _lib
    lib = _lib.lib
    # two ranges of 64 x 64 x 1024 fp32 partial sums need 32 MiB
    assert lib.fm_maxsim_bwd_workspace_size(64, 4096, 64, 1024, 1024) > 16 << 20
    t = torch.empty(16, device=cuda, dtype=torch.float16)
    rc = lib.fm_maxsim_bwd_noalloc(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(),
                                   t.data_ptr(), 64, 4096, 64, 1024, 1024, _lib.stream_of(cuda))
    assert rc == _lib.FM_ERR_SCRATCH_TOO_SMALL
    assert "16 MiB" in _lib.status_string(rc)
