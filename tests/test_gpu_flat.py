"""Parity of the flat-token batched kernel (csrc/fm_flat.cuh), selected with
fm_set_option(FM_OPT_FLAT_KERNEL, 1), against the oracle."""
import numpy as np
import pytest
import torch

from oracle import maxsim_oracle as O

CASES = [(4, 32, 300, 300, 128), (5, 64, 77, 150, 128), (4, 32, 97, 128, 128), (2, 96, 200, 257, 96),
         (3, 64, 50, 200, 64), (40, 128, 20, 300, 128), (16, 1024, 7, 1024, 128), (100, 32, 1000, 300, 128)]


@pytest.mark.gpu
@pytest.mark.parametrize("Nq,Lq,B,Ld,d", CASES)
def test_flat_kernel_vs_oracle(cuda, Nq, Lq, B, Ld, d):
    import flash_maxsim_b200 as fm
    from flash_maxsim_b200 import _lib
    Q, D = O.seeded_inputs(7 * Nq + Ld, (Nq, Lq, d), (B, Ld, d))
    _lib.set_flat_kernel(True)
    try:
        got = fm.flash_maxsim_batched(torch.from_numpy(Q).to(cuda), torch.from_numpy(D).to(cuda))
        fm.check_status(cuda)
    finally:
        _lib.set_flat_kernel(False)
    want = O.maxsim_batched(Q, D)
    np.testing.assert_allclose(got.cpu().numpy(), want, atol=1e-2, rtol=1e-3)
