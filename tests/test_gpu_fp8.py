"""FP8 (e4m3) document storage on the GPU: quantize_fp8 must give exactly
the oracle's codes and scales, and flash_maxsim_fp8 must match maxsim_naive
on the dequantised documents within abs 1e-2 / rel 1e-3."""
import numpy as np
import pytest
import torch

from oracle import maxsim_oracle as O

pytestmark = pytest.mark.gpu


def dev(x, cuda):
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32, torch.bfloat16])
def test_quantize_fp8_bit_exact(cuda, dtype):
    import flash_maxsim_b200 as fm
    _, D = O.seeded_inputs(1, (1, 8), (300, 77, 128))
    D = torch.from_numpy(D.astype(np.float32)).to(dtype)
    D[0, 0] = 0.0  # an all-zero token: scale 1, codes 0
    codes, scales = fm.quantize_fp8(D.to(cuda))
    wv, ws = O.quantize_fp8(D.float().numpy())
    np.testing.assert_array_equal(scales.cpu().numpy(), ws)
    got = codes.cpu().view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(got, wv)
    assert codes.dtype == torch.uint8 and scales.shape == (300, 77, 1)


@pytest.mark.parametrize("Lq,B,Ld,d,varlen", [
    (32, 1000, 300, 128, False),   # config 1 / 4 shapes
    (32, 20000, 300, 128, True),   # many documents per CTA
    (64, 333, 520, 128, True),
    (17, 50, 33, 64, True),
    (32, 40, 200, 256, False),
    (1, 7, 5, 16, False),
])
def test_fp8_vs_oracle(cuda, Lq, B, Ld, d, varlen):
    import flash_maxsim_b200 as fm
    Q, D = O.seeded_inputs(Lq + B, (Lq, d), (B, Ld, d))
    lens = None
    if varlen:
        lens = np.random.default_rng(3).integers(0, Ld + 1, B).astype(np.int32)
        lens[0] = 0
    codes, scales = fm.quantize_fp8(dev(D, cuda))
    got = fm.flash_maxsim_fp8(dev(Q, cuda), codes, scales, None if lens is None else dev(lens, cuda))
    fm.check_status(cuda)
    Dq = fm.dequantize_fp8(codes, scales).cpu().numpy()
    want = O.maxsim(Q, Dq, lens)
    g = got.cpu().numpy()
    ninf = np.isneginf(want)
    np.testing.assert_array_equal(np.isneginf(g), ninf)
    np.testing.assert_allclose(g[~ninf], want[~ninf], atol=1e-2, rtol=1e-3)
    # the dequantised documents are close to the originals (e4m3: 3 mantissa bits)
    assert np.abs(Dq - D.astype(np.float32)).max() <= np.abs(D).max() / 8
