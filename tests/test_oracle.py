"""The numpy oracle against the reference's own outputs (tests/golden)."""
import numpy as np

from oracle import maxsim_oracle as O
from tests.conftest import golden

ATOL, RTOL = 1e-4, 1e-5  # fp32 vs fp32: only summation order differs


def test_textual_full_and_lengths():
    g = golden("textual")
    np.testing.assert_allclose(O.maxsim(g["Q"], g["D"]), g["scores"], atol=ATOL, rtol=RTOL)
    got = O.maxsim(g["Q"], g["D"], g["lengths"])
    want = g["scores_len"]
    assert np.isneginf(want[0]) and np.isneginf(got[0])  # empty document
    np.testing.assert_allclose(got, want, atol=ATOL, rtol=RTOL)


def test_chunking_invariance():
    g = golden("textual")
    a = O.maxsim(g["Q"], g["D"], g["lengths"], doc_chunk=5)
    b = O.maxsim(g["Q"], g["D"], g["lengths"], doc_chunk=1000)
    np.testing.assert_array_equal(a, b)


def test_batched():
    g = golden("batched")
    np.testing.assert_allclose(O.maxsim_batched(g["Q"], g["D"]), g["scores"], atol=ATOL, rtol=RTOL)
    # per-query docs: the same docs repeated per query give the same scores
    Dq = np.broadcast_to(g["D"][None], (5,) + g["D"].shape)
    np.testing.assert_allclose(O.maxsim_batched(g["Q"], Dq, shared_docs=False), g["scores"],
                               atol=ATOL, rtol=RTOL)


def test_quantize_bit_exact_fp16_and_fp32():
    g = golden("int8")
    u8, sc, mn = O.quantize_int8(g["D"])
    np.testing.assert_array_equal(u8, g["u8"])
    np.testing.assert_array_equal(sc.view(np.uint16), g["scales"].view(np.uint16))
    np.testing.assert_array_equal(mn.view(np.uint16), g["mins"].view(np.uint16))
    u8, sc, mn = O.quantize_int8(g["D32"])
    np.testing.assert_array_equal(u8, g["u8_32"])
    np.testing.assert_array_equal(sc.view(np.uint16), g["scales_32"].view(np.uint16))
    np.testing.assert_array_equal(mn.view(np.uint16), g["mins_32"].view(np.uint16))


def test_dequant_and_int8_scores():
    g = golden("int8")
    deq = O.dequantize_int8(g["u8"], g["scales"], g["mins"])
    np.testing.assert_array_equal(deq, g["deq"])
    np.testing.assert_allclose(O.maxsim(g["Q"], deq), g["scores"], atol=ATOL, rtol=RTOL)


def test_sparse():
    g = golden("sparse")
    np.testing.assert_allclose(O.maxsim_sparse(g["Q"], g["D"], g["indices"]), g["scores"],
                               atol=ATOL, rtol=RTOL)


def test_train_grads():
    g = golden("train")
    s, am, gap = O.maxsim_argmax(g["Q"], g["D"])
    np.testing.assert_allclose(s, g["scores"], atol=ATOL, rtol=RTOL)
    assert (gap > 0).all()  # no exact ties in this fixture: argmax is unique
    dQ, dD = O.maxsim_grads(g["Q"][None], g["D"], am[None], g["grad_scores"][None])
    np.testing.assert_allclose(dQ[0], g["dQ"], atol=1e-5, rtol=1e-5)
    np.testing.assert_allclose(dD, g["dD"], atol=1e-5, rtol=1e-5)


def test_large_d():
    g = golden("large_d")
    for d in (256, 512, 1024, 2048):
        np.testing.assert_allclose(O.maxsim(g[f"Q{d}"], g[f"D{d}"]), g[f"s{d}"], atol=ATOL, rtol=RTOL)


def test_argmax_first_occurrence():
    Q = np.array([[1.0, 0.0]], dtype=np.float32)
    D = np.array([[[0.5, 0.0], [1.0, 0.0], [1.0, 0.0], [0.2, 0.0]]], dtype=np.float32)
    s, am, gap = O.maxsim_argmax(Q, D)
    assert am[0, 0] == 1 and s[0] == 1.0 and gap[0, 0] == 0.0
    s, am, _ = O.maxsim_argmax(Q, D, doc_lengths=np.array([1]))
    assert am[0, 0] == 0 and s[0] == 0.5


def test_e4m3_rounding_matches_torch():
    # the oracle's e4m3 rounding (FP8 document format) against torch's own
    # float8_e4m3fn conversion: random values over many scales, every exact
    # midpoint between neighbouring codes (ties to even) and every code
    import torch
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-4, 1e-2, 1.0, 50.0)])
    x = x[np.abs(x) <= 448]
    grid = torch.arange(0, 256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    grid = np.unique(grid[np.isfinite(grid)])
    mids = ((grid[1:] + grid[:-1]) / 2).astype(np.float32)
    x = np.concatenate([x, mids, -mids, grid, -grid])
    want = torch.from_numpy(x).to(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(O.e4m3_round(x), want)
    # values past the largest code saturate (torch would give NaN there)
    np.testing.assert_array_equal(O.e4m3_round(np.array([460.0, -1e4], np.float32)), [448.0, -448.0])
