"""Index-time quantisation fused with L2 normalisation: the GPU result must
equal, bit for bit, the oracle's quantize_int8 / quantize_fp8 of rows
normalised in the library's fixed summation order, and stay within one code
of quantising torch's own F.normalize output."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import maxsim_oracle as O

pytestmark = pytest.mark.gpu


def raw_embeddings(d, dtype, seed=0):
    x = np.random.default_rng(seed).standard_normal((60, 37, d)).astype(np.float32) * 3.0
    x[0, 0] = 0.0  # an all-zero row (norm clamped to 1e-12)
    return torch.from_numpy(x).to(dtype)


@pytest.mark.parametrize("d", [64, 96, 128, 256, 512])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
def test_normalize_quantize_int8_bit_exact(cuda, d, dtype):
    import flash_maxsim_b200 as fm
    x = raw_embeddings(d, dtype)
    u8, sc, mn = fm.quantize_int8(x.to(cuda), normalize=True)
    wu, ws, wm = O.normalize_quantize_int8(x.float().numpy())
    np.testing.assert_array_equal(u8.cpu().numpy(), wu)
    np.testing.assert_array_equal(sc.cpu().numpy(), ws)
    np.testing.assert_array_equal(mn.cpu().numpy(), wm)
    # against torch's normalize (another summation order): codes within one step
    u2, _, _ = fm.quantize_int8(F.normalize(x.to(cuda).float(), dim=-1))
    assert (u8.int() - u2.int()).abs().max().item() <= 1


@pytest.mark.parametrize("d", [64, 128, 256, 2048])
@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_normalize_quantize_fp8_bit_exact(cuda, d, dtype):
    import flash_maxsim_b200 as fm
    x = raw_embeddings(d, dtype, seed=1)
    codes, sc = fm.quantize_fp8(x.to(cuda), normalize=True)
    wv, ws = O.normalize_quantize_fp8(x.float().numpy())
    np.testing.assert_array_equal(sc.cpu().numpy(), ws)
    np.testing.assert_array_equal(codes.cpu().view(torch.float8_e4m3fn).float().numpy(), wv)


def test_indexed_corpus_scores(cuda):
    # encode -> normalise+quantise in one pass -> score: matches scoring the
    # normalised fp32 embeddings within the quantisation error
    import flash_maxsim_b200 as fm
    emb = raw_embeddings(128, torch.float16, seed=2).to(cuda)
    q = F.normalize(torch.randn(32, 128, device=cuda), dim=-1).half()
    u8, sc, mn = fm.quantize_int8(emb, normalize=True)
    s8 = fm.flash_maxsim_int8(q, u8, sc, mn)
    ref = fm.maxsim_naive(q.float(), F.normalize(emb.float(), dim=-1))
    assert (s8 - ref).abs().max().item() < 0.1


@pytest.mark.parametrize("fmt", ["fp16", "int8", "fp8"])
def test_build_and_load_sharded_corpus(cuda, tmp_path, fmt):
    # encoder batches -> corpus files -> two ranks' shards on the GPU -> scores
    # equal to scoring the whole corpus at once
    import flash_maxsim_b200 as fm
    from flash_maxsim_b200 import corpus
    B, Ld, d = 300, 64, 128
    emb = torch.randn(B, Ld, d, generator=torch.Generator().manual_seed(3)).half()
    lens = torch.randint(1, Ld + 1, (B,), generator=torch.Generator().manual_seed(4), dtype=torch.int32)
    batches = [(emb[i:i + 70], lens[i:i + 70]) for i in range(0, B, 70)]
    corpus.build_corpus(tmp_path, batches, fmt, B, Ld, d)
    q = F.normalize(torch.randn(32, d, device=cuda), dim=-1).half()
    whole = corpus.score_shard(q, corpus.load_shard(tmp_path, 0, 1, device=cuda, chunk_bytes=1 << 16))
    parts = [corpus.score_shard(q, corpus.load_shard(tmp_path, r, 2, device=cuda, chunk_bytes=1 << 16))
             for r in range(2)]
    assert torch.equal(torch.cat(parts), whole)
    # the stored documents are the normalised (and quantised) embeddings
    normed = F.normalize(emb.float(), dim=-1).to(cuda)
    ref = fm.maxsim_naive(q.float(), normed, lens.to(cuda))
    tol = {"fp16": 1e-2, "int8": 0.1, "fp8": 0.2}[fmt]
    assert (whole - ref).abs().max().item() < tol
