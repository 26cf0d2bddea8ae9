"""CPU oracle for the MaxSim hot path -- TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's own CPU definitions (roipony/flash-maxsim
0.1.0). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
may use it, and only as the checker or the timed CPU baseline; the product
(flash_maxsim_b200) never imports it.

Parity pin: tests/golden/*.npz hold outputs of the reference itself (its
torch functions imported from the reference checkout by
tests/golden/make_golden.py); tests/test_oracle.py checks every function
here against them.
"""
from __future__ import annotations

import numpy as np

_DOC_CHUNK = 256  # documents per einsum chunk (bounds the [B, Lq, Ld] temporary)


def _f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)


def maxsim(Q, D, doc_lengths=None, doc_chunk: int = _DOC_CHUNK) -> np.ndarray:
    """maxsim_naive (flash_maxsim/flash_maxsim.py:294-301).

    S[b, q, l] = <Q[q], D[b, l]> in fp32; positions l >= doc_lengths[b] are
    -inf; score[b] = sum_q max_l S[b, q, l].  Q: [Lq, d], D: [B, Ld, d].
    Documents are processed in chunks; every per-document result is
    independent of the chunking.
    """
    Q = _f32(Q)
    D = _f32(D)
    B, Ld, _ = D.shape
    out = np.empty(B, dtype=np.float32)
    pos = np.arange(Ld)
    for b0 in range(0, B, doc_chunk):
        Dc = D[b0:b0 + doc_chunk]
        S = np.matmul(Dc, Q.T)  # [b, Ld, Lq]
        if doc_lengths is not None:
            lens = np.asarray(doc_lengths)[b0:b0 + doc_chunk]
            S = np.where((pos[None, :] >= lens[:, None])[:, :, None], np.float32(-np.inf), S)
        out[b0:b0 + Dc.shape[0]] = S.max(axis=1).sum(axis=1, dtype=np.float32)
    return out


def maxsim_batched(Q, D, doc_lengths=None, shared_docs: bool = True) -> np.ndarray:
    """flash_maxsim_batched semantics (flash_maxsim/flash_maxsim.py:233-250)
    computed as one maxsim per query (the reference's own oracle loop,
    benchmarks/bench.py:100-101).  Q: [Nq, Lq, d]; D: [B, Ld, d] shared or
    [Nq, B, Ld, d] per query; doc_lengths: [B] or [Nq * B]."""
    Q = _f32(Q)
    Nq = Q.shape[0]
    if shared_docs:
        return np.stack([maxsim(Q[n], D, doc_lengths) for n in range(Nq)])
    B = D.shape[1]
    lens = None if doc_lengths is None else np.asarray(doc_lengths).reshape(Nq, B)
    return np.stack([maxsim(Q[n], D[n], None if lens is None else lens[n]) for n in range(Nq)])


def maxsim_argmax(Q, D, doc_lengths=None, doc_chunk: int = _DOC_CHUNK):
    """Scores plus the first index of every row maximum (the reference's
    forward with save_argmax, flash_maxsim/flash_maxsim.py:131-144: strict
    '>' across tiles, first occurrence inside a tile).  Also returns the gap
    between the largest and second-largest entry of each row (for tie-aware
    gradient checks).  Q: [Lq, d], D: [B, Ld, d]."""
    Q = _f32(Q)
    D = _f32(D)
    B, Ld, _ = D.shape
    Lq = Q.shape[0]
    scores = np.empty(B, dtype=np.float32)
    am = np.empty((B, Lq), dtype=np.int32)
    gap = np.empty((B, Lq), dtype=np.float32)
    pos = np.arange(Ld)
    for b0 in range(0, B, doc_chunk):
        Dc = D[b0:b0 + doc_chunk]
        S = np.matmul(Q[None], Dc.transpose(0, 2, 1))  # [b, Lq, Ld]
        if doc_lengths is not None:
            lens = np.asarray(doc_lengths)[b0:b0 + doc_chunk]
            S = np.where((pos[None, :] >= lens[:, None])[:, None, :], np.float32(-np.inf), S)
        n = Dc.shape[0]
        scores[b0:b0 + n] = S.max(axis=2).sum(axis=1, dtype=np.float32)
        am[b0:b0 + n] = S.argmax(axis=2)
        if Ld > 1:
            part = np.partition(S, Ld - 2, axis=2)
            gap[b0:b0 + n] = part[:, :, Ld - 1] - part[:, :, Ld - 2]
        else:
            gap[b0:b0 + n] = np.inf
    return scores, am, gap


def maxsim_grads(Q, D, argmax, grad_scores):
    """Closed-form MaxSim gradients for given argmax indices, in float64
    (the math of _maxsim_bwd_dQ_kernel / _maxsim_bwd_dD_kernel,
    flash_maxsim/flash_maxsim.py:153-188):
        dQ[n, q] = sum_b g[n, b] D[b, a[n, b, q]]
        dD[b, t] = sum_{(n, q): a[n, b, q] = t} g[n, b] Q[n, q]
    Q: [Nq, Lq, d], D: [B, Ld, d], argmax: [Nq, B, Lq] (-1 = no token),
    grad_scores: [Nq, B]."""
    Q = np.asarray(Q, dtype=np.float64)
    D = np.asarray(D, dtype=np.float64)
    am = np.asarray(argmax)
    g = np.asarray(grad_scores, dtype=np.float64)
    Nq, Lq, d = Q.shape
    B, Ld, _ = D.shape
    dQ = np.zeros_like(Q)
    dD = np.zeros_like(D)
    bidx = np.arange(B)
    for n in range(Nq):
        for q in range(Lq):
            a = am[n, :, q]
            ok = a >= 0
            rows = D[bidx[ok], a[ok]]  # [nb, d]
            dQ[n, q] = (g[n, ok][:, None] * rows).sum(axis=0)
            np.add.at(dD, (bidx[ok], a[ok]), g[n, ok][:, None] * Q[n, q][None, :])
    return dQ, dD


def quantize_int8(D):
    """quantize_int8 (flash_maxsim/flash_maxsim_quant.py:11-28), in numpy fp32:
    min/max over d, scale = max((max - min) / 255, 1e-8),
    u = clip(round_half_even((x - min) / scale), 0, 255) as uint8;
    scale and min returned as fp16 [B, Ld, 1]."""
    Df = np.asarray(D).astype(np.float32)
    mn = Df.min(axis=-1, keepdims=True)
    mx = Df.max(axis=-1, keepdims=True)
    scale = (mx - mn) / np.float32(255.0)
    scale = np.maximum(scale, np.float32(1e-8)).astype(np.float32)
    u = np.clip(np.round((Df - mn) / scale), 0, 255).astype(np.uint8)
    return u, scale.astype(np.float16), mn.astype(np.float16)


def dequantize_int8(u8, scales, mins) -> np.ndarray:
    """dequantize_int8 (flash_maxsim/flash_maxsim_quant.py:31-33): u*s + m in fp32."""
    return (np.asarray(u8).astype(np.float32) * np.asarray(scales).astype(np.float32)
            + np.asarray(mins).astype(np.float32))


def l2_normalize_rows(x) -> np.ndarray:
    """Rows divided by max(||x||_2, 1e-12) (torch.nn.functional.normalize's
    rule) with the norm summed in the library's fixed order: lane
    l = 0..LPR-1 of a row sums x*x over its elements k = (s * LPR + l) * 8 + j
    (s, then j ascending; fp32, rounded after every operation), then the
    lanes are combined by an xor butterfly (offsets LPR/2, ..., 1); LPR = 8
    for d <= 64, 16 for d <= 128, else 32 (both quantisers)."""
    x = np.asarray(x, dtype=np.float32)
    d = x.shape[-1]
    return _l2_normalize_rows(x, 8 if d <= 64 else (16 if d <= 128 else 32))


def _l2_normalize_rows(x, lpr: int) -> np.ndarray:
    d = x.shape[-1]
    flat = x.reshape(-1, d)
    lanes = []
    for l in range(lpr):
        acc = np.zeros(flat.shape[0], dtype=np.float32)
        s = 0
        while (s * lpr + l) * 8 < d:
            for j in range(8):
                k = (s * lpr + l) * 8 + j
                if k < d:
                    acc = (acc + (flat[:, k] * flat[:, k]).astype(np.float32)).astype(np.float32)
            s += 1
        lanes.append(acc)
    o = lpr // 2
    while o > 0:
        lanes = [(lanes[i] + lanes[i ^ o]).astype(np.float32) for i in range(lpr)]
        o //= 2
    den = np.maximum(np.sqrt(lanes[0]).astype(np.float32), np.float32(1e-12))
    return (flat / den[:, None]).astype(np.float32).reshape(x.shape)


def normalize_quantize_int8(D):
    """Index-time INT8: quantize_int8 of the L2-normalised rows."""
    return quantize_int8(l2_normalize_rows(D))


def normalize_quantize_fp8(D):
    """Index-time FP8: quantize_fp8 of the L2-normalised rows."""
    return quantize_fp8(l2_normalize_rows(D))


def e4m3_round(x) -> np.ndarray:
    """Round fp32 values to the nearest e4m3 (fn variant: 4 exponent bits,
    bias 7, 3 mantissa bits, subnormal step 2**-9, largest finite 448, no
    infinities), ties to even, saturating at +-448; returned as fp32."""
    x = np.asarray(x, dtype=np.float32)
    ax = np.abs(x).astype(np.float64)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(ax > 0, ax, 1.0)))
    e = np.maximum(e, -6.0)  # below the smallest normal 2**-6 the step is fixed
    step = np.exp2(e - 3.0)
    q = np.rint(ax / step) * step  # rint: ties to even
    q = np.minimum(q, 448.0)
    return (np.sign(x) * q).astype(np.float32)


def quantize_fp8(D):
    """Per-token e4m3 quantisation (the library's FP8 document format):
    scale = max|x| / 448 in fp32 (1 for an all-zero token),
    code = e4m3(x / scale). Returns (e4m3 values as fp32 [B, Ld, d],
    scales fp32 [B, Ld, 1])."""
    Df = np.asarray(D).astype(np.float32)
    amax = np.abs(Df).max(axis=-1, keepdims=True)
    scale = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
    return e4m3_round(Df / scale), scale


def dequantize_fp8(codes_f32, scales) -> np.ndarray:
    """e4m3 value * scale in fp32."""
    return np.asarray(codes_f32, dtype=np.float32) * np.asarray(scales, dtype=np.float32)


def maxsim_sparse(Q, D, indices, doc_lengths=None) -> np.ndarray:
    """maxsim_sparse_naive (flash_maxsim/flash_maxsim_sparse.py:143-157), plus
    the length mask the sparse kernel applies (:60-80):
    score[b] = sum_k max_{l < len_b} <Q[indices[b, k]], D[b, l]>."""
    Q = _f32(Q)
    D = _f32(D)
    idx = np.asarray(indices).astype(np.int64)
    B, Ld, _ = D.shape
    out = np.empty(B, dtype=np.float32)
    pos = np.arange(Ld)
    for b in range(B):
        S = D[b] @ Q[idx[b]].T  # [Ld, K]
        if doc_lengths is not None:
            S = np.where((pos >= int(np.asarray(doc_lengths)[b]))[:, None], np.float32(-np.inf), S)
        out[b] = S.max(axis=0).sum(dtype=np.float32)
    return out


def seeded_inputs(seed: int, *shapes, dtype=np.float16):
    """Seeded N(0, 1) tensors with every last-axis row L2-normalised (the
    input distribution of every BASELINE configuration), rounded to fp16."""
    rng = np.random.default_rng(seed)
    out = []
    for shp in shapes:
        x = rng.standard_normal(shp, dtype=np.float32)
        x /= np.maximum(np.linalg.norm(x, axis=-1, keepdims=True), np.float32(1e-12))
        out.append(x.astype(dtype))
    return out
